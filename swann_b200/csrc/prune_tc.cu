// prune_tc.cu -- robust_prune's pair distances on the tensor cores, with the
// decisions of the dimension-ordered fmaf prune, bit for bit.
//
// Replaces robust_prune (swann/build.py:48-91) for the build's two prune
// passes.  The prune keeps candidate i of node u unless an already-kept j has
// alpha * pair(j, i) <= d(u, i); pair() comes from the Gram matrix of the
// node's (up to 128) candidates: 1 - <x_i, x_j> (ip), or (|x_i|^2 -
// 2<x_i, x_j>) + |x_j|^2 clamped at 0 (l2).  The contract of this library
// (and of its oracle) is that every <x_i, x_j> is one fmaf chain in dimension
// order; build.cu's prune_kernel forms all 128 x 128 of them on CUDA cores.
//
// Here one CTA per node forms the Gram matrix with tcgen05.mma into TMEM
// (kind::f16 for fp16-valued rows, whose products are exact; 3xTF32 --
// hi*hi + hi*lo + lo*hi -- otherwise), reads it back with tcgen05.ld, and
// decides every pair (i, j) from it whose detour test clears the threshold by
// more than a rigorous bound on the gap between the tensor-core value and the
// fmaf chain's: such a decision is the fmaf prune's.  The few pairs inside
// the bound are recomputed with the fmaf chain itself, spread over the CTA's
// threads.  The violation sets are then folded by the sequential keep rule as
// 128-bit masks.  Same output as prune_kernel, for every input.
//
// The bound.  For rows x, y of d elements, S = |x| |y| >= sum |x_k y_k|:
//   fmaf chain:        |g_f - <x,y>| <= d u S                 (u = 2^-24)
//   kind::f16 MMA:     products exact; each K = 16 step adds 17 terms whose
//                      bits below the largest one's ulp may be truncated:
//                      |g_tc - <x,y>| <= 68 u S per step, d / 16 steps
//   3xTF32:            the dropped lo*lo and the tf32 rounding of lo add
//                      3 * 2^-22 S; three MMA chains of d / 8 steps, 36 u S each
// and the expressions' own roundings (a few u of their operands' magnitudes).
// The host doubles the sum (gram_err); a generous bound only costs recomputes.
//
// Every mbarrier wait is bounded: a wait that runs out writes SWB_ERR_TIMEOUT
// to the status word, drains the CTA's copies, frees its TMEM and returns.

#include <cstring>

#include "abi_util.h"
#include "common.cuh"
#include "tcgen05.cuh"

namespace swb {
namespace prune_tc {

constexpr int CP = 128;                  // candidates per node, padded: M = N = 128
constexpr int NT = 128;                  // threads: one per Gram row
constexpr int GS = CP + 1;               // Gram row stride in floats (conflict-free rows)
constexpr int GRAM_BYTES = CP * GS * 4;
constexpr int LIST_CAP = 2048;           // pairs queued for the exact recompute

enum Mode { MODE_F16 = 0, MODE_TF32X3 = 1 };

template <int MODE>
struct Cfg;
template <>
struct Cfg<MODE_F16> {
    static constexpr int KC = 64;        // elements of K per stage (128 bytes a row)
    static constexpr int ESZ = 2;
    static constexpr int NOPS = 1;
    static constexpr int STAGES = 6;     // 96 KB: two CTAs an SM still fit
    static constexpr uint32_t FMT = 0;   // F16
};
template <>
struct Cfg<MODE_TF32X3> {
    static constexpr int KC = 32;
    static constexpr int ESZ = 4;
    static constexpr int NOPS = 2;       // hi and lo
    static constexpr int STAGES = 3;
    static constexpr uint32_t FMT = 2;   // TF32
};

template <int MODE>
struct Ly {
    static constexpr int OP = CP * 128;                       // one operand: 128 rows x 128 bytes
    static constexpr int STAGE = Cfg<MODE>::NOPS * OP;
    static constexpr int RING = Cfg<MODE>::STAGES * STAGE;
    static constexpr int UNION = RING > GRAM_BYTES ? RING : GRAM_BYTES;   // the Gram reuses the ring
    static constexpr int LIST = UNION;                        // uint32 [LIST_CAP]: i << 16 | j
    static constexpr int CID = LIST + LIST_CAP * 4;           // int [CP]
    static constexpr int DU = CID + CP * 4;                   // float [CP]
    static constexpr int NRM = DU + CP * 4;                   // float [CP]
    static constexpr int VIOL = NRM + CP * 4;                 // uint32 [CP][4]
    static constexpr int BARS = VIOL + CP * 16;               // uint64 [STAGES]
    static constexpr int MISC = BARS + Cfg<MODE>::STAGES * 8; // tmem base, list count
    static constexpr int TOTAL = MISC + 16;
    static constexpr int ALLOC = TOTAL + 1024;                // slack to align the ring to 1024 bytes
};

struct Params {
    const void* A;            // tensor-core operand rows [n, adim]: fp16, or the tf32 high parts
    const void* A_lo;         // the tf32 low parts (3xTF32), else null
    int adim;                 // a multiple of Cfg::KC (zero-padded)
    const float* X;           // fp32 rows [n, dim] for the exact recompute
    int dim;
    const float* norms;       // [n] squared norms, the same fmaf chain (swb_row_norms)
    int64_t n;
    const int32_t* cand;
    const float* cdist;
    int C, deg;
    float alpha;
    int metric;
    const int32_t* dpn;
    const uint8_t* protect;
    int32_t* out;
    float gram_err;           // bound per unit S on |g_tc - g_f|
    unsigned long long* recomputed;   // optional: pairs recomputed exactly
    int32_t* status;
};

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mma_f16(uint32_t dtm, uint64_t ad, uint64_t bd, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(dtm),
        "l"(ad), "l"(bd), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void mma_tf32(uint32_t dtm, uint64_t ad, uint64_t bd, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(dtm),
        "l"(ad), "l"(bd), "r"(idesc), "r"(acc)
        : "memory");
}

template <int MODE>
__host__ __device__ constexpr uint32_t idesc() {
    return (1u << 4)                                        // D in fp32
           | (Cfg<MODE>::FMT << 7) | (Cfg<MODE>::FMT << 10)   // A, B format
           | (uint32_t(CP >> 3) << 17)                      // N = 128
           | (uint32_t(CP >> 4) << 24);                     // M = 128
}

// Stage `kc` of the node's candidate rows into `stage`: for each operand, 128
// rows x 128 bytes in the 128B-swizzled K-major layout (16-byte chunk c of
// row r at r * 128 + ((c ^ (r & 7)) << 4)).  Thread t copies chunk t & 7 of
// rows t / 8 + 16 q; absent rows were zeroed once and are not touched.
template <int MODE>
__device__ __forceinline__ void load_stage(const Params& P, char* stage, const int* cid, int kc, int tid) {
    constexpr int KB = Cfg<MODE>::KC * Cfg<MODE>::ESZ;   // 128
    const int c = tid & 7;
#pragma unroll
    for (int op = 0; op < Cfg<MODE>::NOPS; ++op) {
        const char* src = reinterpret_cast<const char*>(op ? P.A_lo : P.A);
        char* dst = stage + op * Ly<MODE>::OP;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const int r = (tid >> 3) + 16 * q;
            const int v = cid[r];
            if (v >= 0)
                cp_async16(smem_u32(dst + r * 128 + ((c ^ (r & 7)) << 4)),
                           src + ((size_t)v * P.adim) * Cfg<MODE>::ESZ + (size_t)kc * KB + c * 16);
        }
    }
}

// <x_a, x_b> as one fmaf chain in dimension order (the oracle's and
// prune_kernel's arithmetic)
__device__ float fmaf_chain(const float* __restrict__ a, const float* __restrict__ b, int dim) {
    float acc = 0.f;
    if ((dim & 3) == 0 && ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 15) == 0) {
        const float4* a4 = reinterpret_cast<const float4*>(a);
        const float4* b4 = reinterpret_cast<const float4*>(b);
        for (int k = 0; k < dim / 4; ++k) {
            const float4 x = __ldg(a4 + k), y = __ldg(b4 + k);
            acc = fmaf(x.x, y.x, acc);
            acc = fmaf(x.y, y.y, acc);
            acc = fmaf(x.z, y.z, acc);
            acc = fmaf(x.w, y.w, acc);
        }
    } else {
        for (int k = 0; k < dim; ++k) acc = fmaf(__ldg(a + k), __ldg(b + k), acc);
    }
    return acc;
}

__device__ __forceinline__ float pair_dist(float g, float gii, float gjj, int metric) {
    if (metric == METRIC_IP) return __fsub_rn(1.f, g);
    float pr = __fadd_rn(__fsub_rn(gii, __fmul_rn(2.f, g)), gjj);
    return pr < 0.f ? 0.f : pr;
}

template <int MODE>
__global__ void __launch_bounds__(NT) prune_tc_kernel(const __grid_constant__ Params P) {
    extern __shared__ __align__(128) char smem_raw[];
    char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    using L = Ly<MODE>;
    constexpr int S = Cfg<MODE>::STAGES;
    char* ring = sm;
    float* gram = reinterpret_cast<float*>(sm);                 // after the products
    uint32_t* list = reinterpret_cast<uint32_t*>(sm + L::LIST);
    int* cid = reinterpret_cast<int*>(sm + L::CID);
    float* du = reinterpret_cast<float*>(sm + L::DU);
    float* nrm = reinterpret_cast<float*>(sm + L::NRM);
    uint32_t* viol = reinterpret_cast<uint32_t*>(sm + L::VIOL);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::BARS);
    uint32_t* tmem_ptr = reinterpret_cast<uint32_t*>(sm + L::MISC);
    int* nlist = reinterpret_cast<int*>(sm + L::MISC + 4);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t u = blockIdx.x;

    {
        const int i = tid;
        const int v = (i < P.C) ? P.cand[u * P.C + i] : -1;
        cid[i] = (v >= 0 && v < P.n) ? v : -1;   // an id outside the corpus is no candidate
        du[i] = (i < P.C) ? P.cdist[u * P.C + i] : 0.f;
        nrm[i] = (cid[i] >= 0) ? __ldg(P.norms + cid[i]) : 0.f;
        viol[4 * i] = viol[4 * i + 1] = viol[4 * i + 2] = viol[4 * i + 3] = 0u;
    }
    if (tid == 0) {
        for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
        *nlist = 0;
    }
    if (warp == 0) {
        tmem_alloc(tmem_ptr, CP);
        tmem_relinquish();
    }
    __syncthreads();
    // absent rows read as zeros in every stage
    {
        const int c = tid & 7;
        for (int s = 0; s < S; ++s)
#pragma unroll
            for (int op = 0; op < Cfg<MODE>::NOPS; ++op)
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const int r = (tid >> 3) + 16 * q;
                    if (cid[r] < 0)
                        *reinterpret_cast<uint4*>(ring + s * L::STAGE + op * L::OP + r * 128 + ((c ^ (r & 7)) << 4)) =
                            make_uint4(0u, 0u, 0u, 0u);
                }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_ptr;

    // -- the Gram matrix: stages of K through the ring, one MMA issuer --------
    const int nk = P.adim / Cfg<MODE>::KC;
    for (int s = 0; s < S - 1; ++s) {
        if (s < nk) load_stage<MODE>(P, ring + s * L::STAGE, cid, s, tid);
        cp_async_commit();
    }
    bool aborted = false;
    for (int kc = 0; kc < nk && !aborted; ++kc) {
        cp_async_wait<S - 2>();      // this thread's copies of stage kc have landed
        fence_proxy_async_smem();    // ... and are visible to the tensor core
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            const char* st = ring + (kc % S) * L::STAGE;
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {   // 4 MMAs of 32 bytes of K each
                const uint32_t acc = (kc | ks) ? 1u : 0u;
                const uint64_t hi = smem_desc(st + 32 * ks);
                if constexpr (MODE == MODE_F16) {
                    mma_f16(tmem, hi, hi, idesc<MODE>(), acc);
                } else {
                    const uint64_t lo = smem_desc(st + L::OP + 32 * ks);
                    mma_tf32(tmem, hi, hi, idesc<MODE>(), acc);
                    mma_tf32(tmem, hi, lo, idesc<MODE>(), 1u);
                    mma_tf32(tmem, lo, hi, idesc<MODE>(), 1u);
                }
            }
            umma_commit(&bars[kc % S]);
        }
        // the stage chunk kc - 1 used is refilled with chunk kc + S - 1 once
        // that chunk's MMAs are done; every thread waits, and the outcome is
        // voted on so that all threads leave the loop together
        const int nxt = kc + S - 1;
        bool ok = true;
        if (nxt < nk && kc >= 1) ok = mbar_wait_sleep(&bars[(kc - 1) % S], ((kc - 1) / S) & 1);
        aborted = __syncthreads_or(!ok) != 0;
        if (!aborted && nxt < nk) load_stage<MODE>(P, ring + (nxt % S) * L::STAGE, cid, nxt, tid);
        cp_async_commit();
    }
    if (!aborted) {   // the last commit covers every MMA
        const bool ok = mbar_wait_sleep(&bars[(nk - 1) % S], ((nk - 1) / S) & 1);
        aborted = __syncthreads_or(!ok) != 0;
    }
    cp_async_wait<0>();
    tc_fence_before();
    __syncthreads();
    if (!aborted) {
        // -- TMEM -> shared memory: thread t holds Gram row t (its TMEM lane)
        tc_fence_after();
        const int t = tid;
#pragma unroll 1
        for (int ch = 0; ch < CP / 32; ++ch) {
            float v[32];
            __syncwarp();
            tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + ch * 32, v);
#pragma unroll
            for (int x = 0; x < 32; ++x) gram[t * GS + ch * 32 + x] = v[x];
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, CP);   // no MMA or tcgen05.ld is in flight any more
    if (aborted) {
        if (tid == 0 && P.status) atomicExch(P.status, ERR_TIMEOUT);
        return;
    }

    // -- violation sets: bit j of row i when alpha * pair(j, i) <= d(u, i) -----
    {
        const int i = tid;
        if (cid[i] >= 0) {
            const float gii = nrm[i], di = du[i];
            const float si = sqrtf(gii);
            uint32_t vm[4] = {0u, 0u, 0u, 0u};
            for (int j = 0; j < i; ++j) {
                if (cid[j] < 0) continue;
                const float g = gram[i * GS + j];
                const float gjj = nrm[j];
                const float a = __fmul_rn(P.alpha, pair_dist(g, gii, gjj, P.metric));
                const float dg = P.gram_err * si * sqrtf(gjj);   // |g_tc - g_f| <= dg
                const float ex = (P.metric == METRIC_IP) ? (dg + 1.2e-7f * (1.f + fabsf(g)))
                                                          : (2.f * dg + 2.4e-7f * (gii + 2.f * fabsf(g) + gjj));
                const float tol = P.alpha * ex + 2.4e-7f * (fabsf(di) + fabsf(a));
                // a threshold that is not finite (the reverse pass's empty
                // slots carry +inf) is decided by any finite pair distance alike
                if (!isfinite(di) || fabsf(a - di) > tol) {
                    if (a <= di) vm[j >> 5] |= 1u << (j & 31);
                } else {
                    const int slot = atomicAdd(nlist, 1);
                    if (slot < LIST_CAP) {
                        list[slot] = ((uint32_t)i << 16) | (uint32_t)j;
                    } else {   // the queue is full: this thread recomputes the pair itself
                        const float gf = fmaf_chain(P.X + (size_t)cid[i] * P.dim, P.X + (size_t)cid[j] * P.dim, P.dim);
                        if (__fmul_rn(P.alpha, pair_dist(gf, gii, gjj, P.metric)) <= di) vm[j >> 5] |= 1u << (j & 31);
                    }
                }
            }
#pragma unroll
            for (int w = 0; w < 4; ++w) atomicOr(&viol[4 * i + w], vm[w]);
        }
    }
    __syncthreads();
    // -- the queued pairs with the fmaf chain, spread over the threads --------
    const int nq = *nlist < LIST_CAP ? *nlist : LIST_CAP;
    for (int e = tid; e < nq; e += NT) {
        const int i = (int)(list[e] >> 16), j = (int)(list[e] & 0xFFFFu);
        const float gf = fmaf_chain(P.X + (size_t)cid[i] * P.dim, P.X + (size_t)cid[j] * P.dim, P.dim);
        if (__fmul_rn(P.alpha, pair_dist(gf, nrm[i], nrm[j], P.metric)) <= du[i])
            atomicOr(&viol[4 * i + (j >> 5)], 1u << (j & 31));
    }
    if (tid == 0 && P.recomputed && *nlist > 0) atomicAdd(P.recomputed, (unsigned long long)*nlist);
    __syncthreads();

    // -- the keep rule (swann/build.py:48-91), violation sets as masks ---------
    if (warp == 0) {
        const int cap = P.dpn ? min(P.dpn[u], P.deg) : P.deg;
        const uint8_t* prot = P.protect ? P.protect + u * P.C : nullptr;
        uint32_t kept[4] = {0u, 0u, 0u, 0u};
        int nkeep = 0;
        for (int i = 0; i < P.C && nkeep < cap; ++i) {
            if (cid[i] < 0) continue;
            bool v = ((viol[4 * i] & kept[0]) | (viol[4 * i + 1] & kept[1]) | (viol[4 * i + 2] & kept[2]) |
                      (viol[4 * i + 3] & kept[3])) != 0u;
            if (prot && prot[i]) v = false;   // a protected pair survives the detour test
            if (!v) {
                kept[i >> 5] |= 1u << (i & 31);
                ++nkeep;
            }
        }
        // compact in candidate order
        int w = 0;
        for (int b = 0; b < P.C; b += 32) {
            const int i = b + lane;
            const bool k = i < P.C && ((kept[b >> 5] >> lane) & 1u);
            const unsigned m = __ballot_sync(FULL, k);
            if (k) {
                const int p = w + __popc(m & lanemask_lt());
                if (p < P.deg) P.out[u * P.deg + p] = cid[i];
            }
            w += __popc(m);
        }
        for (int p = w + lane; p < P.deg; p += 32) P.out[u * P.deg + p] = -1;
    }
}

}  // namespace prune_tc
}  // namespace swb

// ===========================================================================
// host side

using namespace swb;

namespace swb {
namespace prune_tc {

// bound per unit |x||y| on |g_tc - g_f| for rows of `dim` elements (operands
// padded to adim), doubled for margin
float gram_err_bound(int mode, int dim, int adim) {
    const double u = 1.0 / (1 << 24);
    double b = dim * u;                                           // the fmaf chain
    if (mode == MODE_F16) b += 68.0 * u * ((adim + 15) / 16);    // K = 16 steps, 17 terms each
    else b += 3.0 * 4.0 * u + 3.0 * 36.0 * u * ((adim + 7) / 8);   // 3xTF32: split error, 3 chains of K = 8
    return (float)(2.0 * b);
}

int launch(const Params& P0, int mode, int64_t rows, cudaStream_t st) {
    Params P = P0;
    const char* scale = std::getenv("SWB_PRUNE_TOL_SCALE");   // tests: force the exact path (inf) or probe it
    P.gram_err = gram_err_bound(mode, P.dim, P.adim) * (scale && *scale ? (float)std::atof(scale) : 1.f);
    const int smem = mode == MODE_F16 ? Ly<MODE_F16>::ALLOC : Ly<MODE_TF32X3>::ALLOC;
    if (smem > abi::max_smem_optin()) return abi::fail(SWB_ERR_SMEM, "tensor-core prune needs %d B of shared memory", smem);
    cudaError_t e;
    if (mode == MODE_F16) {
        e = cudaFuncSetAttribute(prune_tc_kernel<MODE_F16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return abi::cuda_fail(e, "cudaFuncSetAttribute(prune_tc)");
        prune_tc_kernel<MODE_F16><<<(unsigned)rows, NT, smem, st>>>(P);
    } else {
        e = cudaFuncSetAttribute(prune_tc_kernel<MODE_TF32X3>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return abi::cuda_fail(e, "cudaFuncSetAttribute(prune_tc)");
        prune_tc_kernel<MODE_TF32X3><<<(unsigned)rows, NT, smem, st>>>(P);
    }
    return abi::cuda_check("tensor-core prune launch");
}

}  // namespace prune_tc
}  // namespace swb

// Shared by swb_prune_tc and the reverse pass: checks and launches.
int swb_prune_tc_launch(const float* X, const void* A, const void* A_lo, int a_dtype, int adim, const float* norms,
                        int64_t n, int dim, const int32_t* cand, const float* cdist, int64_t rows, int C, int deg,
                        float alpha, int metric, const int32_t* deg_per_node, const uint8_t* protect, int32_t* out,
                        unsigned long long* recomputed, int32_t* status, cudaStream_t st) {
    using namespace swb::prune_tc;
    if (!X || !A || !norms || !cand || !cdist || !out) return abi::fail(SWB_ERR_ARG, "null buffer");
    if (C < 1 || C > CP) return abi::fail(SWB_ERR_ARG, "candidates per node must be 1..%d", CP);
    if (deg < 1) return abi::fail(SWB_ERR_ARG, "degree must be positive");
    if (a_dtype != SWB_F16 && a_dtype != SWB_F32) return abi::fail(SWB_ERR_ARG, "operand rows must be f16 or f32");
    const int mode = a_dtype == SWB_F16 ? MODE_F16 : MODE_TF32X3;
    if (mode == MODE_TF32X3 && !A_lo) return abi::fail(SWB_ERR_ARG, "3xTF32 needs the low parts");
    const int kc = mode == MODE_F16 ? Cfg<MODE_F16>::KC : Cfg<MODE_TF32X3>::KC;
    if (adim < dim || adim % kc) return abi::fail(SWB_ERR_ARG, "operand rows must be padded to a multiple of %d", kc);
    if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(A_lo)) % 16)
        return abi::fail(SWB_ERR_ARG, "operand rows must be 16-byte aligned");
    if (rows <= 0) return SWB_OK;
    Params P;
    std::memset(&P, 0, sizeof(P));
    P.A = A; P.A_lo = A_lo; P.adim = adim; P.X = X; P.dim = dim; P.norms = norms; P.n = n;
    P.cand = cand; P.cdist = cdist; P.C = C; P.deg = deg; P.alpha = alpha; P.metric = metric;
    P.dpn = deg_per_node; P.protect = protect; P.out = out; P.recomputed = recomputed; P.status = status;
    return launch(P, mode, rows, st);
}

extern "C" int swb_prune_tc(const float* X, const void* A, const void* A_lo, int a_dtype, int adim,
                            const float* norms, int64_t n, int dim, const int32_t* cand, const float* cdist,
                            int64_t rows, int C, int deg, float alpha, int metric, const int32_t* deg_per_node,
                            const uint8_t* protect, int32_t* out, unsigned long long* recomputed, int32_t* status,
                            void* stream) {
    return swb_prune_tc_launch(X, A, A_lo, a_dtype, adim, norms, n, dim, cand, cdist, rows, C, deg, alpha, metric,
                               deg_per_node, protect, out, recomputed, status, (cudaStream_t)stream);
}
