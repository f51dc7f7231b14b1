// build.cu -- graph construction kernels for sm_100a.
//
// Replaces swann/build.py's three stages:
//   knn_candidates  (build.py:30-43)   per-row top-C selection (this file) over
//                                       dot-product tiles (sweep_mma.cu / a GEMM)
//   robust_prune    (build.py:48-91)   prune_kernel
//   add_reverse     (build.py:96-150)  stable radix sort by target + merge_row_kernel
//                                       + prune_kernel
//
// Arithmetic contract (the oracle, oracle/swann_oracle.c, computes the same):
// every dot product of the prune and of the reverse pass is accumulated by one
// thread in dimension order with fmaf, so the pruned graph is reproducible bit
// for bit from the same candidates.  The reference leaves that order to BLAS.

#include <cub/device/device_radix_sort.cuh>

#include "abi_util.h"
#include "common.cuh"

namespace swb {

constexpr float SELF_DIST = 3.4e38f;   // build.py:41 marks the diagonal so

// ---------------------------------------------------------------------------
// squared row norms, sequential fmaf (one thread per row)

template <typename XT>
__global__ void norms_kernel(const XT* __restrict__ X, int64_t n, int dim, float* __restrict__ out) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n) return;
    const XT* row = X + r * dim;
    constexpr int V = VecN<XT>::N;
    float acc = 0.f;
    for (int k = 0; k < dim; k += V) {
        float x[V];
        widen16(row + k, x);
#pragma unroll
        for (int i = 0; i < V; ++i) acc = fmaf(x[i], x[i], acc);
    }
    out[r] = acc;
}

// ---------------------------------------------------------------------------
// top-C of one row: a warp keeps the C best (distance, id) sorted in shared
// memory, filters incoming values against the C-th, buffers the survivors and
// folds the buffer in with a merge when it fills.

struct TopC {
    float* bd;   // [C] best, sorted
    int* bi;
    float* nd;   // [C] merge output
    int* ni;
    float* ud;   // [UB] buffer
    int* ui;
    int C, count, nbuf;
    float thd;   // current C-th (INF while fewer than C)
    int thi;
};
constexpr int UB = 256;   // buffer entries per warp

__device__ void topc_init(TopC& t, char* base, int C, int lane) {
    t.bd = reinterpret_cast<float*>(base);
    t.bi = reinterpret_cast<int*>(t.bd + C);
    t.nd = reinterpret_cast<float*>(t.bi + C);
    t.ni = reinterpret_cast<int*>(t.nd + C);
    t.ud = reinterpret_cast<float*>(t.ni + C);
    t.ui = reinterpret_cast<int*>(t.ud + UB);
    t.C = C;
    t.count = 0;
    t.nbuf = 0;
    t.thd = __int_as_float(0x7f800000);
    t.thi = 0x7fffffff;
    for (int i = lane; i < C; i += 32) { t.bd[i] = __int_as_float(0x7f800000); t.bi[i] = 0x7fffffff; }
    __syncwarp();
}

__device__ __forceinline__ int topc_bytes(int C) { return C * 16 + UB * 8; }

// sort the buffer (padded to a power of two), merge with the best, keep C
__device__ void topc_flush(TopC& t, int lane) {
    if (t.nbuf == 0) return;
    int ms = 2;
    while (ms < t.nbuf) ms <<= 1;
    for (int i = t.nbuf + lane; i < ms; i += 32) { t.ud[i] = __int_as_float(0x7f800000); t.ui[i] = 0x7fffffff; }
    __syncwarp();
    for (int k = 2; k <= ms; k <<= 1)
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = lane; i < ms; i += 32) {
                const int x = i ^ j;
                if (x > i) {
                    const bool asc = (i & k) == 0;
                    const bool need = asc ? key_lt(t.ud[x], t.ui[x], t.ud[i], t.ui[i])
                                          : key_lt(t.ud[i], t.ui[i], t.ud[x], t.ui[x]);
                    if (need) {
                        const float a = t.ud[i]; t.ud[i] = t.ud[x]; t.ud[x] = a;
                        const int b = t.ui[i]; t.ui[i] = t.ui[x]; t.ui[x] = b;
                    }
                }
            }
            __syncwarp();
        }
    const int na = t.count, nb = t.nbuf;
    const int outn = min(t.C, na + nb);
    for (int o = lane; o < outn; o += 32) {
        int lo = max(0, o - nb), hi = min(o, na);
        while (lo < hi) {
            const int i = (lo + hi) >> 1, j = o - i;
            if (j > 0 && !key_lt(t.ud[j - 1], t.ui[j - 1], t.bd[i], t.bi[i])) lo = i + 1;
            else hi = i;
        }
        const int i = lo, j = o - i;
        const bool takeA = (j >= nb) || (i < na && key_lt(t.bd[i], t.bi[i], t.ud[j], t.ui[j]));
        t.nd[o] = takeA ? t.bd[i] : t.ud[j];
        t.ni[o] = takeA ? t.bi[i] : t.ui[j];
    }
    __syncwarp();
    for (int o = lane; o < outn; o += 32) { t.bd[o] = t.nd[o]; t.bi[o] = t.ni[o]; }
    __syncwarp();
    t.count = outn;
    t.nbuf = 0;
    if (t.count == t.C) { t.thd = t.bd[t.C - 1]; t.thi = t.bi[t.C - 1]; }
}

// offer one (d, id) per lane (valid = false to offer nothing)
__device__ __forceinline__ void topc_offer(TopC& t, float d, int id, bool valid, int lane) {
    const bool pass = valid && key_lt(d, id, t.thd, t.thi);
    const unsigned m = __ballot_sync(FULL, pass);
    if (!m) return;
    const int cnt = __popc(m);
    if (t.nbuf + cnt > UB) topc_flush(t, lane);
    const bool pass2 = valid && key_lt(d, id, t.thd, t.thi);   // the threshold may have tightened
    const unsigned m2 = __ballot_sync(FULL, pass2);
    if (pass2) {
        const int p = t.nbuf + __popc(m2 & lanemask_lt());
        t.ud[p] = d;
        t.ui[p] = id;
    }
    t.nbuf += __popc(m2);
    __syncwarp();
}

// Distances from a block of dot products.  dots[r * ld + j] = <x_{row0+r}, x_j>
// for j in [col0, col0 + ncols); the block is folded into the running top-C.
__device__ __forceinline__ float metric_dist(float dot, int metric, float an, float bn) {
    if (metric == METRIC_IP) return __fsub_rn(1.f, dot);
    const float v = __fadd_rn(__fsub_rn(bn, __fmul_rn(2.f, dot)), an);
    return v < 0.f ? 0.f : v;
}

__global__ void __launch_bounds__(256) topc_rows_kernel(const float* __restrict__ dots, int64_t rows, int64_t ld,
                                                       int64_t ncols, int64_t row0, int64_t col0,
                                                       const float* __restrict__ norms, int metric, int C,
                                                       int32_t* __restrict__ idx, float* __restrict__ dst,
                                                       int resume) {
    extern __shared__ __align__(128) char smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
    if (r >= rows) return;
    TopC t;
    topc_init(t, smem + (size_t)warp * topc_bytes(C), C, lane);
    if (resume) {
        // continue from the lists a previous column block left
        for (int i = lane; i < C; i += 32) {
            t.bd[i] = dst[r * C + i];
            t.bi[i] = idx[r * C + i];
        }
        __syncwarp();
        int valid = 0;
        for (int i = 0; i < C; ++i) valid += (t.bi[i] >= 0 && t.bi[i] != 0x7fffffff) ? 1 : 0;
        t.count = valid;
        if (t.count == C) { t.thd = t.bd[C - 1]; t.thi = t.bi[C - 1]; }
    }
    const int64_t grow = row0 + r;
    const float an = (metric == METRIC_L2) ? norms[grow] : 0.f;
    const float* drow = dots + r * ld;
    for (int64_t base = 0; base < ncols; base += 128) {
        const int64_t j0 = base + lane * 4;
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        if (j0 + 3 < ncols && (ld % 4) == 0) {
            const float4 f = __ldcs(reinterpret_cast<const float4*>(drow + j0));
            v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i)
                if (j0 + i < ncols) v[i] = __ldcs(drow + j0 + i);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int64_t j = col0 + j0 + i;
            const bool ok = (j0 + i) < ncols;
            float d = 0.f;
            if (ok) {
                d = metric_dist(v[i], metric, an, metric == METRIC_L2 ? __ldg(&norms[j]) : 0.f);
                if (j == grow) d = SELF_DIST;
            }
            topc_offer(t, d, (int)j, ok, lane);
        }
    }
    topc_flush(t, lane);
    for (int i = lane; i < C; i += 32) {
        const bool ok = i < t.count;
        idx[r * C + i] = ok ? t.bi[i] : -1;
        dst[r * C + i] = ok ? t.bd[i] : __int_as_float(0x7f800000);
    }
}

// ---------------------------------------------------------------------------
// prune: one block per node.  The Gram matrix of the node's (up to 128)
// candidates is built in shared memory, then one warp runs the sequential keep
// rule.  Every Gram entry is one thread's dimension-ordered fmaf chain, so the
// matrix is exactly symmetric and reproducible.
//
// Tiling (SIMT, fp32): the 128 x 128 matrix is split over a 16 x 16 thread
// grid, thread (ty, tx) owning rows {4ty..4ty+3, 64+4ty..64+4ty+3} and the same
// pattern of columns for tx, so each k step reads its operands as four 16-byte
// shared loads (conflict-free) for 64 fmaf.  The candidates' rows come in
// chunks of PR_KC dimensions, transposed into a k-major stage [PR_KC][128]
// (double-buffered through registers: the next chunk's global loads are in
// flight while the current one is multiplied).  The stage aliases the Gram
// array, which is written only after the last chunk.

constexpr int PR_THREADS = 256;
constexpr int PR_KC = 16;    // dimensions staged per chunk
constexpr int PR_CP = 128;   // candidates per node, padded
constexpr int PR_GRAM = PR_CP * PR_CP * 4;
constexpr int PR_SMEM = PR_GRAM + PR_CP * 4 + PR_CP * 4 + PR_CP;
static_assert(2 * PR_KC * PR_CP * 4 <= PR_GRAM, "the stage must fit in the Gram array");

// The next chunk of this thread's two (candidate, 4-dimension) pieces:
// candidate c = tid & 127, dimensions k0 + 4*kq .. k0 + 4*kq + 3 with
// kq = (tid >> 7) + 2s.  Dimensions at or past dim read as zero (VEC: dim is a
// multiple of 4, so a piece is all inside or all outside).
template <bool VEC>
__device__ __forceinline__ void prune_fetch(const float* __restrict__ row, int k0, int dim, int kq0, float4 (&pf)[2]) {
#pragma unroll
    for (int s = 0; s < 2; ++s) {
        const int k = k0 + 4 * (kq0 + 2 * s);
        if (VEC) {
            pf[s] = (row && k < dim) ? __ldg(reinterpret_cast<const float4*>(row + k)) : make_float4(0.f, 0.f, 0.f, 0.f);
        } else {
            pf[s].x = (row && k + 0 < dim) ? __ldg(row + k + 0) : 0.f;
            pf[s].y = (row && k + 1 < dim) ? __ldg(row + k + 1) : 0.f;
            pf[s].z = (row && k + 2 < dim) ? __ldg(row + k + 2) : 0.f;
            pf[s].w = (row && k + 3 < dim) ? __ldg(row + k + 3) : 0.f;
        }
    }
}

__device__ __forceinline__ void prune_put(float* stage, int c, int kq0, const float4 (&pf)[2]) {
#pragma unroll
    for (int s = 0; s < 2; ++s) {
        const int kk = 4 * (kq0 + 2 * s);
        stage[(kk + 0) * PR_CP + c] = pf[s].x;
        stage[(kk + 1) * PR_CP + c] = pf[s].y;
        stage[(kk + 2) * PR_CP + c] = pf[s].z;
        stage[(kk + 3) * PR_CP + c] = pf[s].w;
    }
}

template <bool VEC>
__global__ void __launch_bounds__(PR_THREADS, 2) prune_kernel(const float* __restrict__ X, int64_t n, int dim,
                                                             const int32_t* __restrict__ cand,
                                                             const float* __restrict__ cdist, int C, int deg,
                                                             float alpha, int metric,
                                                             const int32_t* __restrict__ dpn,
                                                             const uint8_t* __restrict__ protect,
                                                             int32_t* __restrict__ out) {
    extern __shared__ __align__(128) char smem[];
    float* gram = reinterpret_cast<float*>(smem);                  // [128][128]
    float* stage = gram;                                           // [2][PR_KC][128], during the products
    int* cid = reinterpret_cast<int*>(smem + PR_GRAM);             // [128]
    float* du = reinterpret_cast<float*>(cid + PR_CP);             // [128]
    uint8_t* kept = reinterpret_cast<uint8_t*>(du + PR_CP);        // [128]
    const int64_t u = blockIdx.x;
    const int tid = threadIdx.x;
    if (tid < PR_CP) {
        const int i = tid;
        const int v = (i < C) ? cand[u * C + i] : -1;
        cid[i] = (v < n) ? v : -1;   // an id outside the corpus is no candidate
        du[i] = (i < C) ? cdist[u * C + i] : 0.f;
        kept[i] = 0;
    }
    __syncthreads();
    const int ty = tid >> 4, tx = tid & 15;
    const int sc = tid & (PR_CP - 1), kq0 = tid >> 7;
    const float* row = cid[sc] >= 0 ? X + (size_t)cid[sc] * dim : nullptr;
    float acc[8][8];
#pragma unroll
    for (int a = 0; a < 8; ++a)
#pragma unroll
        for (int b = 0; b < 8; ++b) acc[a][b] = 0.f;
    float4 pf[2];
    prune_fetch<VEC>(row, 0, dim, kq0, pf);
    prune_put(stage, sc, kq0, pf);
    __syncthreads();
    int buf = 0;
    for (int k0 = 0; k0 < dim; k0 += PR_KC) {
        const bool more = k0 + PR_KC < dim;
        if (more) prune_fetch<VEC>(row, k0 + PR_KC, dim, kq0, pf);
        const float* st = stage + buf * PR_KC * PR_CP;
        const int kn = min(PR_KC, dim - k0);   // no products past dim: the chains end exactly there
#pragma unroll
        for (int kk = 0; kk < PR_KC; ++kk) {
            if (kk < kn) {
                const float4 a0 = *reinterpret_cast<const float4*>(st + kk * PR_CP + 4 * ty);
                const float4 a1 = *reinterpret_cast<const float4*>(st + kk * PR_CP + 64 + 4 * ty);
                const float4 b0 = *reinterpret_cast<const float4*>(st + kk * PR_CP + 4 * tx);
                const float4 b1 = *reinterpret_cast<const float4*>(st + kk * PR_CP + 64 + 4 * tx);
                const float ra[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                const float rb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
                for (int a = 0; a < 8; ++a)
#pragma unroll
                    for (int b = 0; b < 8; ++b) acc[a][b] = fmaf(ra[a], rb[b], acc[a][b]);
            }
        }
        if (more) prune_put(stage + (buf ^ 1) * PR_KC * PR_CP, sc, kq0, pf);
        buf ^= 1;
        __syncthreads();
    }
    // the stage is dead (the barrier above ends its last reads): write the Gram
#pragma unroll
    for (int a = 0; a < 8; ++a) {
        const int r = (a < 4) ? 4 * ty + a : 64 + 4 * ty + (a - 4);
        *reinterpret_cast<float4*>(gram + r * PR_CP + 4 * tx) = make_float4(acc[a][0], acc[a][1], acc[a][2], acc[a][3]);
        *reinterpret_cast<float4*>(gram + r * PR_CP + 64 + 4 * tx) =
            make_float4(acc[a][4], acc[a][5], acc[a][6], acc[a][7]);
    }
    __syncthreads();
    if (tid < 32) {
        // deg is the output width; a node's own cap is dpn[u] when per-node
        // degrees are given (robust_prune's deg_per_node, swann/build.py:48-91)
        const int lane = tid;
        const int cap = dpn ? min(dpn[u], deg) : deg;
        const uint8_t* prot = protect ? protect + u * C : nullptr;
        int nk = 0;
        for (int i = 0; i < C && nk < cap; ++i) {
            if (cid[i] < 0) continue;
            bool viol = false;
            const float gii = gram[i * PR_CP + i];
            for (int j = lane; j < i; j += 32) {
                if (!kept[j]) continue;
                const float g = gram[i * PR_CP + j];   // = gram[j][i]: the same chain
                float pr;
                if (metric == METRIC_IP) {
                    pr = __fsub_rn(1.f, g);
                } else {
                    pr = __fadd_rn(__fsub_rn(gii, __fmul_rn(2.f, g)), gram[j * PR_CP + j]);
                    if (pr < 0.f) pr = 0.f;
                }
                if (__fmul_rn(alpha, pr) <= du[i]) viol = true;
            }
            viol = __any_sync(FULL, viol);
            if (prot && prot[i]) viol = false;   // a protected pair survives the detour test
            if (!viol) {
                if (lane == 0) kept[i] = 1;
                ++nk;
            }
            __syncwarp();
        }
        // compact in candidate order
        int w = 0;
        for (int b = 0; b < C; b += 32) {
            const int i = b + lane;
            const bool k = i < C && kept[i];
            const unsigned m = __ballot_sync(FULL, k);
            if (k) {
                const int p = w + __popc(m & lanemask_lt());
                if (p < deg) out[u * deg + p] = cid[i];
            }
            w += __popc(m);
        }
        for (int p = w + lane; p < deg; p += 32) out[u * deg + p] = -1;
    }
}

// ---------------------------------------------------------------------------
// reverse pass

__global__ void edge_keys_kernel(const int32_t* __restrict__ G, int64_t total, int64_t n,
                                 int32_t* __restrict__ keys, int32_t* __restrict__ vals) {
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= total) return;
    const int t = G[e];
    keys[e] = (t >= 0 && t < n) ? t : 0x7fffffff;   // no-edge slots sort past every target
    vals[e] = (int32_t)e;                  // (source, slot) in row-major order
}

// starts[t] = first position of target t in the sorted keys (binary search)
__global__ void seg_starts_kernel(const int32_t* __restrict__ skeys, int64_t total, int64_t n,
                                  int64_t* __restrict__ starts) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t > n) return;
    int64_t lo = 0, hi = total;
    while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if ((int64_t)skeys[mid] < t) lo = mid + 1;
        else hi = mid;
    }
    starts[t] = lo;
}

// One block per target t: its own row plus the first max_in offers, self and
// duplicates removed (by id order), scored against x_t, ordered by distance
// (ties by id), the first `keepn` written as prune candidates.
constexpr int RV_THREADS = 128;

// <x_v, x_t>-style chains of one entry, in dimension order: xs is the row
// (fp32, or fp16 holding the same values), xt the target in shared memory.
// VEC: 16-byte loads (dim a multiple of the vector width, rows aligned).
template <typename XT, bool VEC>
__device__ __forceinline__ float entry_dist(const XT* __restrict__ xv, const float* __restrict__ xt, int dim,
                                            int metric) {
    float acc = 0.f;
    if (VEC) {
        constexpr int V = VecN<XT>::N;
        const uint4* p = reinterpret_cast<const uint4*>(xv);
#pragma unroll 4
        for (int c = 0; c < dim / V; ++c) {
            float x[V];
            widen_u4<XT>(__ldg(p + c), x);
#pragma unroll
            for (int e = 0; e < V; ++e) {
                if (metric == METRIC_IP) {
                    acc = fmaf(x[e], xt[c * V + e], acc);
                } else {
                    const float df = __fsub_rn(x[e], xt[c * V + e]);
                    acc = fmaf(df, df, acc);
                }
            }
        }
    } else {
        for (int k = 0; k < dim; ++k) {
            const float x = static_cast<float>(__ldg(&xv[k]));
            if (metric == METRIC_IP) {
                acc = fmaf(x, xt[k], acc);
            } else {
                const float df = __fsub_rn(x, xt[k]);
                acc = fmaf(df, df, acc);
            }
        }
    }
    return metric == METRIC_IP ? __fsub_rn(1.f, acc) : acc;
}

// XS: the element type the candidates' rows are read in (fp16 for an
// fp16-valued corpus: the same values, half the bytes), at row stride xs.
template <typename XS, bool VEC>
__global__ void __launch_bounds__(RV_THREADS) merge_row_kernel(const float* __restrict__ X, int dim,
                                                              const XS* __restrict__ Xs, int64_t xs,
                                                              const int32_t* __restrict__ G, int deg,
                                                              const int32_t* __restrict__ svals,
                                                              const int64_t* __restrict__ starts, int max_in,
                                                              int metric, int keepn, int64_t n, int64_t row0,
                                                              int32_t* __restrict__ cand,
                                                              float* __restrict__ cdist) {
    extern __shared__ __align__(128) char smem[];
    const int width = deg + max_in;
    int Wp = 2;
    while (Wp < width) Wp <<= 1;
    int* ids = reinterpret_cast<int*>(smem);           // [Wp]
    float* dd = reinterpret_cast<float*>(ids + Wp);    // [Wp]
    int* pos = reinterpret_cast<int*>(dd + Wp);        // [Wp]
    float* xt = reinterpret_cast<float*>(pos + Wp);    // [dim]
    const int64_t t = row0 + blockIdx.x;   // global row; outputs are row-local
    const int64_t tl = blockIdx.x;
    const int tid = threadIdx.x;
    const int64_t s0 = starts[t], s1 = starts[t + 1];
    const int64_t span = s1 - s0;
    const int nin = (int)(span < (int64_t)max_in ? span : (int64_t)max_in);
    constexpr int INVALID = 1 << 30;
    for (int i = tid; i < Wp; i += RV_THREADS) {
        int v = -1;
        if (i < deg) v = G[t * deg + i];
        else if (i < deg + nin) v = svals[s0 + (i - deg)] / deg;
        if (i >= width || v < 0 || v >= n || v == (int)t) v = INVALID;
        ids[i] = v;
    }
    for (int k = tid; k < dim; k += RV_THREADS) xt[k] = X[t * dim + k];
    __syncthreads();
    // sort ids ascending
    for (int k = 2; k <= Wp; k <<= 1)
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = tid; i < Wp; i += RV_THREADS) {
                const int x = i ^ j;
                if (x > i) {
                    const bool asc = (i & k) == 0;
                    const int a = ids[i], b = ids[x];
                    if (asc ? (b < a) : (a < b)) { ids[i] = b; ids[x] = a; }
                }
            }
            __syncthreads();
        }
    // mark repeats (against the sorted values, before any is replaced)
    int rep[(256 + RV_THREADS - 1) / RV_THREADS + 1];
    int nr = 0;
    for (int i = tid; i < Wp; i += RV_THREADS) rep[nr++] = (i > 0 && ids[i] == ids[i - 1]) ? 1 : 0;
    __syncthreads();
    nr = 0;
    for (int i = tid; i < Wp; i += RV_THREADS) {
        if (rep[nr++]) ids[i] = INVALID;
    }
    __syncthreads();
    // distances, one thread per entry, dimension order
    for (int i = tid; i < Wp; i += RV_THREADS) {
        const int v = ids[i];
        pos[i] = i;
        if (i >= width || v >= INVALID) {
            dd[i] = __int_as_float(0x7f800000);
            ids[i] = (i < width) ? 0 : 0x7fffffff;   // the reference scores no-entry slots as id 0, +inf
            continue;
        }
        dd[i] = entry_dist<XS, VEC>(Xs + (size_t)v * xs, xt, dim, metric);
    }
    __syncthreads();
    // order by (distance, position)
    for (int k = 2; k <= Wp; k <<= 1)
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = tid; i < Wp; i += RV_THREADS) {
                const int x = i ^ j;
                if (x > i) {
                    const bool asc = (i & k) == 0;
                    const bool xlt = key_lt(dd[x], pos[x], dd[i], pos[i]);
                    const bool ilt = key_lt(dd[i], pos[i], dd[x], pos[x]);
                    if (asc ? xlt : ilt) {
                        const float a = dd[i]; dd[i] = dd[x]; dd[x] = a;
                        const int b = ids[i]; ids[i] = ids[x]; ids[x] = b;
                        const int c = pos[i]; pos[i] = pos[x]; pos[x] = c;
                    }
                }
            }
            __syncthreads();
        }
    for (int i = tid; i < keepn; i += RV_THREADS) {
        cand[tl * keepn + i] = ids[i];
        cdist[tl * keepn + i] = dd[i];
    }
}

}  // namespace swb

// ===========================================================================
// host side

using namespace swb;

namespace {

uint64_t align256(uint64_t x) { return (x + 255) & ~uint64_t(255); }

size_t radix_temp_bytes(int64_t total) {
    size_t bytes = 0;
    cub::DeviceRadixSort::SortPairs(nullptr, bytes, (const int32_t*)nullptr, (int32_t*)nullptr,
                                    (const int32_t*)nullptr, (int32_t*)nullptr, (int)total);
    return bytes;
}

// n rows of candidates over a corpus of nx rows
template <bool VEC>
int launch_prune_t(const float* X, int64_t nx, int64_t n, int dim, const int32_t* cand, const float* cdist, int C,
                   int deg, float alpha, int metric, const int32_t* dpn, const uint8_t* protect, int32_t* out,
                   cudaStream_t st) {
    if (PR_SMEM > abi::max_smem_optin()) return abi::fail(SWB_ERR_SMEM, "prune needs %d B of shared memory", PR_SMEM);
    cudaError_t e = cudaFuncSetAttribute(prune_kernel<VEC>, cudaFuncAttributeMaxDynamicSharedMemorySize, PR_SMEM);
    if (e != cudaSuccess) return abi::cuda_fail(e, "cudaFuncSetAttribute(prune)");
    prune_kernel<VEC><<<(unsigned)n, PR_THREADS, PR_SMEM, st>>>(X, nx, dim, cand, cdist, C, deg, alpha, metric, dpn,
                                                               protect, out);
    return abi::cuda_check("prune launch");
}

int launch_prune(const float* X, int64_t nx, int64_t n, int dim, const int32_t* cand, const float* cdist, int C,
                 int deg, float alpha, int metric, const int32_t* dpn, const uint8_t* protect, int32_t* out,
                 cudaStream_t st) {
    if (C > PR_CP) return abi::fail(SWB_ERR_ARG, "candidates per node must be at most %d", PR_CP);
    const bool vec = (dim % 4 == 0) && (reinterpret_cast<uintptr_t>(X) % 16 == 0);
    return vec ? launch_prune_t<true>(X, nx, n, dim, cand, cdist, C, deg, alpha, metric, dpn, protect, out, st)
               : launch_prune_t<false>(X, nx, n, dim, cand, cdist, C, deg, alpha, metric, dpn, protect, out, st);
}

}  // namespace

extern "C" int swb_row_norms(const void* X, int x_dtype, int64_t n, int dim, float* norms, void* stream) {
    if (!X || !norms || n <= 0) return abi::fail(SWB_ERR_ARG, "bad norms arguments");
    const int vec = x_dtype == SWB_F16 ? 8 : 4;
    if (dim % vec) return abi::fail(SWB_ERR_ARG, "dimension must be a multiple of %d", vec);
    const unsigned blocks = (unsigned)((n + 255) / 256);
    if (x_dtype == SWB_F16)
        norms_kernel<__half><<<blocks, 256, 0, (cudaStream_t)stream>>>((const __half*)X, n, dim, norms);
    else
        norms_kernel<float><<<blocks, 256, 0, (cudaStream_t)stream>>>((const float*)X, n, dim, norms);
    return abi::cuda_check("norms launch");
}

// Top-C of a block of precomputed dot products (columns [col0, col0 + ncols)),
// folded into idx/dst; resume = 0 starts the lists fresh.
extern "C" int swb_topc_block(const float* dots, int64_t rows, int64_t ld, int64_t ncols, int64_t row0, int64_t col0,
                              const float* norms, int metric, int C, int32_t* idx, float* dst, int resume,
                              void* stream) {
    if (!dots || !idx || !dst || rows <= 0) return abi::fail(SWB_ERR_ARG, "bad top-C arguments");
    if (C < 1 || C > 256) return abi::fail(SWB_ERR_ARG, "C must be 1..256");
    if (metric == SWB_METRIC_L2 && !norms) return abi::fail(SWB_ERR_ARG, "l2 needs row norms");
    const int warps = 8;
    const size_t smem = (size_t)warps * (C * 16 + UB * 8);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(topc_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return abi::cuda_fail(e, "cudaFuncSetAttribute(topc)");
    }
    const unsigned blocks = (unsigned)((rows + warps - 1) / warps);
    topc_rows_kernel<<<blocks, warps * 32, smem, (cudaStream_t)stream>>>(dots, rows, ld, ncols, row0, col0, norms,
                                                                         metric, C, idx, dst, resume);
    return abi::cuda_check("top-C launch");
}

extern "C" int swb_prune(const float* X, int64_t n, int dim, const int32_t* cand, const float* cdist, int64_t rows,
                         int C, int deg, float alpha, int metric, const int32_t* deg_per_node,
                         const uint8_t* protect, int32_t* out, void* stream) {
    if (!X || !cand || !cdist || !out) return abi::fail(SWB_ERR_ARG, "null buffer");
    if (C < 1 || C > 128) return abi::fail(SWB_ERR_ARG, "candidates per node must be 1..128");
    if (deg < 1) return abi::fail(SWB_ERR_ARG, "degree must be positive");
    if (rows <= 0) return SWB_OK;
    return launch_prune(X, n, rows, dim, cand, cdist, C, deg, alpha, metric, deg_per_node, protect, out,
                        (cudaStream_t)stream);
}

extern "C" uint64_t swb_reverse_workspace(int64_t n, int64_t rows, int deg, int max_in) {
    const int64_t total = n * (int64_t)deg;
    const int keepn = (deg + max_in) < 128 ? (deg + max_in) : 128;
    uint64_t b = 0;
    b += align256(total * 4) * 4;                 // keys, vals, sorted keys, sorted vals
    b += align256((n + 1) * 8);                   // starts
    b += align256(rows * (int64_t)keepn * 4) * 2; // candidates, their distances
    b += align256(radix_temp_bytes(total));
    return b;
}

// The tensor-core prune (prune_tc.cu).
int swb_prune_tc_launch(const float* X, const void* A, const void* A_lo, int a_dtype, int adim, const float* norms,
                        int64_t n, int dim, const int32_t* cand, const float* cdist, int64_t rows, int C, int deg,
                        float alpha, int metric, const int32_t* deg_per_node, const uint8_t* protect, int32_t* out,
                        unsigned long long* recomputed, int32_t* status, cudaStream_t st);

namespace {

// The operands of a tensor-core prune (A == nullptr: the CUDA-core prune).
struct TcOps {
    const void* A;
    const void* A_lo;
    int a_dtype, adim;
    const float* norms;
    unsigned long long* recomputed;
    int32_t* status;
};

int reverse_impl(const float* X, int64_t n, int dim, const int32_t* G, int deg, float alpha, int max_in, int metric,
                 const int32_t* deg_per_node, int64_t row0, int64_t rows, int32_t* out, void* workspace,
                 uint64_t ws_bytes, const TcOps& tc, cudaStream_t st);

}  // namespace

extern "C" int swb_reverse(const float* X, int64_t n, int dim, const int32_t* G, int deg, float alpha, int max_in,
                           int metric, const int32_t* deg_per_node, int64_t row0, int64_t rows, int32_t* out,
                           void* workspace, uint64_t ws_bytes, void* stream) {
    const TcOps none{nullptr, nullptr, 0, 0, nullptr, nullptr, nullptr};
    return reverse_impl(X, n, dim, G, deg, alpha, max_in, metric, deg_per_node, row0, rows, out, workspace, ws_bytes,
                        none, (cudaStream_t)stream);
}

extern "C" int swb_reverse_tc(const float* X, const void* A, const void* A_lo, int a_dtype, int adim,
                              const float* norms, int64_t n, int dim, const int32_t* G, int deg, float alpha,
                              int max_in, int metric, const int32_t* deg_per_node, int64_t row0, int64_t rows,
                              int32_t* out, void* workspace, uint64_t ws_bytes, unsigned long long* recomputed,
                              int32_t* status, void* stream) {
    if (!A || !norms) return abi::fail(SWB_ERR_ARG, "the tensor-core reverse pass needs its operand rows and norms");
    const TcOps tc{A, A_lo, a_dtype, adim, norms, recomputed, status};
    return reverse_impl(X, n, dim, G, deg, alpha, max_in, metric, deg_per_node, row0, rows, out, workspace, ws_bytes,
                        tc, (cudaStream_t)stream);
}

namespace {

int reverse_impl(const float* X, int64_t n, int dim, const int32_t* G, int deg, float alpha, int max_in, int metric,
                 const int32_t* deg_per_node, int64_t row0, int64_t rows, int32_t* out, void* workspace,
                 uint64_t ws_bytes, const TcOps& tc, cudaStream_t st) {
    if (!X || !G || !out || !workspace) return abi::fail(SWB_ERR_ARG, "null buffer");
    if (n <= 0 || rows <= 0) return SWB_OK;
    if (row0 < 0 || row0 + rows > n) return abi::fail(SWB_ERR_ARG, "row range outside the graph");
    const int64_t total = n * (int64_t)deg;
    if (total >= (int64_t)1 << 31) return abi::fail(SWB_ERR_ARG, "n * degree must be below 2^31");
    if (ws_bytes < swb_reverse_workspace(n, rows, deg, max_in)) return abi::fail(SWB_ERR_ARG, "workspace too small");
    if (deg + max_in > 256) return abi::fail(SWB_ERR_ARG, "degree + max_in must be at most 256");
    const int keepn = (deg + max_in) < 128 ? (deg + max_in) : 128;
    char* p = (char*)workspace;
    int32_t* keys = (int32_t*)p; p += align256(total * 4);
    int32_t* vals = (int32_t*)p; p += align256(total * 4);
    int32_t* skeys = (int32_t*)p; p += align256(total * 4);
    int32_t* svals = (int32_t*)p; p += align256(total * 4);
    int64_t* starts = (int64_t*)p; p += align256((n + 1) * 8);
    int32_t* cand = (int32_t*)p; p += align256(rows * (int64_t)keepn * 4);
    float* cdist = (float*)p; p += align256(rows * (int64_t)keepn * 4);
    void* tmp = p;
    size_t tmp_bytes = radix_temp_bytes(total);
    edge_keys_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(G, total, n, keys, vals);
    int rc = abi::cuda_check("edge keys launch");
    if (rc) return rc;
    // LSD radix sort is stable: offers to one target stay in (source, slot) order
    cudaError_t e = cub::DeviceRadixSort::SortPairs(tmp, tmp_bytes, keys, skeys, vals, svals, (int)total, 0, 32, st);
    if (e != cudaSuccess) return abi::cuda_fail(e, "radix sort");
    seg_starts_kernel<<<(unsigned)((n + 1 + 255) / 256), 256, 0, st>>>(skeys, total, n, starts);
    rc = abi::cuda_check("segment starts launch");
    if (rc) return rc;
    int Wp = 2;
    while (Wp < deg + max_in) Wp <<= 1;
    const int smem = Wp * 12 + dim * 4;
    if (smem > abi::max_smem_optin()) return abi::fail(SWB_ERR_SMEM, "reverse merge needs %d B of shared memory", smem);
    // the candidates' rows: the fp16 operand copy when the tensor-core prune has
    // one (fp16-valued corpus), else the fp32 rows; 16-byte loads when aligned
    const bool half = tc.A && tc.a_dtype == SWB_F16;
    const void* rowsrc = half ? tc.A : (const void*)X;
    const int64_t stride = half ? tc.adim : dim;
    const int vw = half ? 8 : 4;
    const bool vec = dim % vw == 0 && stride % vw == 0 && reinterpret_cast<uintptr_t>(rowsrc) % 16 == 0;
    auto launch_merge = [&](auto kern, const auto* src) -> int {
        if (smem > 48 * 1024) {
            cudaError_t ea = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (ea != cudaSuccess) return abi::cuda_fail(ea, "cudaFuncSetAttribute(merge_row)");
        }
        kern<<<(unsigned)rows, RV_THREADS, smem, st>>>(X, dim, src, stride, G, deg, svals, starts, max_in, metric,
                                                       keepn, n, row0, cand, cdist);
        return abi::cuda_check("reverse merge launch");
    };
    if (half) {
        const __half* hs = static_cast<const __half*>(rowsrc);
        rc = vec ? launch_merge(merge_row_kernel<__half, true>, hs) : launch_merge(merge_row_kernel<__half, false>, hs);
    } else {
        rc = vec ? launch_merge(merge_row_kernel<float, true>, X) : launch_merge(merge_row_kernel<float, false>, X);
    }
    if (rc) return rc;
    const int32_t* dpn = deg_per_node ? deg_per_node + row0 : nullptr;
    if (tc.A)
        return swb_prune_tc_launch(X, tc.A, tc.A_lo, tc.a_dtype, tc.adim, tc.norms, n, dim, cand, cdist, rows, keepn,
                                   deg, alpha, metric, dpn, nullptr, out, tc.recomputed, tc.status, st);
    return launch_prune(X, n, rows, dim, cand, cdist, keepn, deg, alpha, metric, dpn, nullptr, out, st);
}

}  // namespace

extern "C" const char* swb_last_error(void) { return abi::last_error().c_str(); }
extern "C" int swb_version(void) { return 1; }
