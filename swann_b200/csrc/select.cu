// select.cu -- the top-E of entry (seed) selection.
//
// Replaces the torch.topk calls of select_nearest (swann/_select.py:93-130):
// the E catalogue entries nearest each query, from a slice of query x catalogue
// scores (a library TF32 GEMM's output), turned into the corpus metric with
// the reference's expressions -- 1 - s (ip), (|v|^2 - 2s) + |q|^2 (l2), each
// operation rounded once as torch evaluates it -- and folded into a running
// sorted list, so slices of the catalogue can come one after another.
//
// One warp per query row.  The row's list (at most 32 * R entries, sorted by
// (distance, index)) lives in shared memory; each lane reads four scores at a
// time, values that cannot enter the list are dropped against its E-th key,
// and the survivors are buffered in shared memory; each time 32 have gathered
// they are sorted across the warp and merged: every entry's new position is
// its own index plus the number of entries of the other sequence before it
// (binary lifting over the lanes), so both sequences are scattered straight
// into the other half of a ping-pong pair.  (A row of 4096 scores has about
// 155 survivors against a running E = 32: buffering merges them in ~5-10
// rounds rather than once per 32-column group that holds one.)  The filter
// only drops keys that cannot be in the final list, so the result does not
// depend on when the merges happen.  Ties between equal distances go to the
// lower index; torch.topk leaves that order unspecified.

#include <cstdint>

#include "abi_util.h"
#include "common.cuh"

namespace swb {
namespace sel {

constexpr int WARPS = 8;

// Merge 32 candidates (lane l holds one; invalid ones are +inf keys) into the
// sorted list `src` (nb entries, lane-major blocks of R per lane) and write the
// first min(E, nb + kept) entries of the union to `dst`.  Returns the new length.
template <int R>
__device__ int merge32(const float* src_d, const int* src_i, float* dst_d, int* dst_i, int nb, int E, float bd,
                       int bi, int lane) {
    const float INF = __int_as_float(0x7f800000);
    const int bcnt = __popc(__ballot_sync(FULL, bi != 0x7fffffff));
    float ed[R];
    int ei[R];
#pragma unroll
    for (int u = 0; u < R; ++u) {
        const int idx = lane * R + u;
        const bool ok = idx < nb;
        ed[u] = ok ? src_d[idx] : INF;
        ei[u] = ok ? src_i[idx] : 0x7fffffff;
    }
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            const float pd = __shfl_xor_sync(FULL, bd, j);
            const int pi = __shfl_xor_sync(FULL, bi, j);
            const bool up = (lane & k) == 0, lower = (lane & j) == 0;
            const bool take = (lower == up) ? key_lt(pd, pi, bd, bi) : key_lt(bd, bi, pd, pi);
            if (take) { bd = pd; bi = pi; }
        }
    }
    // list entries: candidates before each
    int epos[R];
#pragma unroll
    for (int u = 0; u < R; ++u) epos[u] = 0;
#pragma unroll
    for (int step = 16; step > 0; step >>= 1) {
#pragma unroll
        for (int u = 0; u < R; ++u) {
            const int m = epos[u] + step - 1;
            const float pd = __shfl_sync(FULL, bd, m);
            const int pi = __shfl_sync(FULL, bi, m);
            if (key_lt(pd, pi, ed[u], ei[u])) epos[u] += step;
        }
    }
    {
        const float pd = __shfl_sync(FULL, bd, 31);
        const int pi = __shfl_sync(FULL, bi, 31);
#pragma unroll
        for (int u = 0; u < R; ++u)
            if (epos[u] == 31 && key_lt(pd, pi, ed[u], ei[u])) epos[u] = 32;
    }
    // candidates: whole lanes of the list before it, then entries of the next lane
    const float lastd = ed[R - 1];
    const int lasti = ei[R - 1];
    int lb = 0;
#pragma unroll
    for (int step = 16; step > 0; step >>= 1) {
        const int m = lb + step - 1;
        const float pd = __shfl_sync(FULL, lastd, m);
        const int pi = __shfl_sync(FULL, lasti, m);
        if (key_lt(pd, pi, bd, bi)) lb += step;
    }
    {
        const float pd = __shfl_sync(FULL, lastd, 31);
        const int pi = __shfl_sync(FULL, lasti, 31);
        if (lb == 31 && key_lt(pd, pi, bd, bi)) lb = 32;
    }
    const int srcl = lb < 32 ? lb : 31;
    int inlane = 0;
#pragma unroll
    for (int u = 0; u < R; ++u) {
        const float pd = __shfl_sync(FULL, ed[u], srcl);
        const int pi = __shfl_sync(FULL, ei[u], srcl);
        if (lb < 32 && key_lt(pd, pi, bd, bi)) ++inlane;
    }
    const int mine = lb * R + inlane;
#pragma unroll
    for (int u = 0; u < R; ++u) {
        const int pos = lane * R + u + epos[u];
        if (lane * R + u < nb && pos < E) {
            dst_d[pos] = ed[u];
            dst_i[pos] = ei[u];
        }
    }
    if (lane < bcnt) {
        const int pos = lane + mine;
        if (pos < E) {
            dst_d[pos] = bd;
            dst_i[pos] = bi;
        }
    }
    __syncwarp();
    return min(E, nb + bcnt);
}

template <int R>
__global__ void __launch_bounds__(WARPS * 32) topk_kernel(const float* __restrict__ S, int64_t rows, int P,
                                                          int64_t ld, const float* __restrict__ vn,
                                                          const float* __restrict__ qn, int metric, int E, int col0,
                                                          float* __restrict__ best_d, int64_t* __restrict__ best_i,
                                                          int resume, int vec) {
    __shared__ float s_d[WARPS][2][32 * R];
    __shared__ int s_i[WARPS][2][32 * R];
    __shared__ float b_d[WARPS][64];   // survivors waiting for a merge (at most 63)
    __shared__ int b_i[WARPS][64];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * WARPS + warp;
    if (row >= rows) return;   // whole warps only: nothing below synchronises the block
    const float INF = __int_as_float(0x7f800000);
    int cur = 0, nb = 0;
    if (resume) {   // the running list of earlier slices: a sorted prefix of valid entries
        int c = 0;
        for (int e = lane; e < E; e += 32) {
            const int64_t id = best_i[row * E + e];
            s_d[warp][0][e] = best_d[row * E + e];
            s_i[warp][0][e] = id >= 0 ? (int)id : 0x7fffffff;
            c += id >= 0 ? 1 : 0;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) c += __shfl_xor_sync(FULL, c, off);
        nb = c;
        __syncwarp();
    }
    float thd = INF;
    int thi = 0x7fffffff;
    if (nb == E) {
        thd = s_d[warp][cur][E - 1];
        thi = s_i[warp][cur][E - 1];
    }
    const float q2 = (metric == METRIC_L2) ? qn[row] : 0.f;
    int cnt = 0;   // buffered survivors
    const float* srow = S + row * ld;
    for (int c0 = 0; c0 < P; c0 += 128) {
        const int jb = c0 + 4 * lane;
        float s[4];
        if (vec && jb + 3 < P) {
            const float4 t = __ldg(reinterpret_cast<const float4*>(srow + jb));
            s[0] = t.x; s[1] = t.y; s[2] = t.z; s[3] = t.w;
        } else {
#pragma unroll
            for (int u = 0; u < 4; ++u) s[u] = (jb + u < P) ? __ldg(srow + jb + u) : 0.f;
        }
        float d[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            if (metric == METRIC_IP) d[u] = __fsub_rn(1.f, s[u]);
            else d[u] = __fadd_rn(__fsub_rn(jb + u < P ? __ldg(vn + jb + u) : 0.f, __fmul_rn(2.f, s[u])), q2);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int j = col0 + jb + u;
            const bool keep = (jb + u < P) && (nb < E || key_lt(d[u], j, thd, thi));
            const unsigned km = __ballot_sync(FULL, keep);
            if (!km) continue;
            if (keep) {
                const int pos = cnt + __popc(km & lanemask_lt());
                b_d[warp][pos] = d[u];
                b_i[warp][pos] = j;
            }
            cnt += __popc(km);
            __syncwarp();
            if (cnt >= 32) {   // merge 32 buffered survivors, keep the rest
                nb = merge32<R>(s_d[warp][cur], s_i[warp][cur], s_d[warp][cur ^ 1], s_i[warp][cur ^ 1], nb, E,
                                b_d[warp][lane], b_i[warp][lane], lane);
                cur ^= 1;
                const float rd = (lane + 32 < cnt) ? b_d[warp][lane + 32] : INF;
                const int ri = (lane + 32 < cnt) ? b_i[warp][lane + 32] : 0x7fffffff;
                __syncwarp();
                b_d[warp][lane] = rd;
                b_i[warp][lane] = ri;
                cnt -= 32;
                __syncwarp();
                if (nb == E) {
                    thd = s_d[warp][cur][E - 1];
                    thi = s_i[warp][cur][E - 1];
                }
            }
        }
    }
    if (cnt > 0) {   // the last survivors (fewer than 32; the rest of the lanes offer nothing)
        const bool ok = lane < cnt;
        nb = merge32<R>(s_d[warp][cur], s_i[warp][cur], s_d[warp][cur ^ 1], s_i[warp][cur ^ 1], nb, E,
                        ok ? b_d[warp][lane] : INF, ok ? b_i[warp][lane] : 0x7fffffff, lane);
        cur ^= 1;
    }
    for (int e = lane; e < E; e += 32) {
        const bool ok = e < nb;
        best_d[row * E + e] = ok ? s_d[warp][cur][e] : INF;
        best_i[row * E + e] = ok ? (int64_t)s_i[warp][cur][e] : -1;
    }
}

}  // namespace sel
}  // namespace swb

using namespace swb;

extern "C" int swb_select_topk(const float* scores, int64_t rows, int P, int64_t ld, const float* vnorm,
                               const float* qnorm, int metric, int E, int col0, float* best_d, int64_t* best_i,
                               int resume, void* stream) {
    if (!scores || !best_d || !best_i) return abi::fail(SWB_ERR_ARG, "null buffer");
    if (rows <= 0 || P <= 0) return SWB_OK;
    if (E < 1 || E > 128) return abi::fail(SWB_ERR_ARG, "E must be 1..128");
    if (ld < P) return abi::fail(SWB_ERR_ARG, "row stride below the slice width");
    if (metric == SWB_METRIC_L2 && (!vnorm || !qnorm)) return abi::fail(SWB_ERR_ARG, "l2 needs both norm vectors");
    if (col0 < 0 || (int64_t)col0 + P >= ((int64_t)1 << 31)) return abi::fail(SWB_ERR_ARG, "catalogue index range");
    const int vec = (ld % 4 == 0) && (reinterpret_cast<uintptr_t>(scores) % 16 == 0);
    const unsigned blocks = (unsigned)((rows + sel::WARPS - 1) / sel::WARPS);
    cudaStream_t st = (cudaStream_t)stream;
    if (E <= 32)
        sel::topk_kernel<1><<<blocks, sel::WARPS * 32, 0, st>>>(scores, rows, P, ld, vnorm, qnorm, metric, E, col0,
                                                                best_d, best_i, resume, vec);
    else if (E <= 64)
        sel::topk_kernel<2><<<blocks, sel::WARPS * 32, 0, st>>>(scores, rows, P, ld, vnorm, qnorm, metric, E, col0,
                                                                best_d, best_i, resume, vec);
    else
        sel::topk_kernel<4><<<blocks, sel::WARPS * 32, 0, st>>>(scores, rows, P, ld, vnorm, qnorm, metric, E, col0,
                                                                best_d, best_i, resume, vec);
    return abi::cuda_check("select launch");
}
