// offline.cu -- the offline graph builder's extras for sm_100a.
//
// Replaces the torch passes of offline/build_graph.py that sit around the
// build's three stages:
//   candidates_from_graph (build_graph.py:73-99)   graph_candidates_kernel
//   mutual_rank           (build_graph.py:102-130)  mutual_kernel
//   fill_degree           (build_graph.py:133-202)  fill_kernel, chunk by chunk
//   enforce_min_in        (build_graph.py:309-386)  a host loop of min_in_* kernels
// Per-node degrees (the pool boost) and protected pairs are arguments of the
// prune itself (build.cu).
//
// Where the reference's outcome depends on an unspecified order (torch.sort
// and torch.argsort without stable=True), the order here is fixed and stated:
// ties by position for the candidate sort, the lowest source node for "one
// writer per target".

#include <cstdint>
#include <vector>

#include "abi_util.h"
#include "common.cuh"

namespace swb {
namespace offline {

constexpr float FAR = 3.4e38f;   // build_graph.py's "no distance"

// ---------------------------------------------------------------------------
// candidates_from_graph: node u's first C graph neighbours with exact
// distances (dimension-ordered fmaf, as the reverse pass scores), -1 entries
// and u itself at FAR, ordered by (distance, position).
constexpr int GC_THREADS = 128;

__global__ void __launch_bounds__(GC_THREADS) graph_candidates_kernel(const float* __restrict__ X, int64_t n,
                                                                       int dim, const int32_t* __restrict__ Gc,
                                                                       int gw, int C, int Cp, int metric,
                                                                       int32_t* __restrict__ idx,
                                                                       float* __restrict__ dst) {
    extern __shared__ __align__(16) char smem[];
    float* xu = reinterpret_cast<float*>(smem);            // [dim]
    float* sd = xu + dim;                                   // [Cp]
    int* sp = reinterpret_cast<int*>(sd + Cp);              // [Cp] positions
    const int64_t u = blockIdx.x;
    for (int k = threadIdx.x; k < dim; k += GC_THREADS) xu[k] = X[u * dim + k];
    __syncthreads();
    for (int i = threadIdx.x; i < Cp; i += GC_THREADS) {
        float d = __int_as_float(0x7f800000);   // padding beyond C sorts last
        if (i < C) {
            const int v = Gc[u * gw + i];
            d = FAR;
            if (v >= 0 && v < n && v != u) {
                const float* xv = X + (size_t)v * dim;
                float acc = 0.f;
                if (metric == METRIC_IP) {
                    for (int k = 0; k < dim; ++k) acc = fmaf(__ldg(&xv[k]), xu[k], acc);
                    d = __fsub_rn(1.f, acc);
                } else {
                    for (int k = 0; k < dim; ++k) {
                        const float df = __fsub_rn(xu[k], __ldg(&xv[k]));
                        acc = fmaf(df, df, acc);
                    }
                    d = acc;
                }
            }
        }
        sd[i] = d;
        sp[i] = i;
    }
    __syncthreads();
    for (int k = 2; k <= Cp; k <<= 1)
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < Cp; i += GC_THREADS) {
                const int l = i ^ j;
                if (l > i) {
                    const bool up = (i & k) == 0;
                    const bool gt = key_lt(sd[l], sp[l], sd[i], sp[i]);   // (d, position) order
                    if (gt == up) {
                        const float td = sd[i]; sd[i] = sd[l]; sd[l] = td;
                        const int tp = sp[i]; sp[i] = sp[l]; sp[l] = tp;
                    }
                }
            }
            __syncthreads();
        }
    for (int i = threadIdx.x; i < C; i += GC_THREADS) {
        idx[u * C + i] = Gc[u * gw + sp[i]];
        dst[u * C + i] = sd[i];
    }
}

// ---------------------------------------------------------------------------
// mutual_rank: out[u, i] (i < M) = cand[u, i] >= 0 and u is among the first M
// entries of cand[cand[u, i]]; columns from M on are 0.  One warp per node.
__global__ void mutual_kernel(const int32_t* __restrict__ cand, int64_t n, int C, int M, uint8_t* __restrict__ out) {
    const int64_t u = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (u >= n) return;
    for (int i = lane; i < C; i += 32) {
        uint8_t r = 0;
        if (i < M) {
            const int v = cand[u * C + i];
            if (v >= 0 && v < n) {
                const int32_t* back = cand + (size_t)v * C;
                for (int t = 0; t < M; ++t)
                    if (back[t] == (int32_t)u) { r = 1; break; }
            }
        }
        out[u * C + i] = r;
    }
}

// ---------------------------------------------------------------------------
// fill_degree for rows [s, s + rows): the empty slots of a node's row get its
// refused candidates, in candidate order ("near", "bridge") or reverse order
// ("far"); "bridge" offers only candidates with no two-hop path back through
// the kept graph.  Reads G as the earlier chunks left it and writes the new
// rows to `tmp`, so rows of one chunk see each other unfilled -- the
// reference's chunk loop does the same.
constexpr int FILL_THREADS = 128;
enum { RULE_NEAR = 0, RULE_FAR = 1, RULE_BRIDGE = 2 };

__device__ __forceinline__ uint32_t fill_hash(int v, uint32_t mask) { return (2654435761u * (uint32_t)v) & mask; }

__global__ void __launch_bounds__(FILL_THREADS) fill_kernel(const int32_t* __restrict__ G, int64_t n, int W,
                                                            const int32_t* __restrict__ cand, int C, int rule,
                                                            int64_t s, int hbits, int32_t* __restrict__ tmp) {
    extern __shared__ __align__(16) char smem[];
    int* hs = reinterpret_cast<int*>(smem);                 // two-hop set, open addressing, -1 = empty
    int* row = hs + (rule == RULE_BRIDGE ? (1 << hbits) : 0);   // [W] this node's row
    uint8_t* fre = reinterpret_cast<uint8_t*>(row + W);         // [C] free flags
    __shared__ int s_free[256], s_empty[256];
    __shared__ int s_nfree, s_nempty;
    const int64_t u = s + blockIdx.x;
    const uint32_t hmask = (1u << hbits) - 1u;
    for (int i = threadIdx.x; i < W; i += FILL_THREADS) row[i] = G[u * W + i];
    if (rule == RULE_BRIDGE)
        for (int i = threadIdx.x; i < (1 << hbits); i += FILL_THREADS) hs[i] = -1;
    __syncthreads();
    if (rule == RULE_BRIDGE) {
        // the kept neighbours' own neighbours
        for (int e = threadIdx.x; e < W * W; e += FILL_THREADS) {
            const int w = row[e / W];
            if (w < 0 || w >= n) continue;
            const int x = G[(size_t)w * W + e % W];
            if (x < 0) continue;
            uint32_t h = fill_hash(x, hmask);
            for (;;) {
                const int old = atomicCAS(&hs[h], -1, x);
                if (old == -1 || old == x) break;
                h = (h + 1) & hmask;
            }
        }
        __syncthreads();
    }
    for (int i = threadIdx.x; i < C; i += FILL_THREADS) {
        const int v = cand[u * C + i];
        bool taken = v < 0 || v == (int)u;
        for (int k = 0; k < W && !taken; ++k) taken = row[k] == v;
        bool ok = !taken;
        if (ok && rule == RULE_BRIDGE) {
            uint32_t h = fill_hash(v, hmask);
            for (;;) {
                const int x = hs[h];
                if (x == -1) break;
                if (x == v) { ok = false; break; }
                h = (h + 1) & hmask;
            }
        }
        fre[i] = ok ? 1 : 0;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int nf = 0, ne = 0;
        if (rule == RULE_FAR) {
            for (int i = C - 1; i >= 0; --i)
                if (fre[i]) s_free[nf++] = i;
        } else {
            for (int i = 0; i < C; ++i)
                if (fre[i]) s_free[nf++] = i;
        }
        for (int k = 0; k < W; ++k)
            if (row[k] < 0) s_empty[ne++] = k;
        s_nfree = nf;
        s_nempty = ne;
    }
    __syncthreads();
    const int take = min(s_nfree, s_nempty);
    for (int t = threadIdx.x; t < take; t += FILL_THREADS) row[s_empty[t]] = cand[u * C + s_free[t]];
    __syncthreads();
    for (int i = threadIdx.x; i < W; i += FILL_THREADS) tmp[(size_t)blockIdx.x * W + i] = row[i];
}

// ---------------------------------------------------------------------------
// enforce_min_in, one candidate column at a time:
//   propose  every node still short of in-edges offers itself to its i-th
//            candidate t (t valid, not itself, not already pointing at it);
//            the lowest offering node wins t (atomicMin)
//   place    each winner s takes t's last slot (not slot 0) whose head is
//            above the floor, in-degrees read as they were before the step
//   apply    victims lose one in-edge (once per victim, as the reference's
//            indexed assignment does), then winners gain one, then the edge
//            is written and the winner's shortfall drops
__global__ void indeg_kernel(const int32_t* __restrict__ G, int64_t total, int64_t n, int32_t* __restrict__ indeg) {
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= total) return;
    const int v = G[e];
    if (v >= 0 && v < n) atomicAdd(&indeg[v], 1);
}

__global__ void min_in_init(const int32_t* __restrict__ indeg, int64_t n, int min_in, int C,
                            int32_t* __restrict__ remaining, int32_t* __restrict__ counts) {
    const int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (v >= n) return;
    const int need = min_in - indeg[v];
    const int r = need > 0 ? (need < C ? need : C) : 0;
    remaining[v] = r;
    if (r > 0) {
        atomicAdd(&counts[0], 1);        // nodes below the floor
        atomicAdd(&counts[1], r);        // edges to place
    }
}

__global__ void min_in_propose(const int32_t* __restrict__ G, int64_t n, int W, const int32_t* __restrict__ cand,
                               int C, int col, const int32_t* __restrict__ remaining, int32_t* __restrict__ claim,
                               int32_t* __restrict__ counts) {
    const int64_t sidx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (sidx >= n || remaining[sidx] <= 0) return;
    atomicAdd(&counts[2], 1);   // nodes still short: the host stops when none are
    const int t = cand[sidx * C + col];
    if (t < 0 || t >= n || t == (int)sidx) return;
    const int32_t* rt = G + (size_t)t * W;
    for (int k = 0; k < W; ++k)
        if (rt[k] == (int32_t)sidx) {
            atomicAdd(&counts[3], 1);   // already linked
            return;
        }
    atomicMin(&claim[t], (int)sidx);
}

__global__ void min_in_place(const int32_t* __restrict__ G, int64_t n, int W, const int32_t* __restrict__ cand,
                             int C, int col, const int32_t* __restrict__ remaining, const int32_t* __restrict__ claim,
                             const int32_t* __restrict__ indeg, int min_in, int32_t* __restrict__ slot_of,
                             int32_t* __restrict__ victim_of) {
    const int64_t sidx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (sidx >= n) return;
    slot_of[sidx] = -1;
    if (remaining[sidx] <= 0) return;
    const int t = cand[sidx * C + col];
    if (t < 0 || t >= n || claim[t] != (int)sidx) return;
    const int32_t* rt = G + (size_t)t * W;
    int slot = -1;
    for (int k = 0; k < W; ++k) {
        const int h = rt[k];
        if (h >= 0 && h < n && indeg[h] > min_in) slot = k;
    }
    if (slot >= 1) {
        slot_of[sidx] = slot;
        victim_of[sidx] = rt[slot];
    }
}

__global__ void min_in_victims(int64_t n, const int32_t* __restrict__ slot_of, const int32_t* __restrict__ victim_of,
                               const int32_t* __restrict__ indeg0, int32_t* __restrict__ indeg) {
    const int64_t sidx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (sidx >= n || slot_of[sidx] < 0) return;
    const int v = victim_of[sidx];
    indeg[v] = indeg0[v] - 1;
}

__global__ void min_in_apply(int32_t* __restrict__ G, int64_t n, int W, const int32_t* __restrict__ cand, int C,
                             int col, const int32_t* __restrict__ slot_of, int32_t* __restrict__ indeg,
                             int32_t* __restrict__ remaining, int32_t* __restrict__ counts) {
    const int64_t sidx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (sidx >= n || slot_of[sidx] < 0) return;
    const int t = cand[sidx * C + col];
    indeg[sidx] += 1;
    G[(size_t)t * W + slot_of[sidx]] = (int32_t)sidx;
    remaining[sidx] -= 1;
    atomicAdd(&counts[4], 1);   // placed
}

}  // namespace offline
}  // namespace swb

using namespace swb;
using namespace swb::offline;

extern "C" int swb_graph_candidates(const float* X, int64_t n, int dim, const int32_t* Gc, int gc_width, int C,
                                    int metric, int32_t* idx, float* dst, void* stream) {
    if (!X || !Gc || !idx || !dst) return abi::fail(SWB_ERR_ARG, "null buffer");
    if (n <= 0) return SWB_OK;
    if (C < 1 || C > gc_width || C > 1024) return abi::fail(SWB_ERR_ARG, "C must be 1..min(graph width, 1024)");
    int Cp = 2;
    while (Cp < C) Cp <<= 1;
    const size_t smem = (size_t)dim * 4 + (size_t)Cp * 8;
    if (smem > (size_t)abi::max_smem_optin()) return abi::fail(SWB_ERR_SMEM, "dimension too large for one block");
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(graph_candidates_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return abi::cuda_fail(e, "cudaFuncSetAttribute(graph candidates)");
    }
    graph_candidates_kernel<<<(unsigned)n, GC_THREADS, smem, (cudaStream_t)stream>>>(X, n, dim, Gc, gc_width, C, Cp,
                                                                                      metric, idx, dst);
    return abi::cuda_check("graph candidates launch");
}

extern "C" int swb_mutual_rank(const int32_t* cand, int64_t n, int C, int M, uint8_t* out, void* stream) {
    if (!cand || !out) return abi::fail(SWB_ERR_ARG, "null buffer");
    if (n <= 0) return SWB_OK;
    if (M < 0) return abi::fail(SWB_ERR_ARG, "M must be non-negative");
    if (M > C) M = C;
    const int warps = 8;
    mutual_kernel<<<(unsigned)((n + warps - 1) / warps), warps * 32, 0, (cudaStream_t)stream>>>(cand, n, C, M, out);
    return abi::cuda_check("mutual rank launch");
}

extern "C" int swb_fill_degree(int32_t* G, int64_t n, int W, const int32_t* cand, int C, int rule, int chunk,
                               int32_t* tmp, void* stream) {
    if (!G || !cand || !tmp) return abi::fail(SWB_ERR_ARG, "null buffer");
    if (n <= 0) return SWB_OK;
    if (rule < RULE_NEAR || rule > RULE_BRIDGE) return abi::fail(SWB_ERR_ARG, "rule must be near, far or bridge");
    if (C < 1 || C > 256 || W < 1 || W > 256) return abi::fail(SWB_ERR_ARG, "widths must be 1..256");
    if (chunk < 1) return abi::fail(SWB_ERR_ARG, "chunk must be positive");
    int hbits = 0;
    if (rule == RULE_BRIDGE) {
        hbits = 4;
        while ((1 << hbits) < 2 * W * W) ++hbits;   // load at most one half
    }
    const size_t smem = (rule == RULE_BRIDGE ? ((size_t)4 << hbits) : 0) + (size_t)W * 4 + (size_t)C;
    if (smem > (size_t)abi::max_smem_optin()) return abi::fail(SWB_ERR_SMEM, "graph too wide for the bridge rule");
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(fill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return abi::cuda_fail(e, "cudaFuncSetAttribute(fill)");
    }
    cudaStream_t st = (cudaStream_t)stream;
    for (int64_t s = 0; s < n; s += chunk) {
        const int64_t rows = (n - s < chunk) ? n - s : chunk;
        fill_kernel<<<(unsigned)rows, FILL_THREADS, smem, st>>>(G, n, W, cand, C, rule, s, hbits, tmp);
        int rc = abi::cuda_check("fill launch");
        if (rc) return rc;
        cudaError_t e = cudaMemcpyAsync(G + s * W, tmp, (size_t)rows * W * 4, cudaMemcpyDeviceToDevice, st);
        if (e != cudaSuccess) return abi::cuda_fail(e, "fill copy-back");
    }
    return SWB_OK;
}

extern "C" uint64_t swb_min_in_workspace(int64_t n) { return (uint64_t)n * 4 * 6 + 64; }

// Synchronous: the loop needs to know when nothing is short any more.
// stats (optional, host) [rounds][4]: nodes below the floor, edges to place,
// edges placed, already-linked offers skipped.  Returns the rounds run.
extern "C" int swb_enforce_min_in(int32_t* G, int64_t n, int W, const int32_t* cand, int C, int min_in, int rounds,
                                  void* workspace, uint64_t ws_bytes, int32_t* stats, int* rounds_run, void* stream) {
    if (!G || !cand || !workspace) return abi::fail(SWB_ERR_ARG, "null buffer");
    if (rounds_run) *rounds_run = 0;
    if (n <= 0 || min_in <= 0 || rounds <= 0) return SWB_OK;
    if (n >= ((int64_t)1 << 31)) return abi::fail(SWB_ERR_ARG, "at most 2^31 - 1 nodes");
    if (ws_bytes < swb_min_in_workspace(n)) return abi::fail(SWB_ERR_ARG, "workspace too small");
    cudaStream_t st = (cudaStream_t)stream;
    int32_t* indeg = (int32_t*)workspace;
    int32_t* indeg0 = indeg + n;
    int32_t* remaining = indeg0 + n;
    int32_t* claim = remaining + n;
    int32_t* slot_of = claim + n;
    int32_t* victim_of = slot_of + n;
    int32_t* counts = victim_of + n;   // [8]
    const unsigned gb = (unsigned)((n + 255) / 256);
    const int64_t total = n * (int64_t)W;
    int32_t h[8];
    int r = 0;
    for (; r < rounds; ++r) {
        cudaMemsetAsync(indeg, 0, (size_t)n * 4, st);
        cudaMemsetAsync(counts, 0, 8 * 4, st);
        indeg_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(G, total, n, indeg);
        min_in_init<<<gb, 256, 0, st>>>(indeg, n, min_in, C, remaining, counts);
        int rc = abi::cuda_check("min-in launch");
        if (rc) return rc;
        cudaError_t e = cudaMemcpyAsync(h, counts, 8 * 4, cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) return abi::cuda_fail(e, "min-in counts");
        if (h[0] == 0) break;   // the floor is met
        const int below = h[0], need = h[1];
        int placed = 0, skipped = 0;
        for (int col = 0; col < C; ++col) {
            cudaMemsetAsync(claim, 0x7f, (size_t)n * 4, st);
            cudaMemsetAsync(counts + 2, 0, 3 * 4, st);
            min_in_propose<<<gb, 256, 0, st>>>(G, n, W, cand, C, col, remaining, claim, counts);
            min_in_place<<<gb, 256, 0, st>>>(G, n, W, cand, C, col, remaining, claim, indeg, min_in, slot_of,
                                             victim_of);
            cudaMemcpyAsync(indeg0, indeg, (size_t)n * 4, cudaMemcpyDeviceToDevice, st);
            min_in_victims<<<gb, 256, 0, st>>>(n, slot_of, victim_of, indeg0, indeg);
            min_in_apply<<<gb, 256, 0, st>>>(G, n, W, cand, C, col, slot_of, indeg, remaining, counts);
            rc = abi::cuda_check("min-in step launch");
            if (rc) return rc;
            e = cudaMemcpyAsync(h + 2, counts + 2, 3 * 4, cudaMemcpyDeviceToHost, st);
            if (e == cudaSuccess) e = cudaStreamSynchronize(st);
            if (e != cudaSuccess) return abi::cuda_fail(e, "min-in step counts");
            skipped += h[3];
            placed += h[4];
            if (h[2] == 0) break;   // nobody short any more
        }
        if (stats) {
            stats[r * 4 + 0] = below;
            stats[r * 4 + 1] = need;
            stats[r * 4 + 2] = placed;
            stats[r * 4 + 3] = skipped;
        }
    }
    if (rounds_run) *rounds_run = r;
    return SWB_OK;
}
