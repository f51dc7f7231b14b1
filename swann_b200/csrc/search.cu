// search.cu -- multi-branch graph search for sm_100a.
//
// Replaces the reference's init_kernel / advance_kernel / merge_branches_kernel
// (swann/csrc/local_search.cu:271-919).  Same semantics, different machine
// mapping:
//
//  * one WARP per branch (the reference spends a 128-thread CTA).  Selection,
//    compaction, sorting and the queue merge are warp-synchronous (ballots and
//    shuffles, no __syncthreads), and all D neighbours of an expansion probe the
//    shared table at once, one lane per neighbour;
//  * neighbour rows are read straight from HBM into registers in 16-byte
//    chunks, one team of lanes per row; other warps of the SM hide the latency;
//  * the per-query distance table packs (id + 1, distance bits) into one
//    64-bit word: one compare-and-swap claims a node or returns its distance;
//  * Index.search runs as one fused kernel: init, the walk for the whole
//    budget, each branch's best kk, and -- in the last branch of a query to
//    finish -- the merge of that query's branches.
//
// The distance arithmetic is the reference's, bit for bit (common.cuh).

#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "abi_util.h"
#include "common.cuh"

namespace swb {

// ---------------------------------------------------------------------------
// launch knobs and the per-warp shared-memory carve-up

struct Knobs {
    const void* X;
    int64_t n;
    int dim, rowbytes;
    const int32_t* G;
    int D;
    const float* Qv;
    const int32_t* seeds;
    int32_t* ids;
    float* dist;
    uint8_t* expd;
    uint8_t* lin;
    int Q, J, L, V;
    int32_t* visited;
    int H;
    int32_t* counters;
    int metric, delta, max_exp, policy;
    float stop_eps;
    int kstop;
    uint64_t* cache;
    int Hc;
    float* bound;
    int exclusive, stall_patience;
    float crowd_frac;
    const int32_t* active;
    int n_active;
    int32_t* status;
    int k, kk;
    int32_t* branch_ids;
    float* branch_dist;
    int32_t* qdone;
    int32_t* out_ids;
    float* out_dist;
    int W, warp_bytes, q_shared, cmax;
    // sign-code prefilter (advance only; null = off): codes [n][cwords] bits
    // around the corpus mean cmu [dim], per-node scale calpha [n], margin
    const int32_t* codes;
    const float* calpha;
    const float* cmu;
    float cmargin;
    int cwords;
};

__host__ __device__ inline int align16(int x) { return (x + 15) & ~15; }

// A branch's NCTR counters (local_search.cu:35-41), spread over the warp: lane
// c holds counter c; counter 0 (expansions) is also on every lane for the loop
// tests.  Two registers instead of NCTR.
struct Ctr {
    int mine, exp;
    __device__ void zero() { mine = 0; exp = 0; }
    __device__ void add(int lane, int c, int v) { mine += (lane == c) ? v : 0; }
    __device__ void set(int lane, int c, int v) { if (lane == c) mine = v; }
    __device__ void expand() { ++exp; }
    __device__ int value(int lane) const { return lane == 0 ? exp : mine; }
};

struct Layout {
    int q, s_id, s_d, s_e, s_l, n_id, n_d, n_e, n_l, c_id, c_d, c_l, w_v, w_slot, w_d, w_aux,
        retired, total;
};

// q_bytes = 0 when the query lives once per CTA rather than per warp; cmax
// (a power of two >= 32) bounds the candidates, seeds and rows of one step
__host__ __device__ inline Layout warp_layout(int L, int q_bytes, int cmax) {
    Layout w;
    int o = 0;
    w.q = o; o += align16(q_bytes);
    w.s_id = o; o += align16(L * 4);
    w.s_d = o; o += align16(L * 4);
    w.n_id = o; o += align16(L * 4);
    w.n_d = o; o += align16(L * 4);
    w.s_e = o; o += align16(L);
    w.s_l = o; o += align16(L);
    w.n_e = o; o += align16(L);
    w.n_l = o; o += align16(L);
    w.c_id = o; o += cmax * 4;
    w.c_d = o; o += cmax * 4;
    w.c_l = o; o += align16(cmax);
    w.w_v = o; o += cmax * 4;         // w_v .. w_aux are contiguous (4 * cmax ints)
    w.w_slot = o; o += cmax * 4;
    w.w_d = o; o += cmax * 4;
    w.w_aux = o; o += cmax * 4;
    w.retired = o; o += 32;
    w.total = align16(o);
    return w;
}

struct WarpMem {
    float* q;
    int* s_id;
    float* s_d;
    uint8_t* s_e;
    uint8_t* s_l;
    int* n_id;
    float* n_d;
    uint8_t* n_e;
    uint8_t* n_l;
    int* c_id;
    float* c_d;
    uint8_t* c_l;
    int* w_v;
    int* w_slot;
    float* w_d;
    int* w_aux;
    uint32_t* retired;
};

__device__ inline WarpMem carve(char* base, const Layout& l) {
    WarpMem w;
    w.q = reinterpret_cast<float*>(base + l.q);
    w.s_id = reinterpret_cast<int*>(base + l.s_id);
    w.s_d = reinterpret_cast<float*>(base + l.s_d);
    w.n_id = reinterpret_cast<int*>(base + l.n_id);
    w.n_d = reinterpret_cast<float*>(base + l.n_d);
    w.s_e = reinterpret_cast<uint8_t*>(base + l.s_e);
    w.s_l = reinterpret_cast<uint8_t*>(base + l.s_l);
    w.n_e = reinterpret_cast<uint8_t*>(base + l.n_e);
    w.n_l = reinterpret_cast<uint8_t*>(base + l.n_l);
    w.c_id = reinterpret_cast<int*>(base + l.c_id);
    w.c_d = reinterpret_cast<float*>(base + l.c_d);
    w.c_l = reinterpret_cast<uint8_t*>(base + l.c_l);
    w.w_v = reinterpret_cast<int*>(base + l.w_v);
    w.w_slot = reinterpret_cast<int*>(base + l.w_slot);
    w.w_d = reinterpret_cast<float*>(base + l.w_d);
    w.w_aux = reinterpret_cast<int*>(base + l.w_aux);
    w.retired = reinterpret_cast<uint32_t*>(base + l.retired);
    return w;
}

// ---------------------------------------------------------------------------
// hashing (local_search.cu:94-110, 169-183)

__device__ __forceinline__ uint32_t knuth(int key, uint32_t mask) { return (2654435761u * (uint32_t)key) & mask; }

// Per-branch visited set: int slots holding id + 1.  Returns 1 when this call
// inserted `v`; a full table sets `fail` and reports "not new".
__device__ __forceinline__ int visited_insert(int* tab, int H, int v, int& fail) {
    const uint32_t mask = (uint32_t)(H - 1);
    uint32_t pos = knuth(v, mask);
    for (int p = 0; p < H; ++p) {
        const int old = atomicCAS(&tab[pos], 0, v + 1);
        if (old == 0) return 1;
        if (old == v + 1) return 0;
        pos = (pos + 1) & mask;
    }
    fail = 1;
    return 0;
}

// Per-query distance table slot = (id + 1) << 32 | float bits; a claimed but
// not yet scored slot carries FLT_MAX.

// One node's probe of the per-query table, given the outcome of its first
// compare-and-swap (issued by the caller alongside the other neighbours'):
// resolves it and probes on linearly after a collision (CPROBE probes at
// most).  Returns the cached distance (FLT_MAX when none), the slot (-1 when
// the probes ran out) and whether this call claimed it.
__device__ __forceinline__ float cache_probe_rest(uint64_t* tab, int Hc, int v, uint32_t pos,
                                                  unsigned long long old, int& slot, int& claimed) {
    const uint32_t mask = (uint32_t)(Hc - 1);
    const uint32_t key = (uint32_t)(v + 1);
    const unsigned long long want = ((unsigned long long)key << 32) | FLT_MAX_BITS;
    for (int p = 0;;) {
        if (old == 0ull) {
            slot = (int)pos;
            claimed = 1;
            return FLT_MAX;
        }
        if ((uint32_t)(old >> 32) == key) {
            slot = (int)pos;
            claimed = 0;
            return __uint_as_float((uint32_t)old);
        }
        if (++p >= CPROBE) break;
        pos = (pos + 1) & mask;
        old = atomicCAS(reinterpret_cast<unsigned long long*>(&tab[pos]), 0ull, want);
    }
    slot = -1;
    claimed = 0;
    return FLT_MAX;
}

__device__ __forceinline__ uint64_t cache_pack(int v, float d) {
    return ((uint64_t)(uint32_t)(v + 1) << 32) | (uint64_t)__float_as_uint(d);
}

// ---------------------------------------------------------------------------
// distances for a list of rows: w.w_v[0..m) -> w.w_d[0..m)

// Whole-row L2 prefetch as a team starts a row (measured at C3: 733k -> 744-756k
// QPS; prefetching the next round's rows as well measured 1% slower).
#ifndef SWB_ROW_PREFETCH
#define SWB_ROW_PREFETCH 1
#endif
// Rows per team and round (common.cuh team_partial_rows).  Measured at C3
// (fp16, d 1536, 40 registers, 1-chunk segments): 2 rows 877-882k QPS against
// 779-781k for one row at a time; 3 rows 792k and 4 rows 738k (more spills);
// 2 rows with 2-chunk segments 792k.
#ifndef SWB_ROWS
#define SWB_ROWS 2
#endif

// Scores the m rows listed in w.w_v into w.w_d, R * 32/TEAM rows per round:
// each team reads R rows from global memory into registers, SEG 16-byte chunks
// of each at a time, and sums them side by side (common.cuh
// team_partial_rows; a row's sum does not depend on R or SEG); the latency is
// hidden by the other warps of the SM.  Rows with w.w_slot >= 0 are published
// to the per-query table `ctab` as soon as they are scored.
// With nparts > 1 this warp takes rounds part, part + nparts, ... of them (the
// other warps of a CTA the rest).
template <int TEAM, typename XT, int R = SWB_ROWS, int SEG = SWB_LDG_SEG>
__device__ void score_rows(const Knobs& K, const WarpMem& w, int m, const float* sq, uint64_t* ctab, int lane,
                           int part = 0, int nparts = 1) {
    constexpr int P = 32 / TEAM;
    const int team = lane / TEAM, tl = lane % TEAM;
    const XT* X = reinterpret_cast<const XT*>(K.X);
    for (int base = part * R * P; base < m; base += nparts * R * P) {
        const int i0 = base + team;
        float acc[R];
        const XT* rows[R];
        int nrows = 0;
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int i = i0 + r * P;
            rows[r] = (i < m) ? X + (size_t)w.w_v[i] * K.dim : X;
            nrows += (i < m) ? 1 : 0;
        }
        if (nrows > 0) {
#if SWB_ROW_PREFETCH
            // rows longer than one segment: the later segments hit L2
            if (K.rowbytes > TEAM * SEG * 16 && tl < nrows) {
#pragma unroll
                for (int r = 0; r < R; ++r)
                    if (tl == r) prefetch_row_l2(rows[r], (uint32_t)K.rowbytes);
            }
#endif
            team_partial_rows<TEAM, XT, R, SEG>(sq, rows, nrows, K.dim, K.metric, tl, acc);
        } else {
#pragma unroll
            for (int r = 0; r < R; ++r) acc[r] = 0.f;
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const float sum = team_reduce<TEAM>(acc[r]);
            const int i = i0 + r * P;
            if (tl == 0 && i < m) {
                const float d = (K.metric == METRIC_IP) ? __fsub_rn(1.f, sum) : sum;
                w.w_d[i] = d;
                const int slot = w.w_slot[i];
                if (slot >= 0) st_volatile_u64(&ctab[slot], cache_pack(w.w_v[i], d));
            }
        }
    }
    __syncwarp();
}

// ---------------------------------------------------------------------------
// sorting

// 32 keys, one per lane, ascending by (d, id); lineage rides along
__device__ __forceinline__ void warp_sort32(float& d, int& id, int& l, int lane) {
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            const float pd = __shfl_xor_sync(FULL, d, j);
            const int pid = __shfl_xor_sync(FULL, id, j);
            const int pl = __shfl_xor_sync(FULL, l, j);
            const bool up = (lane & k) == 0;
            const bool lower = (lane & j) == 0;
            const bool take = (lower == up) ? key_lt(pd, pid, d, id) : key_lt(d, id, pd, pid);
            if (take) {
                d = pd;
                id = pid;
                l = pl;
            }
        }
    }
}

// n (a power of two, <= 128) keys in shared memory, ascending; warp-synchronous
__device__ void smem_sort(int* cid, float* cd, uint8_t* cl, int n, int lane) {
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = lane; i < n; i += 32) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const bool asc = (i & k) == 0;
                    const bool need = asc ? key_lt(cd[ixj], cid[ixj], cd[i], cid[i])
                                          : key_lt(cd[i], cid[i], cd[ixj], cid[ixj]);
                    if (need) {
                        const float td = cd[i]; cd[i] = cd[ixj]; cd[ixj] = td;
                        const int ti = cid[i]; cid[i] = cid[ixj]; cid[ixj] = ti;
                        if (cl) { const uint8_t tl = cl[i]; cl[i] = cl[ixj]; cl[ixj] = tl; }
                    }
                }
            }
            __syncwarp();
        }
    }
}

// ---------------------------------------------------------------------------
// one branch

__device__ __forceinline__ bool is_retired(const WarpMem& w, unsigned li) {
    return (w.retired[li >> 5] >> (li & 31)) & 1u;
}
__device__ __forceinline__ void set_retired(const WarpMem& w, unsigned li, int lane) {
    if (lane == 0) w.retired[li >> 5] |= (1u << (li & 31));
    __syncwarp();
}

// The selection of local_search.cu:453-511, one ballot per 32 queue slots.
__device__ int select_slot(const Knobs& K, const WarpMem& w, int lane, int ctr0, float limit, bool early) {
    const int L = K.L;
    if (K.policy == POLICY_RR && K.V > 1) {
        int slot = -1;
        for (int turn = 0; turn < K.V && slot < 0; ++turn) {
            const int want = (ctr0 + turn) % K.V;
            if (is_retired(w, (unsigned)want)) continue;
            int found = -1;
            for (int b = 0; b < L && found < 0; b += 32) {
                const int i = b + lane;
                const bool c = i < L && w.s_id[i] >= 0 && w.s_e[i] == 0 && w.s_l[i] == want;
                const unsigned msk = __ballot_sync(FULL, c);
                if (msk) found = b + __ffs(msk) - 1;
            }
            if (found < 0 || (early && w.s_d[found] > limit)) {
                set_retired(w, (unsigned)want, lane);
                continue;
            }
            slot = found;
        }
        if (slot < 0 && !early) {
            for (int b = 0; b < L; b += 32) {
                const int i = b + lane;
                const unsigned msk = __ballot_sync(FULL, i < L && w.s_id[i] >= 0 && w.s_e[i] == 0);
                if (msk) return b + __ffs(msk) - 1;
            }
        }
        return slot;
    }
    for (int b = 0; b < L; b += 32) {
        const int i = b + lane;
        bool c = false;
        if (i < L && w.s_id[i] >= 0 && w.s_e[i] == 0) c = !is_retired(w, w.s_l[i]);
        const unsigned msk = __ballot_sync(FULL, c);
        if (msk) {
            const int f = b + __ffs(msk) - 1;
            return (!early || w.s_d[f] <= limit) ? f : -1;
        }
    }
    return -1;
}

// Merge the nk sorted candidates in c_* into the queue s_* -> n_*, one output
// slot per lane at a time, by the merge-path rule of local_search.cu:637-650
// (ties between a queue entry and a candidate resolve exactly as there).
__device__ void merge_queue(const WarpMem& w, int L, int nk, int lane) {
    for (int o = lane; o < L; o += 32) {
        int lo = max(0, o - nk), hi = min(o, L);
        while (lo < hi) {
            const int i = (lo + hi) >> 1, j = o - i;
            if (j > 0 && !key_lt(w.c_d[j - 1], w.c_id[j - 1], w.s_d[i], w.s_id[i])) lo = i + 1;
            else hi = i;
        }
        const int i = lo, j = o - i;
        const bool takeA = (j >= nk) || (i < L && key_lt(w.s_d[i], w.s_id[i], w.c_d[j], w.c_id[j]));
        int id;
        float d;
        uint8_t e, l;
        if (takeA) { id = w.s_id[i]; d = w.s_d[i]; e = w.s_e[i]; l = w.s_l[i]; }
        else { id = w.c_id[j]; d = w.c_d[j]; e = 0; l = w.c_l[j]; }
        if (id < 0) { d = FLT_MAX; e = 1; l = 0; }
        w.n_id[o] = id; w.n_d[o] = d; w.n_e[o] = e; w.n_l[o] = l;
    }
}

__device__ __forceinline__ void swap_queue(WarpMem& w) {
    int* ti = w.s_id; w.s_id = w.n_id; w.n_id = ti;
    float* td = w.s_d; w.s_d = w.n_d; w.n_d = td;
    uint8_t* te = w.s_e; w.s_e = w.n_e; w.n_e = te;
    uint8_t* tl = w.s_l; w.s_l = w.n_l; w.n_l = tl;
}

// Seeds -> sorted queue (local_search.cu:318-350).  Duplicate seeds keep their
// first occurrence (the CPU reference's rule, _refcpu.py:68-74).
template <int TEAM, typename XT, int R = SWB_ROWS, int SEG = SWB_LDG_SEG>
__device__ void init_branch(const Knobs& K, WarpMem& w, int q, int j, int lane, const float* sq, Ctr& ctr) {
    int* vis = (K.H > 1) ? K.visited + ((size_t)q * K.J + j) * (size_t)K.H : nullptr;
    if (vis) {
        if (K.H >= 128) {
            int4* v4 = reinterpret_cast<int4*>(vis);
            for (int t = lane; t < K.H / 4; t += 32) v4[t] = make_int4(0, 0, 0, 0);
        } else {
            for (int t = lane; t < K.H; t += 32) vis[t] = 0;
        }
    }
    ctr.zero();
    const int V = K.V;
    int nsort = 2;
    while (nsort < V && nsort < MAXV) nsort <<= 1;
    for (int i = lane; i < nsort; i += 32) { w.c_id[i] = -1; w.c_d[i] = FLT_MAX; w.c_l[i] = 0; }
    __syncwarp();   // the clears above are ordered before the inserts below
    const int32_t* sd = K.seeds + ((size_t)q * K.J + j) * (size_t)V;
    int m = 0, fails = 0;
    for (int b = 0; b < V; b += 32) {
        const int i = b + lane;
        int s = (i < V) ? sd[i] : -1;
        if (s >= K.n) s = -1;   // an id outside the corpus is an empty slot
        bool use = s >= 0;
        for (int jj = 0; use && jj < i; ++jj) use = (sd[jj] != s);
        if (use && vis) {
            int fail = 0;
            use = visited_insert(vis, K.H, s, fail) != 0;
            fails += fail;
        }
        const unsigned msk = __ballot_sync(FULL, use);
        if (use) {
            const int pos = m + __popc(msk & lanemask_lt());
            w.w_v[pos] = s;
            w.w_slot[pos] = -1;
            w.w_aux[pos] = i;
        }
        m += __popc(msk);
    }
    for (int off = 16; off > 0; off >>= 1) fails += __shfl_xor_sync(FULL, fails, off);
    __syncwarp();
    score_rows<TEAM, XT, R, SEG>(K, w, m, sq, nullptr, lane);
    ctr.add(lane, 1, m);
    ctr.add(lane, 2, fails);
    for (int t = lane; t < m; t += 32) {
        const int si = w.w_aux[t];
        w.c_id[si] = w.w_v[t];
        w.c_d[si] = w.w_d[t];
        w.c_l[si] = (uint8_t)si;
    }
    __syncwarp();
    smem_sort(w.c_id, w.c_d, w.c_l, nsort, lane);
    for (int i = lane; i < K.L; i += 32) {
        const bool ok = (i < nsort) && (w.c_id[i] >= 0);
        w.s_id[i] = ok ? w.c_id[i] : -1;
        w.s_d[i] = ok ? w.c_d[i] : FLT_MAX;
        w.s_e[i] = ok ? 0 : 1;
        w.s_l[i] = ok ? w.c_l[i] : 0;
    }
    __syncwarp();
}

// The walk: up to `delta` expansions (local_search.cu:451-683).
// -- sign-code prefilter (local_search.cu:205-243, 560-572) ---------------
//
// <q, x> ~= alpha_x * <q, b_x> + <q, mu> with b_x in {-1, +1}^d the signs of
// x - mu, so <q, b> = 2 * (sum of q over set bits) - sum(q).  The query's two
// sums are taken once, in a fixed order (the reference adds them with float
// atomics, whose order varies).
template <typename XT>
__device__ __forceinline__ void code_query_sums(const float* sq, const float* cmu, int dim, int lane, float& qmu,
                                                float& qsum) {
    float a = 0.f, b = 0.f;
    for (int i = lane; i < dim; i += 32) {
        const float qi = sq[QLay<XT>::pos(dim, i)];
        a = __fadd_rn(a, __fmul_rn(qi, cmu[i]));
        b = __fadd_rn(b, qi);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        a = __fadd_rn(a, __shfl_xor_sync(FULL, a, off));
        b = __fadd_rn(b, __shfl_xor_sync(FULL, b, off));
    }
    qmu = a;
    qsum = b;
}

// The estimated distance 1 - <q, x> of row v, on every lane of its team.
template <int TEAM, typename XT>
__device__ __forceinline__ float code_estimate(const Knobs& K, const float* sq, int v, float qmu, float qsum,
                                               int tl) {
    const uint32_t* code = reinterpret_cast<const uint32_t*>(K.codes) + (size_t)v * K.cwords;
    float acc = 0.f;
    for (int w = tl; w < K.cwords; w += TEAM) {
        const uint32_t bits = __ldg(code + w);
        const int base = w * 32;
#pragma unroll 8
        for (int b = 0; b < 32; ++b) {
            const int i = base + b;
            if (i < K.dim && (bits >> b) & 1u) acc = __fadd_rn(acc, sq[QLay<XT>::pos(K.dim, i)]);
        }
    }
#pragma unroll
    for (int off = TEAM / 2; off > 0; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(FULL, acc, off, TEAM));
    const float ip = __fadd_rn(__fmul_rn(__ldg(K.calpha + v), __fsub_rn(__fmul_rn(2.f, acc), qsum)), qmu);
    return __fsub_rn(1.f, ip);
}

// Drops from the work list w_v/w_slot[0..m) every row whose estimate lies
// beyond `limit` by more than the margin; its vector is never read and its
// claimed table slot stays unscored.  Returns the rows kept; `skipped` gets
// the count (on every lane).
template <int TEAM, typename XT>
__device__ int code_filter(const Knobs& K, const WarpMem& w, int m, const float* sq, float limit, float qmu,
                           float qsum, int lane, int& skipped) {
    constexpr int P = 32 / TEAM;
    const int team = lane / TEAM, tl = lane % TEAM;
    for (int base = 0; base < m; base += P) {
        const int i = base + team;
        const int v = (i < m) ? w.w_v[i] : 0;
        const float est = code_estimate<TEAM, XT>(K, sq, v, qmu, qsum, tl);
        if (tl == 0 && i < m) w.w_aux[i] = (est > __fadd_rn(limit, K.cmargin)) ? 1 : 0;
    }
    __syncwarp();
    int kept = 0;
    for (int b = 0; b < m; b += 32) {
        const int i = b + lane;
        const bool keep = i < m && w.w_aux[i] == 0;
        const int v = keep ? w.w_v[i] : 0, sl = keep ? w.w_slot[i] : 0;
        const unsigned km = __ballot_sync(FULL, keep);
        __syncwarp();
        if (keep) {
            const int ps = kept + __popc(km & lanemask_lt());
            w.w_v[ps] = v;
            w.w_slot[ps] = sl;
        }
        kept += __popc(km);
        __syncwarp();
    }
    skipped = m - kept;
    return kept;
}

// CODES: compiled with the sign-code prefilter (the advance kernel, when
// codes are given); the fused search never uses it.
// NT: neighbour slots per lane (the graph degree is at most 32 * NT); 2 for
// degree <= 64 keeps half the per-neighbour registers of 4.
// HELPED: this warp is warp 0 of a CTA whose other warps score with it
// (fused_body); `help` is the CTA's shared word that hands them each step's
// row count.
template <int TEAM, typename XT, int NT, bool CODES = false, int R = SWB_ROWS, int SEG = SWB_LDG_SEG,
          bool HELPED = false>
__device__ void walk(const Knobs& K, WarpMem& w, int q, int j, int lane, const float* sq, Ctr& ctr, int delta,
                     int* help = nullptr) {
    int* vis = (K.H > 1) ? K.visited + ((size_t)q * K.J + j) * (size_t)K.H : nullptr;
    uint64_t* ctab = (K.Hc > 0) ? K.cache + (size_t)q * (size_t)K.Hc : nullptr;
    float* bnd = K.bound ? K.bound + q : nullptr;
    const int L = K.L, D = K.D;
    const int kr = K.kstop < L ? K.kstop : L;
    const bool early = K.stop_eps >= 0.f;
    const float one_eps = __fadd_rn(1.f, K.stop_eps);
    float best_k = FLT_MAX;
    int stall = 0, crowd_run = 0;
    if (lane < 8) w.retired[lane] = 0u;
    float qmu = 0.f, qsum = 0.f;
    if (CODES) code_query_sums<XT>(sq, K.cmu, K.dim, lane, qmu, qsum);
    __syncwarp();

    for (int step = 0; step < delta; ++step) {
        if (ctr.exp >= K.max_exp) break;
        float radius = (kr > 0 && w.s_id[kr - 1] >= 0) ? w.s_d[kr - 1] : FLT_MAX;
        if (bnd) {
            float gb = 0.f;
            if (lane == 0) gb = ld_volatile_f32(bnd);
            gb = __shfl_sync(FULL, gb, 0);
            if (gb < radius) radius = gb;
        }
        const float limit = (radius == FLT_MAX) ? FLT_MAX : __fmul_rn(radius, one_eps);
        const int slot = select_slot(K, w, lane, ctr.exp, limit, early);
        if (slot < 0) {
            ctr.set(lane, 3, 1);
            break;
        }
        const int p = w.s_id[slot];
        const int plin = w.s_l[slot];
        __syncwarp();
        if (lane == 0) w.s_e[slot] = 1;
        ctr.expand();

        // -- expand p: one lane per neighbour slot ------------------------
        int nv[NT], nst[NT], nsl[NT];
        float nd[NT];
        int cov = 0, nbr = 0, fails = 0, hits = 0;
        bool fresh[NT];   // passed the visited table; to be probed in the query's table
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const int nidx = lane + 32 * t;
            int v = (nidx < D) ? __ldg(&K.G[(size_t)p * D + nidx]) : -1;
            if (v >= K.n) v = -1;   // an edge outside the corpus is no edge
            nv[t] = v;
            nst[t] = 0;   // 0 none, 1 candidate with distance, 2 to be scored
            nsl[t] = -1;
            nd[t] = FLT_MAX;
            fresh[t] = false;
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const int v = nv[t];
            if (v < 0) continue;
            ++nbr;
            int isnew = 1, fail = 0;
            if (vis) isnew = visited_insert(vis, K.H, v, fail);
            fails += fail;
            if (!isnew) ++cov;
            else fresh[t] = true;
        }
        // The first probe of every fresh neighbour goes out at once (one
        // compare-and-swap each, independent); only collisions probe on.
        unsigned long long first_old[NT];
        uint32_t first_pos[NT];
        if (ctab) {
            const uint32_t cmask = (uint32_t)(K.Hc - 1);
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                if (!fresh[t]) continue;
                const uint32_t key = (uint32_t)(nv[t] + 1);
                first_pos[t] = knuth(nv[t], cmask);
                first_old[t] = atomicCAS(reinterpret_cast<unsigned long long*>(&ctab[first_pos[t]]), 0ull,
                                         ((unsigned long long)key << 32) | FLT_MAX_BITS);
            }
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            if (!fresh[t]) continue;
            const int v = nv[t];
            int cslot = -1, claimed = 0;
            float d = FLT_MAX;
            if (ctab) d = cache_probe_rest(ctab, K.Hc, v, first_pos[t], first_old[t], cslot, claimed);
            // exclusive == 1: a node another branch has scored is off limits
            // (local_search.cu:553); exclusive == 2 also treats a claim whose
            // distance is still being computed as off limits
            const bool taken = K.exclusive && cslot >= 0 && !claimed && (d != FLT_MAX || K.exclusive == 2);
            if (taken) {
                ++hits;
                ++cov;
            } else if (d == FLT_MAX) {
                nst[t] = 2;
                nsl[t] = cslot;
            } else {
                ++hits;
                nst[t] = 1;
                nd[t] = d;
            }
        }
        // Candidates for the queue: what can still enter it (at most as far as
        // its current worst; the queue does not change until the merge).  The
        // ones with a known distance go to the candidate list now and the rows
        // to score to the work list, so no per-neighbour register state lives
        // across the scoring; the list is sorted by (distance, id) before the
        // merge, so the order it is filled in does not matter.
        const float worst = (w.s_id[L - 1] >= 0) ? w.s_d[L - 1] : FLT_MAX;
        int m = 0, nk = 0, claimed_rows = 0;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const unsigned msk = __ballot_sync(FULL, nst[t] == 2);
            if (nst[t] == 2) {
                const int ps = m + __popc(msk & lanemask_lt());
                w.w_v[ps] = nv[t];
                w.w_slot[ps] = nsl[t];
            }
            m += __popc(msk);
            claimed_rows += __popc(__ballot_sync(FULL, nst[t] == 2 && nsl[t] >= 0));
            const bool keep = nst[t] == 1 && (worst == FLT_MAX || nd[t] <= worst);
            const unsigned km = __ballot_sync(FULL, keep);
            if (keep) {
                const int ps = nk + __popc(km & lanemask_lt());
                w.c_id[ps] = nv[t];
                w.c_d[ps] = nd[t];
                w.c_l[ps] = (uint8_t)plin;
            }
            nk += __popc(km);
        }
        __syncwarp();
        int fanout_extra = 0;
        if (CODES && limit != FLT_MAX && m > 0) {
            int skipped = 0;
            m = code_filter<TEAM, XT>(K, w, m, sq, limit, qmu, qsum, lane, skipped);
            claimed_rows = 0;   // recounted below from the rows actually scored
            for (int b = 0; b < m; b += 32)
                claimed_rows += __popc(__ballot_sync(FULL, b + lane < m && w.w_slot[b + lane] >= 0));
            // The reference keeps a skipped neighbour as a candidate at distance
            // FLT_MAX (local_search.cu:574-585), admitted by the keep test only
            // while the queue's last slot is empty -- where the queue's empty
            // slots, (FLT_MAX, -1), sort before it, so it never enters the queue.
            // Its one trace is the fan-out count (counter 8), kept here too.
            if (worst == FLT_MAX) fanout_extra = skipped;
        }
        if constexpr (HELPED) {
            if (lane == 0) *help = m;
            named_barrier(1, blockDim.x);   // rows listed: the CTA scores them
            score_rows<TEAM, XT, R, SEG>(K, w, m, sq, ctab, lane, 0, blockDim.x / 32);
            named_barrier(2, blockDim.x);   // every share scored
        } else {
            score_rows<TEAM, XT, R, SEG>(K, w, m, sq, ctab, lane);
        }
        for (int b = 0; b < m; b += 32) {
            const int i = b + lane;
            const float d = (i < m) ? w.w_d[i] : FLT_MAX;
            const bool keep = i < m && (worst == FLT_MAX || d <= worst);
            const unsigned km = __ballot_sync(FULL, keep);
            if (keep) {
                const int ps = nk + __popc(km & lanemask_lt());
                w.c_id[ps] = w.w_v[i];
                w.c_d[ps] = d;
                w.c_l[ps] = (uint8_t)plin;
            }
            nk += __popc(km);
        }
        for (int off = 16; off > 0; off >>= 1) {
            cov += __shfl_xor_sync(FULL, cov, off);
            nbr += __shfl_xor_sync(FULL, nbr, off);
            fails += __shfl_xor_sync(FULL, fails, off);
            hits += __shfl_xor_sync(FULL, hits, off);
        }
        ctr.add(lane, 1, m);
        ctr.add(lane, 2, fails);
        ctr.add(lane, 4, hits);
        ctr.add(lane, 5, claimed_rows);
        ctr.add(lane, 8, nk + fanout_extra);
        ctr.add(lane, 9, 1);
        __syncwarp();
        if (nk > 0) {
            if (nk <= 32) {
                float d = (lane < nk) ? w.c_d[lane] : __int_as_float(0x7f800000);
                int id = (lane < nk) ? w.c_id[lane] : 0x7fffffff;
                int l = plin;
                warp_sort32(d, id, l, lane);
                __syncwarp();
                if (lane < nk) { w.c_d[lane] = d; w.c_id[lane] = id; w.c_l[lane] = (uint8_t)l; }
            } else {
                int ms = 2;
                while (ms < nk) ms <<= 1;
                for (int i = nk + lane; i < ms; i += 32) {
                    w.c_d[i] = __int_as_float(0x7f800000);
                    w.c_id[i] = 0x7fffffff;
                    w.c_l[i] = 0;
                }
                __syncwarp();
                smem_sort(w.c_id, w.c_d, w.c_l, ms, lane);
            }
            __syncwarp();
            merge_queue(w, L, nk, lane);
            __syncwarp();
            swap_queue(w);
        }
        if (bnd && lane == 0 && kr > 0 && w.s_id[kr - 1] >= 0)
            atomicMin(reinterpret_cast<int*>(bnd), __float_as_int(w.s_d[kr - 1]));
        if (K.crowd_frac > 0.f) {
            const float cv = (nbr > 0) ? __fdiv_rn((float)cov, (float)nbr) : 0.f;
            if (cv >= K.crowd_frac) {
                if (++crowd_run >= 2) {
                    set_retired(w, (unsigned)plin, lane);
                    ctr.add(lane, 7, 1);
                    crowd_run = 0;
                }
            } else {
                crowd_run = 0;
            }
        }
        if (K.stall_patience > 0) {
            const float bk = (kr > 0 && w.s_id[kr - 1] >= 0) ? w.s_d[kr - 1] : FLT_MAX;
            if (bk < best_k) { best_k = bk; stall = 0; }
            else stall += 1;
            if (stall >= K.stall_patience) {
                ctr.set(lane, 6, 1);
                break;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// per-warp set-up and state transfer

// the query into shared memory, in the layout QLay<XT> describes
template <typename XT>
__device__ __forceinline__ void load_query(float* sq, const float* src, int dim, int tid, int nthreads) {
    const float4* s4 = reinterpret_cast<const float4*>(src);
    float4* d4 = reinterpret_cast<float4*>(sq);
    for (int t = tid; t < dim / 4; t += nthreads) d4[QLay<XT>::pos(dim, 4 * t) >> 2] = __ldg(&s4[t]);
}

__device__ void load_state(const Knobs& K, WarpMem& w, size_t bid, int lane, Ctr& ctr) {
    const size_t o = bid * (size_t)K.L;
    for (int i = lane; i < K.L; i += 32) {
        w.s_id[i] = K.ids[o + i];
        w.s_d[i] = K.dist[o + i];
        w.s_e[i] = K.expd[o + i];
        w.s_l[i] = K.lin[o + i];
    }
    ctr.mine = (lane < NCTR) ? K.counters[bid * NCTR + lane] : 0;
    ctr.exp = __shfl_sync(FULL, ctr.mine, 0);
    __syncwarp();
}

__device__ void store_state(const Knobs& K, const WarpMem& w, size_t bid, int lane, const Ctr& ctr) {
    if (K.ids) {
        const size_t o = bid * (size_t)K.L;
        for (int i = lane; i < K.L; i += 32) {
            K.ids[o + i] = w.s_id[i];
            K.dist[o + i] = w.s_d[i];
            K.expd[o + i] = w.s_e[i];
            K.lin[o + i] = w.s_l[i];
        }
    }
    if (K.counters && lane < NCTR) K.counters[bid * NCTR + lane] = ctr.value(lane);
}

// ---------------------------------------------------------------------------
// kernels

template <int TEAM, typename XT>
__global__ void __launch_bounds__(256) init_kernel(const __grid_constant__ Knobs K) {
    extern __shared__ __align__(128) char smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = blockIdx.x * K.W + warp;
    if (g >= K.Q * K.J) return;
    const int q = g / K.J, j = g % K.J;
    const Layout lay = warp_layout(K.L, K.dim * 4, K.cmax);
    WarpMem w = carve(smem + (size_t)warp * K.warp_bytes, lay);
    load_query<XT>(w.q, K.Qv + (size_t)q * K.dim, K.dim, lane, 32);
    // the per-query table and bound belong to the query; its J branches clear
    // them between them (local_search.cu:302-313)
    if (K.Hc > 0) {
        uint4* c4 = reinterpret_cast<uint4*>(K.cache + (size_t)q * K.Hc);
        const int n4 = K.Hc / 2;
        for (int t = j * 32 + lane; t < n4; t += K.J * 32) c4[t] = make_uint4(0, 0, 0, 0);
        if (K.Hc == 1 && j == 0 && lane == 0) K.cache[q] = 0ull;
    }
    if (K.bound && j == 0 && lane == 0) K.bound[q] = FLT_MAX;
    __syncwarp();
    Ctr ctr;
    init_branch<TEAM, XT>(K, w, q, j, lane, w.q, ctr);
    store_state(K, w, (size_t)q * K.J + j, lane, ctr);
}

template <int TEAM, typename XT, int NT>
__global__ void __launch_bounds__(256) advance_kernel(const __grid_constant__ Knobs K) {
    extern __shared__ __align__(128) char smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = blockIdx.x * K.W + warp;
    int flat;
    if (K.active) {
        if (g >= K.n_active) return;
        flat = K.active[g];
    } else {
        if (g >= K.Q * K.J) return;
        flat = g;
    }
    const int q = flat / K.J, j = flat % K.J;
    const Layout lay = warp_layout(K.L, K.dim * 4, K.cmax);
    WarpMem w = carve(smem + (size_t)warp * K.warp_bytes, lay);
    load_query<XT>(w.q, K.Qv + (size_t)q * K.dim, K.dim, lane, 32);
    Ctr ctr;
    load_state(K, w, (size_t)flat, lane, ctr);
    if (K.codes)
        walk<TEAM, XT, NT, true>(K, w, q, j, lane, w.q, ctr, K.delta);
    else
        walk<TEAM, XT, NT>(K, w, q, j, lane, w.q, ctr, K.delta);
    __syncwarp();
    store_state(K, w, (size_t)flat, lane, ctr);
}

// k nearest unique ids over J sorted branch lists of kk (distance, id) pairs:
// a J-way merge whose heads the warp scans with one ballot-free argmin per
// output.  Copies of an id carry identical distances, so they come out
// consecutively and all but the first are skipped.
__device__ void merge_sorted_lists(const int32_t* bi, const float* bd, int J, int kk, int k, int* head,
                                   int32_t* oi, float* od, int lane) {
    for (int t = lane; t < J; t += 32) head[t] = 0;
    __syncwarp();
    int w = 0, last = -1;
    while (w < k) {
        float bdv = __int_as_float(0x7f800000);
        int bid = 0x7fffffff, bj = -1;
        for (int t = lane; t < J; t += 32) {
            const int h = head[t];
            if (h < kk) {
                const int id = __ldcg(&bi[t * kk + h]);
                const float d = (id >= 0) ? __ldcg(&bd[t * kk + h]) : __int_as_float(0x7f800000);
                const int idk = (id >= 0) ? id : 0x7fffffff;
                if (key_lt(d, idk, bdv, bid)) { bdv = d; bid = idk; bj = t; }
            }
        }
        for (int off = 16; off > 0; off >>= 1) {
            const float pd = __shfl_xor_sync(FULL, bdv, off);
            const int pid = __shfl_xor_sync(FULL, bid, off);
            const int pj = __shfl_xor_sync(FULL, bj, off);
            if (key_lt(pd, pid, bdv, bid) || (pd == bdv && pid == bid && pj >= 0 && (bj < 0 || pj < bj))) {
                bdv = pd; bid = pid; bj = pj;
            }
        }
        if (bj < 0 || bid == 0x7fffffff) break;
        if (lane == 0) head[bj] += 1;
        __syncwarp();
        if (bid != last) {
            if (lane == 0) { oi[w] = bid; od[w] = bdv; }
            ++w;
            last = bid;
        }
    }
    for (int t = w + lane; t < k; t += 32) { oi[t] = -1; od[t] = __int_as_float(0x7f800000); }
}

// Register budget of the fused kernel: 65536 / (128 * 12) -> 40 registers a
// thread, 12 CTAs of 4 warps (4 branches) an SM.  Measured at C3 (1M x 1536
// fp16, batch 65535): occupancy buys more than the spills it costs.  With the
// whole-row L2 prefetch and one row a team, 40 registers and 3-chunk segments
// ran 767k QPS, 48 registers and 4-chunk segments 744-748k, 40 registers and
// 4-chunk segments 732k, 32 registers 710k; 80 registers (no spills) ran
// slowest of all.  Two rows a team: 40 registers 819-856k, 48 registers 852k.
// Kernel-only at C3 (65535 queries, two rows a team, 40 registers: 68.8-70.5
// ms), measured against: three rows at 48 / 64 registers 77.4 / 73.8 ms, four
// rows at 64 registers 74.9 ms, 2-chunk segments at 56 registers 73.9 ms; an
// L1 line prefetch of the next segment (loads allocating in L1) 77.6 ms; each
// lane's chunks staged through a cp.async ring in shared memory (2-8 in
// flight, 9-6 CTAs an SM) 117-133 ms.
// Threads of a fused-search CTA (4 warps: 4 branches of one query) and the
// CTAs an SM should hold; 12 CTAs of 128 threads give ptxas 40 registers a
// thread.
#ifndef SWB_FUSED_THREADS
#define SWB_FUSED_THREADS 128
#endif
#ifndef SWB_FUSED_MINB
#define SWB_FUSED_MINB 12
#endif
// Small batches: when a batch's branches (nearly) all fit on the GPU at once,
// the time is the longest branch's chain of dependent expansions, not
// bandwidth, so the wide form scores SWB_WIDE_ROWS rows a team, SWB_WIDE_SEG
// chunks of each in flight, with the registers that takes (SWB_WIDE_MINB
// CTAs an SM).  Same arithmetic, same results.
#ifndef SWB_WIDE_ROWS
#define SWB_WIDE_ROWS 8
#endif
#ifndef SWB_WIDE_SEG
#define SWB_WIDE_SEG 2
#endif
#ifndef SWB_WIDE_MINB
#define SWB_WIDE_MINB 4
#endif
// HELPED: one branch a CTA; warp 0 walks it and the other warps only score
// its rows, a share of each step's rounds, between two named barriers.
template <int TEAM, typename XT, int NT, int R, int SEG, bool HELPED = false>
__device__ __forceinline__ void fused_body(const Knobs& K) {
    extern __shared__ __align__(128) char smem[];
    __shared__ int help;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = blockIdx.y;
    const int j = HELPED ? (int)blockIdx.x : (int)blockIdx.x * K.W + warp;
    float* sq = reinterpret_cast<float*>(smem);
    const int qbytes = align16(K.dim * 4);
    load_query<XT>(sq, K.Qv + (size_t)q * K.dim, K.dim, threadIdx.x, blockDim.x);
    __syncthreads();
    if (j >= K.J) return;   // HELPED: the grid has one CTA a branch, all of them valid
    const Layout lay = warp_layout(K.L, 0, K.cmax);
    WarpMem w = carve(smem + qbytes + (HELPED ? 0 : (size_t)warp * K.warp_bytes), lay);
    if constexpr (HELPED) {
        if (warp > 0) {
            uint64_t* ctab = (K.Hc > 0) ? K.cache + (size_t)q * (size_t)K.Hc : nullptr;
            for (;;) {
                named_barrier(1, blockDim.x);
                const int m = help;
                if (m < 0) return;   // the walk is over
                score_rows<TEAM, XT, R, SEG>(K, w, m, sq, ctab, lane, warp, blockDim.x / 32);
                named_barrier(2, blockDim.x);
            }
        }
    }
    Ctr ctr;
    init_branch<TEAM, XT, R, SEG>(K, w, q, j, lane, sq, ctr);
    walk<TEAM, XT, NT, false, R, SEG, HELPED>(K, w, q, j, lane, sq, ctr, K.max_exp, &help);
    if constexpr (HELPED) {
        if (lane == 0) help = -1;
        named_barrier(1, blockDim.x);   // releases the helpers
    }
    __syncwarp();
    const size_t bid = (size_t)q * K.J + j;
    store_state(K, w, bid, lane, ctr);
    for (int t = lane; t < K.kk; t += 32) {
        K.branch_ids[bid * K.kk + t] = w.s_id[t];
        K.branch_dist[bid * K.kk + t] = w.s_d[t];
    }
    __threadfence();
    __syncwarp();
    int last = 0;
    if (lane == 0) last = (atomicAdd(&K.qdone[q], 1) == K.J - 1);
    last = __shfl_sync(FULL, last, 0);
    if (!last) return;
    __threadfence();
    // the walk is over: w_v .. w_aux (4 * cmax >= J ints, contiguous) hold the heads
    merge_sorted_lists(K.branch_ids + (size_t)q * K.J * K.kk, K.branch_dist + (size_t)q * K.J * K.kk, K.J, K.kk,
                       K.k, w.w_v, K.out_ids + (size_t)q * K.k, K.out_dist + (size_t)q * K.k, lane);
}

template <int TEAM, typename XT, int NT>
__global__ void __launch_bounds__(SWB_FUSED_THREADS, SWB_FUSED_MINB) fused_kernel(const __grid_constant__ Knobs K) {
    fused_body<TEAM, XT, NT, SWB_ROWS, SWB_LDG_SEG>(K);
}

template <int TEAM, typename XT, int NT>
__global__ void __launch_bounds__(SWB_FUSED_THREADS, SWB_WIDE_MINB) fused_wide_kernel(const __grid_constant__ Knobs K) {
    fused_body<TEAM, XT, NT, SWB_WIDE_ROWS, SWB_WIDE_SEG>(K);
}

template <int TEAM, typename XT, int NT>
__global__ void __launch_bounds__(SWB_FUSED_THREADS, SWB_WIDE_MINB) fused_help_kernel(const __grid_constant__ Knobs K) {
    fused_body<TEAM, XT, NT, SWB_WIDE_ROWS, SWB_WIDE_SEG, true>(K);
}

__global__ void prepare_kernel(int Q, uint64_t* cache, int64_t cache_words, float* bound, int32_t* qdone) {
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    if (cache) {
        uint4* c4 = reinterpret_cast<uint4*>(cache);
        for (int64_t t = tid; t < cache_words / 2; t += stride) c4[t] = make_uint4(0, 0, 0, 0);
        if ((cache_words & 1) && tid == 0) cache[cache_words - 1] = 0ull;
    }
    for (int64_t t = tid; t < Q; t += stride) {
        if (bound) bound[t] = FLT_MAX;
        if (qdone) qdone[t] = 0;
    }
}

// Standalone merge (local_search.cu:863-919): any [Q, J, kk] input; one block
// per query sorts the padded set by (distance, id) and keeps the first copy
// of each id.
__global__ void __launch_bounds__(256) merge_kernel(const int32_t* __restrict__ bi, const float* __restrict__ bd,
                                                    int n, int k, int padded, int32_t* oi, float* od) {
    extern __shared__ __align__(128) char smem[];
    float* sd = reinterpret_cast<float*>(smem);
    int* si = reinterpret_cast<int*>(sd + padded);
    const int q = blockIdx.x;
    const size_t base = (size_t)q * n;
    for (int i = threadIdx.x; i < padded; i += blockDim.x) {
        const int id = (i < n) ? bi[base + i] : -1;
        si[i] = (id >= 0) ? id : 0x7fffffff;
        sd[i] = (id >= 0) ? bd[base + i] : __int_as_float(0x7f800000);
    }
    __syncthreads();
    for (int size = 2; size <= padded; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < padded; i += blockDim.x) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool up = (i & size) == 0;
                    const bool lt = key_lt(sd[i], si[i], sd[j], si[j]);
                    if (up != lt) {
                        const float td = sd[i]; sd[i] = sd[j]; sd[j] = td;
                        const int ti = si[i]; si[i] = si[j]; si[j] = ti;
                    }
                }
            }
            __syncthreads();
        }
    }
    if (threadIdx.x == 0) {
        int w = 0;
        for (int i = 0; i < n && w < k; ++i) {
            if (si[i] == 0x7fffffff) break;
            if (i > 0 && si[i] == si[i - 1]) continue;
            oi[(size_t)q * k + w] = si[i];
            od[(size_t)q * k + w] = sd[i];
            ++w;
        }
        for (; w < k; ++w) {
            oi[(size_t)q * k + w] = -1;
            od[(size_t)q * k + w] = __int_as_float(0x7f800000);
        }
    }
}

}  // namespace swb

// ===========================================================================
// host side

using namespace swb;

namespace {

int esize_of(int x_dtype) { return x_dtype == 0 ? 4 : 2; }

int pow2_at_least(int x) {
    int p = 1;
    while (p < x) p <<= 1;
    return p;
}

int common_checks(const void* X, int x_dtype, int64_t n, int dim, int team, int L) {
    if (!X) return abi::fail(SWB_ERR_ARG, "X is null");
    if (x_dtype != SWB_F32 && x_dtype != SWB_F16) return abi::fail(SWB_ERR_ARG, "X must be float32 or float16");
    if (n <= 0 || dim <= 0) return abi::fail(SWB_ERR_ARG, "empty corpus");
    const int vec = 16 / esize_of(x_dtype);
    if (dim % vec)
        return abi::fail(SWB_ERR_ARG, "the dimension must be a multiple of %d for %s rows (16-byte row chunks); "
                                      "pad the vectors with zeros",
                         vec, x_dtype == 0 ? "float32" : "float16");
    if (reinterpret_cast<uintptr_t>(X) % 16) return abi::fail(SWB_ERR_ARG, "X must be 16-byte aligned");
    if (team != 4 && team != 8 && team != 16 && team != 32)
        return abi::fail(SWB_ERR_TEAM, "team_size must be 4, 8, 16 or 32");
    if (L < 1 || L > MAXL) return abi::fail(SWB_ERR_ARG, "L exceeds MAXL (%d)", MAXL);
    return SWB_OK;
}

bool pow2(int x) { return x > 0 && (x & (x - 1)) == 0; }

template <typename KernelT>
int launch(KernelT kern, dim3 grid, int threads, size_t smem, cudaStream_t st, const Knobs& K) {
    if ((long long)smem > abi::max_smem_optin())
        return abi::fail(SWB_ERR_SMEM, "the search needs %zu B of shared memory per block; the device allows %d. "
                                       "Lower L or the dimension.",
                         smem, abi::max_smem_optin());
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return abi::cuda_fail(e, "cudaFuncSetAttribute");
    }
    kern<<<grid, threads, smem, st>>>(K);
    return abi::cuda_check("search kernel launch");
}

// the query's shared-memory bytes (common.cuh QLay)
int query_bytes(int dim) { return align16(4 * dim); }

// neighbour slots per lane for a graph of degree D (walk's NT)
int slots_for(int D) { return D <= 64 ? 2 : 4; }

#define SWB_CASE(KERNEL, T, TEAMV, DT, ...)                                                    \
    if ((TEAMV) == T)                                                                          \
        return ((DT) == SWB_F32) ? launch(KERNEL<T, float>, __VA_ARGS__)                       \
                                 : launch(KERNEL<T, __half>, __VA_ARGS__);
#define SWB_DISPATCH(KERNEL, TEAMV, DT, ...)                                                   \
    [&]() -> int {                                                                             \
        SWB_CASE(KERNEL, 4, TEAMV, DT, __VA_ARGS__)                                            \
        SWB_CASE(KERNEL, 8, TEAMV, DT, __VA_ARGS__)                                            \
        SWB_CASE(KERNEL, 16, TEAMV, DT, __VA_ARGS__)                                           \
        SWB_CASE(KERNEL, 32, TEAMV, DT, __VA_ARGS__)                                           \
        return abi::fail(SWB_ERR_TEAM, "team_size must be 4, 8, 16 or 32");                   \
    }()
#define SWB_CASE_NT(KERNEL, T, N, TEAMV, NTV, DT, ...)                                         \
    if ((TEAMV) == T && (NTV) == N)                                                            \
        return ((DT) == SWB_F32) ? launch(KERNEL<T, float, N>, __VA_ARGS__)                    \
                                 : launch(KERNEL<T, __half, N>, __VA_ARGS__);
#define SWB_DISPATCH_NT(KERNEL, TEAMV, NTV, DT, ...)                                           \
    [&]() -> int {                                                                             \
        SWB_CASE_NT(KERNEL, 4, 2, TEAMV, NTV, DT, __VA_ARGS__)                                 \
        SWB_CASE_NT(KERNEL, 4, 4, TEAMV, NTV, DT, __VA_ARGS__)                                 \
        SWB_CASE_NT(KERNEL, 8, 2, TEAMV, NTV, DT, __VA_ARGS__)                                 \
        SWB_CASE_NT(KERNEL, 8, 4, TEAMV, NTV, DT, __VA_ARGS__)                                 \
        SWB_CASE_NT(KERNEL, 16, 2, TEAMV, NTV, DT, __VA_ARGS__)                                \
        SWB_CASE_NT(KERNEL, 16, 4, TEAMV, NTV, DT, __VA_ARGS__)                                \
        SWB_CASE_NT(KERNEL, 32, 2, TEAMV, NTV, DT, __VA_ARGS__)                                \
        SWB_CASE_NT(KERNEL, 32, 4, TEAMV, NTV, DT, __VA_ARGS__)                                \
        return abi::fail(SWB_ERR_TEAM, "team_size must be 4, 8, 16 or 32");                   \
    }()


// cmax bounds what one step handles: D candidates, V seeds, and (fused) the
// J branch heads of the final merge, which reuse 4 * cmax ints
void fill_common(Knobs& K, const void* X, int x_dtype, int64_t n, int dim, int team, int L, bool q_shared, int D,
                int V, int J) {
    std::memset(&K, 0, sizeof(K));
    K.X = X;
    K.n = n;
    K.dim = dim;
    K.rowbytes = dim * esize_of(x_dtype);
    K.L = L;
    K.codes = nullptr; K.calpha = nullptr; K.cmu = nullptr; K.cmargin = 0.f; K.cwords = 0;
    K.q_shared = q_shared ? 1 : 0;
    int cm = pow2_at_least(D > V ? D : V);
    const int jq = (J + 3) / 4;
    if (cm < jq) cm = pow2_at_least(jq);
    if (cm < 32) cm = 32;
    K.cmax = cm;
    const Layout lay = warp_layout(L, q_shared ? 0 : query_bytes(dim), cm);
    K.warp_bytes = lay.total;
}

}  // namespace

extern "C" int swb_search_init(const void* X, int x_dtype, int64_t n, int dim, const float* Qv,
                               const int32_t* seeds, int Q, int J, int V, int32_t* ids, float* dist,
                               uint8_t* expanded, uint8_t* lineage, int L, int32_t* visited, int H,
                               int32_t* counters, int metric, int team, uint64_t* cache, int Hc, float* bound,
                               void* stream) {
    int rc = common_checks(X, x_dtype, n, dim, team, L);
    if (rc) return rc;
    if (Q <= 0 || J <= 0) return SWB_OK;
    if (Q > SWB_MAX_BATCH)
        return abi::fail(SWB_ERR_BATCH, "batch of %d queries exceeds the 65535 one call allows; split the batch", Q);
    if (V < 1 || V > MAXV) return abi::fail(SWB_ERR_ARG, "seeds per branch must be 1..%d", MAXV);
    if (!pow2(H)) return abi::fail(SWB_ERR_ARG, "visited table size must be a power of two");
    if (Hc > 0 && !pow2(Hc)) return abi::fail(SWB_ERR_ARG, "cache size must be a power of two");
    if (!Qv || !seeds || !ids || !dist || !expanded || !lineage || !counters || (H > 1 && !visited))
        return abi::fail(SWB_ERR_ARG, "null state buffer");
    Knobs K;
    fill_common(K, X, x_dtype, n, dim, team, L, false, 1, V, 0);
    K.Qv = Qv; K.seeds = seeds; K.ids = ids; K.dist = dist; K.expd = expanded; K.lin = lineage;
    K.Q = Q; K.J = J; K.V = V; K.visited = visited; K.H = H; K.counters = counters;
    K.metric = metric; K.cache = Hc > 0 ? cache : nullptr; K.Hc = Hc > 0 ? Hc : 0; K.bound = bound;
    K.W = 4;
    const long long warps = (long long)Q * J;
    dim3 grid((unsigned)((warps + K.W - 1) / K.W));
    const size_t smem = (size_t)K.W * K.warp_bytes;
    return SWB_DISPATCH(init_kernel, team, x_dtype, grid, K.W * 32, smem, (cudaStream_t)stream, K);
}

extern "C" int swb_search_advance(const void* X, int x_dtype, int64_t n, int dim, const int32_t* G, int D,
                                  const float* Qv, int32_t* ids, float* dist, uint8_t* expanded, uint8_t* lineage,
                                  int Q, int J, int L, int32_t* visited, int H, int32_t* counters, int metric,
                                  int team, int delta, int max_expansions, int policy, int V, float stop_eps,
                                  int kstop, uint64_t* cache, int Hc, float* bound, int exclusive,
                                  int stall_patience, float crowd_frac, const int32_t* active, int n_active,
                                  const int32_t* codes, const float* code_alpha, const float* code_mu,
                                  float code_margin, int code_words, int32_t* status, void* stream) {
    int rc = common_checks(X, x_dtype, n, dim, team, L);
    if (rc) return rc;
    if (!G || D < 1 || D > MAXD) return abi::fail(SWB_ERR_ARG, "graph degree must be 1..%d", MAXD);
    if (V > 256) return abi::fail(SWB_ERR_ARG, "lineage count exceeds 256 (lineage is a uint8)");
    if (codes) {
        if (!code_alpha || !code_mu) return abi::fail(SWB_ERR_ARG, "codes need their scales and the corpus mean");
        if (metric != SWB_METRIC_IP) return abi::fail(SWB_ERR_ARG, "the sign-code prefilter is inner product only");
        if (code_words != (dim + 31) / 32) return abi::fail(SWB_ERR_ARG, "codes must have ceil(dim / 32) words a row");
    }
    if (!pow2(H)) return abi::fail(SWB_ERR_ARG, "visited table size must be a power of two");
    if (Hc > 0 && !pow2(Hc)) return abi::fail(SWB_ERR_ARG, "cache size must be a power of two");
    if (Q <= 0 || J <= 0 || delta <= 0) return SWB_OK;
    if (active && n_active <= 0) return SWB_OK;
    Knobs K;
    fill_common(K, X, x_dtype, n, dim, team, L, false, D, 1, 0);
    K.G = G; K.D = D; K.Qv = Qv; K.ids = ids; K.dist = dist; K.expd = expanded; K.lin = lineage;
    K.Q = Q; K.J = J; K.V = V < 1 ? 1 : V; K.visited = visited; K.H = H; K.counters = counters;
    K.metric = metric; K.delta = delta; K.max_exp = max_expansions; K.policy = policy;
    K.stop_eps = stop_eps; K.kstop = kstop;
    K.cache = Hc > 0 ? cache : nullptr; K.Hc = Hc > 0 ? Hc : 0; K.bound = bound;
    K.exclusive = Hc > 0 ? exclusive : 0;
    K.stall_patience = stall_patience; K.crowd_frac = crowd_frac;
    K.active = active; K.n_active = active ? n_active : 0; K.status = status;
    K.codes = codes; K.calpha = code_alpha; K.cmu = code_mu; K.cmargin = code_margin;
    K.cwords = codes ? code_words : 0;
    K.W = 4;
    const long long warps = active ? (long long)n_active : (long long)Q * J;
    dim3 grid((unsigned)((warps + K.W - 1) / K.W));
    const size_t smem = (size_t)K.W * K.warp_bytes;
    return SWB_DISPATCH_NT(advance_kernel, team, slots_for(D), x_dtype, grid, K.W * 32, smem, (cudaStream_t)stream, K);
}

extern "C" int swb_search_prepare(int Q, uint64_t* cache, int Hc, float* bound, int32_t* qdone, void* stream) {
    if (Q <= 0) return SWB_OK;
    if (Hc > 0 && !cache) return abi::fail(SWB_ERR_ARG, "cache is null");
    const int64_t words = (Hc > 0) ? (int64_t)Q * Hc : 0;
    const int64_t work = words / 2 > Q ? words / 2 : Q;
    int blocks = (int)((work + 255) / 256);
    const int cap = abi::num_sms() * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    prepare_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(Q, Hc > 0 ? cache : nullptr, words, bound, qdone);
    return abi::cuda_check("prepare kernel launch");
}

extern "C" int swb_search_fused(const void* X, int x_dtype, int64_t n, int dim, const int32_t* G, int D,
                                const float* Qv, const int32_t* seeds, int Q, int J, int V, int k, int L, int B,
                                int metric, int team, int policy, float stop_eps, int kstop, int32_t* visited,
                                int H, uint64_t* cache, int Hc, float* bound, int exclusive, int stall_patience,
                                float crowd_frac, int32_t* branch_ids, float* branch_dist, int32_t* qdone,
                                int32_t* out_ids, float* out_dist, int32_t* ids, float* dist, uint8_t* expanded,
                                uint8_t* lineage, int32_t* counters, int32_t* status, void* stream) {
    int rc = common_checks(X, x_dtype, n, dim, team, L);
    if (rc) return rc;
    if (!G || D < 1 || D > MAXD) return abi::fail(SWB_ERR_ARG, "graph degree must be 1..%d", MAXD);
    if (Q > SWB_MAX_BATCH)
        return abi::fail(SWB_ERR_BATCH, "batch of %d queries exceeds the 65535 one call allows; split the batch", Q);
    if (V < 1 || V > MAXV) return abi::fail(SWB_ERR_ARG, "seeds per branch must be 1..%d", MAXV);
    if (!pow2(H)) return abi::fail(SWB_ERR_ARG, "visited table size must be a power of two");
    if (Hc > 0 && !pow2(Hc)) return abi::fail(SWB_ERR_ARG, "cache size must be a power of two");
    if (k < 1) return abi::fail(SWB_ERR_ARG, "k must be positive");
    if (!branch_ids || !branch_dist || !qdone || !out_ids || !out_dist || !seeds || !Qv)
        return abi::fail(SWB_ERR_ARG, "null buffer");
    if (Q <= 0 || J <= 0) return SWB_OK;
    if ((ids || dist || expanded || lineage) && !(ids && dist && expanded && lineage))
        return abi::fail(SWB_ERR_ARG, "state outputs must be all given or all null");
    Knobs K;
    if (J > 4 * MAXD) return abi::fail(SWB_ERR_ARG, "at most %d branches per query", 4 * MAXD);
    fill_common(K, X, x_dtype, n, dim, team, L, true, D, V, J);
    K.G = G; K.D = D; K.Qv = Qv; K.seeds = seeds;
    K.ids = ids; K.dist = dist; K.expd = expanded; K.lin = lineage;
    K.Q = Q; K.J = J; K.V = V; K.visited = visited; K.H = H; K.counters = counters;
    K.metric = metric; K.max_exp = B; K.delta = B; K.policy = policy; K.stop_eps = stop_eps; K.kstop = kstop;
    K.cache = Hc > 0 ? cache : nullptr; K.Hc = Hc > 0 ? Hc : 0; K.bound = bound;
    K.exclusive = Hc > 0 ? exclusive : 0;
    K.stall_patience = stall_patience; K.crowd_frac = crowd_frac;
    K.status = status; K.k = k; K.kk = k < L ? k : L;
    K.branch_ids = branch_ids; K.branch_dist = branch_dist; K.qdone = qdone;
    K.out_ids = out_ids; K.out_dist = out_dist;
    // The smallest batches, up to four waves of one branch a CTA: the CTA's
    // other warps help its branch score rows.  Measured at C3 (team 16, 128
    // branches): batch 1-16 ran 9-21% faster than the wide form below, batch
    // 64 (8192 CTAs) 32% slower.
    const long long help_max = abi::env_int("SWB_HELP_CTAS", abi::num_sms() * SWB_WIDE_MINB * 4);
    if ((long long)Q * J <= help_max) {
        K.W = 1;
        dim3 grid((unsigned)J, (unsigned)Q);
        const size_t smem = (size_t)query_bytes(dim) + (size_t)K.warp_bytes;
        return SWB_DISPATCH_NT(fused_help_kernel, team, slots_for(D), x_dtype, grid, SWB_FUSED_THREADS, smem,
                               (cudaStream_t)stream, K);
    }
    int W = abi::env_int("SWB_WARPS", SWB_FUSED_THREADS / 32);
    if (W > J) W = J;
    if (W < 1) W = 1;
    if (W > SWB_FUSED_THREADS / 32) W = SWB_FUSED_THREADS / 32;
    K.W = W;
    dim3 grid((unsigned)((J + W - 1) / W), (unsigned)Q);
    const size_t smem = (size_t)query_bytes(dim) + (size_t)W * K.warp_bytes;
    // the wide form up to four of its waves: measured at C3 (team 16), 2048
    // CTAs ran 21-23% faster wide (batch 64 x 128 branches, 128 x 64), 8192
    // CTAs 15% slower (batch 512 x 64); batch 1-16 x 128 branches 25-31% faster
    const long long ctas = (long long)grid.x * grid.y;
    const long long wide_max = abi::env_int("SWB_WIDE_CTAS", abi::num_sms() * SWB_WIDE_MINB * 4);
    if (ctas <= wide_max)
        return SWB_DISPATCH_NT(fused_wide_kernel, team, slots_for(D), x_dtype, grid, W * 32, smem,
                               (cudaStream_t)stream, K);
    return SWB_DISPATCH_NT(fused_kernel, team, slots_for(D), x_dtype, grid, W * 32, smem, (cudaStream_t)stream, K);
}

extern "C" int swb_merge_branches(const int32_t* bids, const float* bdist, int Q, int J, int kk, int k,
                                  int32_t* out_ids, float* out_dist, void* stream) {
    if (Q <= 0) return SWB_OK;
    const int n = J * kk;
    if (k < 1 || k > n) return abi::fail(SWB_ERR_ARG, "k must be in 1..J*kk");
    int padded = 1;
    while (padded < n) padded <<= 1;
    const size_t smem = (size_t)padded * 8;
    if ((long long)smem > abi::max_smem_optin())
        return abi::fail(SWB_ERR_SMEM, "merge needs %zu B of shared memory for %d candidates", smem, n);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return abi::cuda_fail(e, "cudaFuncSetAttribute");
    }
    merge_kernel<<<Q, 256, smem, (cudaStream_t)stream>>>(bids, bdist, n, k, padded, out_ids, out_dist);
    return abi::cuda_check("merge kernel launch");
}

// ===========================================================================
// The fused search without caller-provided scratch.
//
// Some callers cannot hand this library device buffers for its scratch: a host
// runtime whose memory manager owns the whole device heap and forbids raw
// cudaMalloc calls, or a latency-critical serving thread that must never call
// into an allocator (an allocation can synchronise the device and stall the
// request).  swb_search_fused_static serves them: it runs the same fused search
// kernel, but everything the search needs besides its inputs and outputs --
// per-query distance tables, bounds and completion counters, per-branch result
// lists, per-branch visited tables -- lives in one fixed array compiled into
// the library.  It calls no allocation routine of any kind.

namespace {

constexpr size_t kStaticScratchBytes = (size_t)SWB_STATIC_SCRATCH_BYTES;

// Every GPU that loads this library holds this array until the process exits.
static __device__ __align__(256) unsigned char swb_static_scratch[kStaticScratchBytes];

std::mutex g_static_mu;
void* g_static_ptr[64] = {nullptr};   // device address of the array, per device ordinal

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// The array's device address on the current device.  The first call on a
// device looks it up (cudaGetSymbolAddress, with that device current).
int static_scratch_ptr(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return abi::cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= 64) return abi::fail(SWB_ERR_ARG, "device ordinal %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_static_mu);
    if (!g_static_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, swb_static_scratch);
        if (e != cudaSuccess) return abi::cuda_fail(e, "cudaGetSymbolAddress(static scratch)");
        g_static_ptr[dev] = p;
    }
    *out = g_static_ptr[dev];
    return SWB_OK;
}

}  // namespace

// Per-branch visited-table slots of the fixed-scratch search: 1 when elided,
// else the next power of two >= 2 (1 + B D), computed in 64 bits; 0 when the
// knobs are out of range (B or D not positive, D beyond the kernel's limit, or
// a table beyond 2^30 slots), which every caller turns into a rejection.
int64_t static_visited_slots(int B, int D, bool elide) {
    if (B < 1 || D < 1 || D > MAXD) return 0;
    if (elide) return 1;
    const int64_t want = 2 * (1 + (int64_t)B * (int64_t)D);
    if (want > ((int64_t)1 << 30)) return 0;
    int64_t p = 1;
    while (p < want) p <<= 1;
    return p;
}

extern "C" uint64_t swb_search_static_bytes(int Q, int J, int k, int L, int B, int D, int Hc, int shared_cache,
                                            int exclusive, int elide_visited) {
    if (Q < 0 || J < 0 || k < 1 || L < 1 || Hc < 0) return UINT64_MAX;
    const int kk = k < L ? k : L;
    const bool table = shared_cache && J > 1 && Hc > 0;
    const bool elide = elide_visited && exclusive && table;
    const int64_t H = static_visited_slots(B, D, elide);
    if (H == 0) return UINT64_MAX;
    size_t b = 0;
    b += align256((size_t)Q * 4);                           // completion counters
    b += align256((size_t)Q * 4);                           // bounds
    b += align256((size_t)Q * J * kk * 4) * 2;              // per-branch ids, distances
    if (table) b += align256((size_t)Q * Hc * 8);           // distance tables
    if (H > 1) b += align256((size_t)Q * J * H * 4);        // visited tables
    return b;
}

extern "C" int swb_search_fused_static(const void* X, int x_dtype, int64_t n, int dim, const int32_t* G, int D,
                                       const float* Qv, const int32_t* seeds, int Q, int J, int k, int L, int B,
                                       int metric, int team, float stop_eps, int shared_cache, int shared_bound,
                                       int exclusive, int elide_visited, int Hc, int32_t* out_ids, float* out_dist,
                                       int32_t* status, void* stream) {
    if (Q <= 0 || J <= 0) return SWB_OK;
    if (Hc > 0 && !pow2(Hc)) return abi::fail(SWB_ERR_ARG, "table size must be a power of two");
    if (k < 1 || L < 1 || B < 1 || D < 1) return abi::fail(SWB_ERR_ARG, "k, L, B and D must be positive");
    if (D > MAXD) return abi::fail(SWB_ERR_ARG, "graph degree must be 1..%d", MAXD);
    if (L > MAXL) return abi::fail(SWB_ERR_ARG, "L exceeds MAXL (%d)", MAXL);
    if (Q > SWB_MAX_BATCH)
        return abi::fail(SWB_ERR_BATCH, "batch of %d queries exceeds the 65535 one call allows; split the batch", Q);
    if (J > 4 * MAXD) return abi::fail(SWB_ERR_ARG, "at most %d branches per query", 4 * MAXD);
    const uint64_t need = swb_search_static_bytes(Q, J, k, L, B, D, Hc, shared_cache, exclusive, elide_visited);
    if (need == UINT64_MAX)
        return abi::fail(SWB_ERR_ARG, "the budget B = %d with degree D = %d needs a visited table beyond 2^30 slots",
                         B, D);
    if (need > kStaticScratchBytes)
        return abi::fail(SWB_ERR_ARG,
                         "this search needs %llu bytes of scratch; the library's fixed scratch holds %llu. "
                         "Search fewer queries per call or use a smaller table.",
                         (unsigned long long)need, (unsigned long long)kStaticScratchBytes);
    void* base = nullptr;
    int rc = static_scratch_ptr(&base);
    if (rc) return rc;
    const int kk = k < L ? k : L;
    const bool table = shared_cache && J > 1 && Hc > 0;
    const bool elide = elide_visited && exclusive && table;
    const int H = (int)static_visited_slots(B, D, elide);   // in range: the size check above passed
    char* p = static_cast<char*>(base);
    int32_t* qdone = reinterpret_cast<int32_t*>(p); p += align256((size_t)Q * 4);
    float* bound = reinterpret_cast<float*>(p); p += align256((size_t)Q * 4);
    int32_t* bids = reinterpret_cast<int32_t*>(p); p += align256((size_t)Q * J * kk * 4);
    float* bdist = reinterpret_cast<float*>(p); p += align256((size_t)Q * J * kk * 4);
    uint64_t* cache = nullptr;
    if (table) { cache = reinterpret_cast<uint64_t*>(p); p += align256((size_t)Q * Hc * 8); }
    int32_t* visited = nullptr;
    if (H > 1) { visited = reinterpret_cast<int32_t*>(p); p += align256((size_t)Q * J * H * 4); }
    cudaStream_t st = (cudaStream_t)stream;
    // What a previous call left behind is cleared on this stream first: the
    // tables, bounds and completion counters must start empty (the visited
    // tables and branch lists are rewritten by the kernel before use).
    rc = swb_search_prepare(Q, table ? cache : nullptr, table ? Hc : 0, shared_bound && J > 1 ? bound : nullptr,
                            qdone, stream);
    if (rc) return rc;
    return swb_search_fused(X, x_dtype, n, dim, G, D, Qv, seeds, Q, J, 1, k, L, B, metric, team, 0, stop_eps, k,
                            visited, H, cache, table ? Hc : 0, shared_bound && J > 1 ? bound : nullptr,
                            table ? exclusive : 0, 0, 0.f, bids, bdist, qdone, out_ids, out_dist, nullptr, nullptr,
                            nullptr, nullptr, nullptr, status, st);
}
