// sweep_mma.cu -- the exact candidate sweep on the 5th-generation tensor cores.
//
// Replaces knn_candidates (swann/build.py:30-43): for a block of rows, the C
// nearest rows of the whole corpus by the metric, with the X x X^T tiles on
// tcgen05 and the per-row top-C selection fused into the epilogue, so the
// n x n distance matrix never exists.
//
// One CTA owns 128 rows (the 128 TMEM lanes) and sweeps every column tile:
//   warp 0      TMA producer: 128B-swizzled tiles of the row block (A) and of
//               the column tile (B) into a ring of shared-memory stages;
//   warp 1      MMA issuer: tcgen05.mma into one of two TMEM accumulators
//               (BN fp32 columns each), committing each stage back to the
//               producer and each finished tile to the epilogue;
//   warps 2..5  epilogue: tcgen05.ld (one thread per row), distance, a filter
//               against the row's current C-th best, a small per-row buffer
//               in shared memory, and a merge into the row's sorted best list
//               (global scratch) when the buffer fills.
// The second accumulator lets the MMAs of tile t+1 run while the epilogue
// reads tile t.
//
// Arithmetic.  fp16 rows (MODE_F16): kind::f16, fp16 x fp16 products are exact
// in fp32, accumulation in fp32.  fp32 rows (MODE_TF32X3): each operand is
// split host-side into hi = tf32(x) and lo = x - hi; the accumulator gets
// hi*hi + hi*lo + lo*hi (kind::tf32), which carries about 2^-22 relative error
// per product, the fp32-faithful 3xTF32 scheme.  The distance expressions are
// the reference's: 1 - <a,b> (ip), max((|b|^2 - 2<a,b>) + |a|^2, 0) (l2).
//
// All mbarrier waits are bounded; a wait that runs out raises a status word and
// the CTA winds down (TMEM is released in every path).

#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>

#include "abi_util.h"
#include "common.cuh"
#include "tcgen05.cuh"

namespace swb {
namespace sweep {

constexpr int BM = 128;
constexpr int ROW_BYTES = 128;   // one 128B swizzle atom of K per row per stage
constexpr int NTHREADS = 192;
constexpr int BUF = 31;          // per-row candidate buffer (shared memory), <= 32
constexpr int GROUP = 16;        // columns filtered between two flush checks
constexpr float SELF = 3.4e38f;

enum Mode { MODE_F16 = 0, MODE_TF32X3 = 1 };

template <int MODE>
struct Cfg;
template <>
struct Cfg<MODE_F16> {
    static constexpr int BN = 256;
    static constexpr int STAGES = 4;
    static constexpr int KSUB = 4;              // MMAs of K = 16 per 64-element stage
    static constexpr int NOPS = 1;              // operand pairs per stage
    static constexpr uint32_t FMT = 0;          // F16
};
template <>
struct Cfg<MODE_TF32X3> {
    static constexpr int BN = 128;
    static constexpr int STAGES = 3;
    static constexpr int KSUB = 4;              // MMAs of K = 8 per 32-element stage
    static constexpr int NOPS = 2;              // hi and lo of A and of B
    static constexpr uint32_t FMT = 2;          // TF32
};

// -- PTX wrappers ------------------------------------------------------------

template <int MODE>
__device__ __forceinline__ void umma(uint32_t dtm, uint64_t ad, uint64_t bd, uint32_t idesc, uint32_t acc) {
    if constexpr (MODE == MODE_F16) {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(dtm),
            "l"(ad), "l"(bd), "r"(idesc), "r"(acc)
            : "memory");
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(dtm),
            "l"(ad), "l"(bd), "r"(idesc), "r"(acc)
            : "memory");
    }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

// -- a CTA pair (cluster of 2) sharing one M = 256 MMA ------------------------
//
// The leader (rank 0) issues tcgen05.mma.cta_group::2: A's 256 rows come 128
// from each CTA's shared memory, B's N columns N/2 from each, and each CTA's
// TMEM receives its own 128 rows x N.  Both CTAs load their halves with TMA
// into their own shared memory and complete the transaction on the leader's
// barrier; the leader's commits arrive on the matching barrier of both CTAs.
// Every TMA load reads this GPU's memory into its own CTA only.

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// the shared::cluster address of this CTA's `p` in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
    uint32_t a;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
    return a;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cbar) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cbar) : "memory");
}
__device__ __forceinline__ void tmem_alloc2(uint32_t* dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish2() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// TMA tile into this CTA's shared memory, completing on a barrier that may be
// the leader's (cbar: a shared::cluster address)
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, int c0, int c1, uint32_t cbar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
        "%3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(cbar)
        : "memory");
}
template <int MODE>
__device__ __forceinline__ void umma_pair(uint32_t dtm, uint64_t ad, uint64_t bd, uint32_t idesc, uint32_t acc) {
    if constexpr (MODE == MODE_F16) {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(dtm),
            "l"(ad), "l"(bd), "r"(idesc), "r"(acc)
            : "memory");
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(dtm),
            "l"(ad), "l"(bd), "r"(idesc), "r"(acc)
            : "memory");
    }
}
// completion of this CTA pair's MMAs so far, to the barrier at the same
// shared-memory offset in both CTAs (a commit, not a load)
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"((uint16_t)0x3)
        : "memory");
}

// barrier of the 128 epilogue threads (named barrier 1) that also ANDs a
// predicate across them, so every epilogue warp takes the same branch
__device__ __forceinline__ bool epi_all(bool ok) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\t"
        "bar.red.and.pred p, 1, 128, q;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)ok)
        : "memory");
    return r != 0;
}

template <int MODE, bool PAIR>
__host__ __device__ constexpr uint32_t instr_desc() {
    return (1u << 4)                                   // D in fp32
           | (Cfg<MODE>::FMT << 7) | (Cfg<MODE>::FMT << 10)   // A, B format
           | (uint32_t(Cfg<MODE>::BN >> 3) << 17)        // N
           | (uint32_t((PAIR ? 2 * BM : BM) >> 4) << 24);   // M: 256 across a CTA pair
}

// -- shared memory ---------------------------------------------------------

// PAIR: a CTA holds half of each B tile, so a stage is smaller and the ring
// deeper in the same shared memory
template <int MODE, bool PAIR>
struct Layout {
    static constexpr int BN = Cfg<MODE>::BN;
    static constexpr int B_ROWS = PAIR ? BN / 2 : BN;
    static constexpr int A_BYTES = BM * ROW_BYTES;
    static constexpr int B_BYTES = B_ROWS * ROW_BYTES;
    static constexpr int STAGE = Cfg<MODE>::NOPS * (A_BYTES + B_BYTES);
    static constexpr int STAGES = PAIR ? (MODE == MODE_F16 ? 6 : 4) : Cfg<MODE>::STAGES;
    static constexpr int RING = STAGES * STAGE;
    static constexpr int NORMS = RING;                          // float [2][BN]
    static constexpr int BUFD = NORMS + 2 * BN * 4;             // float [BUF][BM]
    static constexpr int BUFI = BUFD + BUF * BM * 4;            // int   [BUF][BM]
    static constexpr int BARS = BUFI + BUF * BM * 4;            // full, empty, accf, acce
    static constexpr int TMEMP = BARS + (2 * STAGES + 4) * 8;
    static constexpr int TOTAL = TMEMP + 16;
    static constexpr int ALLOC = TOTAL;   // the 1024-aligned extern declaration aligns the ring
};

struct Params {
    int64_t n;          // corpus rows (columns of the sweep)
    int64_t row0, rows; // the rows swept
    int dim;
    int C;
    int metric;
    const float* norms; // l2: |x|^2 of every row
    float* best_d;      // [rows][2][C] ping-pong sorted lists (scratch)
    int32_t* best_i;
    int32_t* idx;       // [rows][C] out
    float* dst;
    int32_t* status;
};

// Warp-cooperative merge of row r's buffer (bcnt <= BUF entries, shared
// memory) into its sorted best list (global, nb entries, C <= 32 * PER),
// written to the other half of the row's ping-pong pair.  The row's own index
// `self` takes the distance SELF here (the filter lets it through on its true
// distance, which is at most SELF, so nothing the reference keeps is lost).
//
// Lane l holds list entries l*PER .. l*PER+PER-1 (loaded first, so the loads
// overlap the buffer sort); the buffer is sorted across the lanes.  Keys are
// (distance, id) with distinct ids, so no two entries tie, and every entry's
// merged position is its own index plus the number of entries of the other
// sequence before it, found by binary lifting over the lanes:
//   list entry   -> over the sorted buffer lanes;
//   buffer entry -> over the lanes' last list entries, then inside one lane.
// Returns the merged length; when the list is full, the new C-th distance
// comes back in thd on every lane.
constexpr int PER_MAX = 8;   // C <= 256
template <int PER>
__device__ int coop_flush(const Params& P, const float* bufd, const int* bufi, int r, int self, int64_t lrow,
                          int bcnt, int nb, int pp, int lane, float& thd) {
    const int C = P.C;
    const float INF = __int_as_float(0x7f800000);
    const float* ad = P.best_d + (lrow * 2 + pp) * C;
    const int* ai = P.best_i + (lrow * 2 + pp) * C;
    float* od = P.best_d + (lrow * 2 + (pp ^ 1)) * C;
    int* oi = P.best_i + (lrow * 2 + (pp ^ 1)) * C;
    float ed[PER];
    int ei[PER];
#pragma unroll
    for (int u = 0; u < PER; ++u) {
        const int idx = lane * PER + u;
        const bool ok = idx < nb;
        ed[u] = ok ? ad[idx] : INF;
        ei[u] = ok ? ai[idx] : 0x7fffffff;
    }
    float bd = INF;
    int bi = 0x7fffffff;
    if (lane < bcnt) {
        bd = bufd[lane * BM + r];
        bi = bufi[lane * BM + r];
        if (bi == self) bd = SELF;
    }
    // sort the buffer entries across the warp (bitonic, ascending)
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
    // list entries: buffer entries before each (lanes >= bcnt hold +inf)
    int epos[PER];
#pragma unroll
    for (int u = 0; u < PER; ++u) epos[u] = 0;
#pragma unroll
    for (int step = 16; step > 0; step >>= 1) {
#pragma unroll
        for (int u = 0; u < PER; ++u) {
            const int m = epos[u] + step - 1;
            const float pd = __shfl_sync(FULL, bd, m);
            const int pi = __shfl_sync(FULL, bi, m);
            if (key_lt(pd, pi, ed[u], ei[u])) epos[u] += step;
        }
    }
    {   // the 32nd buffer lane (only reachable when every lane is a real entry)
        const float pd = __shfl_sync(FULL, bd, 31);
        const int pi = __shfl_sync(FULL, bi, 31);
#pragma unroll
        for (int u = 0; u < PER; ++u)
            if (epos[u] == 31 && key_lt(pd, pi, ed[u], ei[u])) epos[u] = 32;
    }
    // buffer entries: whole lanes of the list before it, then entries of the next lane
    const float lastd = ed[PER - 1];
    const int lasti = ei[PER - 1];
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
    const int src = lb < 32 ? lb : 31;
    int inlane = 0;
#pragma unroll
    for (int u = 0; u < PER; ++u) {
        const float pd = __shfl_sync(FULL, ed[u], src);
        const int pi = __shfl_sync(FULL, ei[u], src);
        if (lb < 32 && key_lt(pd, pi, bd, bi)) ++inlane;
    }
    const int mine = lb * PER + inlane;
    const int newn = min(C, nb + bcnt);
    bool last = false;   // this lane wrote position C - 1
    float lastw = 0.f;
#pragma unroll
    for (int u = 0; u < PER; ++u) {
        const int pos = lane * PER + u + epos[u];
        if (lane * PER + u < nb && pos < C) {
            od[pos] = ed[u];
            oi[pos] = ei[u];
            if (pos == C - 1) { last = true; lastw = ed[u]; }
        }
    }
    if (lane < bcnt) {
        const int pos = lane + mine;
        if (pos < C) {
            od[pos] = bd;
            oi[pos] = bi;
            if (pos == C - 1) { last = true; lastw = bd; }
        }
    }
    if (newn == C) {
        const unsigned w = __ballot_sync(FULL, last);
        thd = __shfl_sync(FULL, lastw, __ffs(w) - 1);
    }
    return newn;
}

// a row's filter state: buffered entries, best-list length, which half of the
// ping-pong pair holds the list, and the list's C-th distance (the threshold)
struct RowState {
    int cnt, nb, pp;
    float th;
};

// flush every row of the warp whose flag is set; kept out of line (state in
// and out by value) so the filter loop that calls it stays small in the
// instruction cache
__device__ __noinline__ RowState flush_rows(const Params& P, const float* bufd, const int* bufi, int lane, int t,
                                            int64_t lrow, int64_t rb0, bool want, RowState st) {
    unsigned m = __ballot_sync(FULL, want);
    while (m) {
        const int src = __ffs(m) - 1;
        m &= m - 1;
        const int r = __shfl_sync(FULL, t, src);
        const long long lr = __shfl_sync(FULL, (long long)lrow, src);
        const int bc = __shfl_sync(FULL, st.cnt, src);
        const int n0 = __shfl_sync(FULL, st.nb, src);
        const int p0 = __shfl_sync(FULL, st.pp, src);
        float td = st.th;
        const int n1 = (P.C <= 128) ? coop_flush<4>(P, bufd, bufi, r, (int)(rb0 + r), lr, bc, n0, p0, lane, td)
                                    : coop_flush<PER_MAX>(P, bufd, bufi, r, (int)(rb0 + r), lr, bc, n0, p0, lane, td);
        __syncwarp();
        if (lane == src) {
            st.nb = n1;
            st.pp ^= 1;
            st.cnt = 0;
            if (n1 == P.C) st.th = td;
        }
    }
    return st;
}

// The filter over 16 consecutive columns j0 .. j0+15 of this thread's row:
// every value below the row's threshold goes to the row's buffer.  Ids already
// merged into the row's best list are all below j0, so the (distance, id) key
// order reduces to the distance alone here.  The common case -- nothing in the
// group beats the threshold on any lane of the warp -- costs a balanced
// max (IP) or min (L2, after the 16 distances) tree and one vote.  Otherwise each kept value is stored at
// cnt + (kept values before it), in column order, so a discarded value's store
// is overwritten by the next kept one (positions stay below cnt + 16 <= BUF: a
// group starts at cnt <= BUF - GROUP).  Returns whether any lane of the warp
// kept a value (warp-uniform).  TAIL: only the first `lim` columns lie inside
// the corpus.
template <int METRIC, bool TAIL>
__device__ __forceinline__ bool filter16(const float* v, const float* nrm, float an, int j0, int lim, float th,
                                         int& cnt, float* myd, int* myi) {
    float d[16];
    float mn;
    if (METRIC == METRIC_IP) {
        // 1 - v is non-increasing in v and rounding is monotone, so the group's
        // smallest distance is 1 - (its largest similarity), NaNs ignored by
        // both forms: one subtraction on the common path instead of sixteen.
        float m[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float a = (TAIL && 2 * i >= lim) ? __int_as_float(0xff800000) : v[2 * i];
            const float b = (TAIL && 2 * i + 1 >= lim) ? __int_as_float(0xff800000) : v[2 * i + 1];
            m[i] = fmaxf(a, b);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) m[i] = fmaxf(m[2 * i], m[2 * i + 1]);
        mn = __fsub_rn(1.f, fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3])));
        if (!__any_sync(FULL, mn < th)) return false;
#pragma unroll
        for (int i = 0; i < 16; ++i)
            d[i] = (TAIL && i >= lim) ? __int_as_float(0x7f800000) : __fsub_rn(1.f, v[i]);
    } else {
        // |b|^2 - 2<a,b> in one rounding (2<a,b> is exact, so the fma rounds
        // the same value the reference's two operations do); adding |a|^2 and
        // the clamp at 0 are monotone, so they move to after the min.
        float e[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
            e[i] = (TAIL && i >= lim) ? __int_as_float(0x7f800000) : __fmaf_rn(-2.f, v[i], nrm[i]);
        float m[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) m[i] = fminf(e[2 * i], e[2 * i + 1]);
#pragma unroll
        for (int i = 0; i < 4; ++i) m[i] = fminf(m[2 * i], m[2 * i + 1]);
        mn = __fadd_rn(fminf(fminf(m[0], m[1]), fminf(m[2], m[3])), an);
        mn = mn < 0.f ? 0.f : mn;
        if (!__any_sync(FULL, mn < th)) return false;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const float x = __fadd_rn(e[i], an);
            d[i] = (TAIL && i >= lim) ? __int_as_float(0x7f800000) : (x < 0.f ? 0.f : x);
        }
    }
    unsigned mk = 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) mk |= (d[i] < th ? 1u : 0u) << i;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const int pos = cnt + __popc(mk & ((1u << i) - 1u));
        myd[pos * BM] = d[i];
        myi[pos * BM] = j0 + i;
    }
    cnt += __popc(mk);
    return true;
}

// One CTA (PAIR = false), or one CTA of a pair (PAIR = true: launched as
// clusters of two, the leader issuing M = 256 MMAs over both CTAs' tiles).
template <int MODE, bool PAIR>
__global__ void __launch_bounds__(NTHREADS, 1) sweep_kernel(const __grid_constant__ CUtensorMap tmA,
                                                            const __grid_constant__ CUtensorMap tmA2,
                                                            const __grid_constant__ CUtensorMap tmB,
                                                            const __grid_constant__ CUtensorMap tmB2,
                                                            const __grid_constant__ Params P) {
    using Ly = Layout<MODE, PAIR>;
    constexpr int BN = Cfg<MODE>::BN;
    constexpr int STAGES = Ly::STAGES;
    constexpr int KSUB = Cfg<MODE>::KSUB;
    constexpr int KELEM = (MODE == MODE_F16) ? 64 : 32;          // K elements per stage
    constexpr uint32_t IDESC = instr_desc<MODE, PAIR>();
    extern __shared__ __align__(1024) char smem_raw[];
    char* sm = smem_raw;
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + Ly::BARS);
    uint64_t* empty = full + STAGES;
    uint64_t* accf = empty + STAGES;
    uint64_t* acce = accf + 2;
    uint32_t* tmem_ptr = reinterpret_cast<uint32_t*>(sm + Ly::TMEMP);
    float* norms_s = reinterpret_cast<float*>(sm + Ly::NORMS);
    float* bufd = reinterpret_cast<float*>(sm + Ly::BUFD);
    int* bufi = reinterpret_cast<int*>(sm + Ly::BUFI);
    __shared__ int s_abort_store;
    volatile int* s_abort = &s_abort_store;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = PAIR ? cluster_rank() : 0u;
    const bool leader = rank == 0;
    const int64_t rb0 = P.row0 + (int64_t)blockIdx.x * BM;   // first global row of this block
    const int ntiles = (int)((P.n + BN - 1) / BN);
    const int ksteps = P.dim / KELEM;

    if (threadIdx.x == 0) {
        // the 128B swizzle needs every stage on a 1024-byte boundary; the extern
        // declaration asks for it, and a block that did not get it does no work
        // (it still takes part in every barrier, so a pair cannot hang on it)
        *s_abort = (smem_u32(sm) & 1023u) ? 2 : 0;
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(&accf[0], 1);
        mbar_init(&accf[1], 1);
        mbar_init(&acce[0], PAIR ? 256 : 128);   // a pair's leader hears both CTAs' epilogues
        mbar_init(&acce[1], PAIR ? 256 : 128);
        fence_mbar_init();
    }
    if (warp == 1) {
        if constexpr (PAIR) {
            tmem_alloc2(tmem_ptr, 2 * BN);
            tmem_relinquish2();
        } else {
            tmem_alloc(tmem_ptr, 2 * BN);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    if constexpr (PAIR) cluster_sync();   // both CTAs' barriers exist before either signals the other
    else __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_ptr;

    if (warp == 0) {
        // ---------------- TMA producer (in both CTAs of a pair)
        if (lane == 0) {
            int it = 0;
            for (int ct = 0; ct < ntiles && !*s_abort; ++ct) {
                for (int ks = 0; ks < ksteps; ++ks, ++it) {
                    const int st = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1;
                    if (!mbar_wait_sleep(&empty[st], ph ^ 1)) { *s_abort = 1; break; }
                    char* base = sm + st * Ly::STAGE;
                    const int k0 = ks * KELEM;
                    if constexpr (PAIR) {
                        // the leader's barrier counts both CTAs' bytes
                        if (leader) mbar_expect_tx(&full[st], 2 * Ly::STAGE);
                        const uint32_t fb = cluster_addr(&full[st], 0);
                        const int bcol = ct * BN + (int)rank * Ly::B_ROWS;
                        tma_load_2d_pair(base, &tmA, k0, (int)rb0, fb);
                        tma_load_2d_pair(base + Ly::A_BYTES, &tmB, k0, bcol, fb);
                        if constexpr (MODE == MODE_TF32X3) {
                            tma_load_2d_pair(base + Ly::A_BYTES + Ly::B_BYTES, &tmA2, k0, (int)rb0, fb);
                            tma_load_2d_pair(base + 2 * Ly::A_BYTES + Ly::B_BYTES, &tmB2, k0, bcol, fb);
                        }
                    } else {
                        mbar_expect_tx(&full[st], Ly::STAGE);
                        tma_load_2d(base, &tmA, k0, (int)rb0, &full[st]);
                        tma_load_2d(base + Ly::A_BYTES, &tmB, k0, ct * BN, &full[st]);
                        if constexpr (MODE == MODE_TF32X3) {
                            tma_load_2d(base + Ly::A_BYTES + Ly::B_BYTES, &tmA2, k0, (int)rb0, &full[st]);
                            tma_load_2d(base + 2 * Ly::A_BYTES + Ly::B_BYTES, &tmB2, k0, ct * BN, &full[st]);
                        }
                    }
                }
            }
        }
        __syncwarp();   // reconverge before the block-wide barrier below
    } else if (warp == 1) {
        // ---------------- MMA issuer (the leader of a pair only)
        if (lane == 0 && leader) {
            int it = 0;
            for (int ct = 0; ct < ntiles && !*s_abort; ++ct) {
                const int acc = ct & 1;
                if (!mbar_wait_sleep(&acce[acc], ((ct >> 1) & 1) ^ 1)) { *s_abort = 1; break; }
                tc_fence_after();
                const uint32_t dtm = tmem + acc * BN;
                for (int ks = 0; ks < ksteps; ++ks, ++it) {
                    const int st = it % STAGES;
                    if (!mbar_wait_sleep(&full[st], (it / STAGES) & 1)) { *s_abort = 1; break; }
                    tc_fence_after();
                    const char* base = sm + st * Ly::STAGE;
                    const char* a_hi = base;
                    const char* b_hi = base + Ly::A_BYTES;
#pragma unroll
                    for (int k = 0; k < KSUB; ++k) {
                        const uint32_t first = (ks == 0 && k == 0) ? 0u : 1u;
                        const uint64_t ah = smem_desc(a_hi + 32 * k), bh = smem_desc(b_hi + 32 * k);
                        if constexpr (PAIR) umma_pair<MODE>(dtm, ah, bh, IDESC, first);
                        else umma<MODE>(dtm, ah, bh, IDESC, first);
                        if constexpr (MODE == MODE_TF32X3) {
                            const char* a_lo = base + Ly::A_BYTES + Ly::B_BYTES;
                            const char* b_lo = base + 2 * Ly::A_BYTES + Ly::B_BYTES;
                            const uint64_t al = smem_desc(a_lo + 32 * k), bl = smem_desc(b_lo + 32 * k);
                            if constexpr (PAIR) {
                                umma_pair<MODE>(dtm, ah, bl, IDESC, 1u);
                                umma_pair<MODE>(dtm, al, bh, IDESC, 1u);
                            } else {
                                umma<MODE>(dtm, ah, bl, IDESC, 1u);
                                umma<MODE>(dtm, al, bh, IDESC, 1u);
                            }
                        }
                    }
                    if constexpr (PAIR) umma_commit_pair(&empty[st]);
                    else umma_commit(&empty[st]);
                }
                if constexpr (PAIR) umma_commit_pair(&accf[acc]);
                else umma_commit(&accf[acc]);
            }
        }
        __syncwarp();
    } else {
        // ---------------- epilogue: thread t owns row t of the block
        const int q = warp & 3;                      // TMEM lane quarter this warp may read
        const int t = q * 32 + lane;
        const int et = threadIdx.x - 64;             // 0..127 among the epilogue threads
        const int64_t grow = rb0 + t;
        const int64_t lrow = (int64_t)blockIdx.x * BM + t;   // row within the swept range
        const bool live = (grow < P.row0 + P.rows) && (grow < P.n);
        const float an = (P.metric == METRIC_L2 && live) ? P.norms[grow] : 0.f;
        RowState rs{0, 0, 0, live ? __int_as_float(0x7f800000) : __int_as_float(0xff800000)};
        float* myd = bufd + t;
        int* myi = bufi + t;
        for (int ct = 0; ct < ntiles; ++ct) {
            const int acc = ct & 1;
            if (P.metric == METRIC_L2) {
                for (int c = et; c < BN; c += 128) {
                    const int64_t j = (int64_t)ct * BN + c;
                    norms_s[acc * BN + c] = (j < P.n) ? __ldg(&P.norms[j]) : 0.f;
                }
            }
            const bool ok = !*s_abort && mbar_wait_sleep(&accf[acc], (ct >> 1) & 1);
            if (!epi_all(ok && !*s_abort)) {   // also publishes the norms written above
                *s_abort = 1;
                break;
            }
            tc_fence_after();
            const int cbase = ct * BN;
            const int lim = (int)(P.n - cbase);   // columns of this tile inside the corpus
#pragma unroll 1
            for (int ch = 0; ch < BN / 32; ++ch) {
                float v[32];
                __syncwarp();   // tcgen05.ld is .sync.aligned: the warp must be converged
                tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + acc * BN + ch * 32, v);
                if (ch == BN / 32 - 1) {
                    tc_fence_before();
                    if constexpr (PAIR) mbar_arrive_cluster(cluster_addr(&acce[acc], 0));
                    else mbar_arrive(&acce[acc]);
                }
#pragma unroll
                for (int g = 0; g < 32 / GROUP; ++g) {
                    const int c0 = ch * 32 + g * GROUP;   // column within the tile
                    const float* nrm = norms_s + acc * BN + c0;
                    const int l = lim - c0;
                    bool kept;
                    if (P.metric == METRIC_IP) {
                        kept = (l >= GROUP)
                                   ? filter16<METRIC_IP, false>(v + g * GROUP, nrm, an, cbase + c0, l, rs.th, rs.cnt, myd, myi)
                                   : filter16<METRIC_IP, true>(v + g * GROUP, nrm, an, cbase + c0, l, rs.th, rs.cnt, myd, myi);
                    } else {
                        kept = (l >= GROUP)
                                   ? filter16<METRIC_L2, false>(v + g * GROUP, nrm, an, cbase + c0, l, rs.th, rs.cnt, myd, myi)
                                   : filter16<METRIC_L2, true>(v + g * GROUP, nrm, an, cbase + c0, l, rs.th, rs.cnt, myd, myi);
                    }
                    if (kept) {   // warp-uniform: only a group that stored can fill a buffer
                        const bool full = rs.cnt > BUF - GROUP;
                        if (__any_sync(FULL, full)) rs = flush_rows(P, bufd, bufi, lane, t, lrow, rb0, full, rs);
                    }
                }
            }
        }
        rs = flush_rows(P, bufd, bufi, lane, t, lrow, rb0, live && rs.cnt > 0, rs);
        const int nb = rs.nb, pp = rs.pp;
        // rows of this warp to the output, one row at a time, coalesced
        for (int src = 0; src < 32; ++src) {
            const bool lv = __shfl_sync(FULL, live, src);
            if (!lv) continue;
            const long long lr = __shfl_sync(FULL, (long long)lrow, src);
            const int n1 = __shfl_sync(FULL, nb, src);
            const int p1 = __shfl_sync(FULL, pp, src);
            const float* fd = P.best_d + (lr * 2 + p1) * P.C;
            const int* fi = P.best_i + (lr * 2 + p1) * P.C;
            for (int c = lane; c < P.C; c += 32) {
                const bool okc = c < n1;
                P.idx[lr * P.C + c] = okc ? fi[c] : -1;
                P.dst[lr * P.C + c] = okc ? fd[c] : __int_as_float(0x7f800000);
            }
        }
    }
    tc_fence_before();
    if constexpr (PAIR) cluster_sync();   // nothing of the pair is still in flight to either CTA
    else __syncthreads();
    if (*s_abort && threadIdx.x == 0 && P.status) atomicExch(P.status, *s_abort == 2 ? SWB_ERR_SMEM : ERR_TIMEOUT);
    if (warp == 1) {
        tc_fence_after();
        if constexpr (PAIR) tmem_dealloc2(tmem, 2 * BN);
        else tmem_dealloc(tmem, 2 * BN);
    }
}

// split fp32 rows into tf32 hi (low 13 mantissa bits cleared after rounding to
// nearest) and lo = x - hi (exact in fp32)
__global__ void split_tf32_kernel(const float* __restrict__ X, int64_t count, float* __restrict__ hi,
                                  float* __restrict__ lo) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= count) return;
    const float x = X[i];
    uint32_t b = __float_as_uint(x);
    b = (b + 0x1000u) & 0xFFFFE000u;   // round half up on the 13 dropped bits
    float h = __uint_as_float(b);
    if (!isfinite(h)) h = x;
    hi[i] = h;
    lo[i] = __fsub_rn(x, h);
}

}  // namespace sweep
}  // namespace swb

// ===========================================================================
// host side

using namespace swb;
using namespace swb::sweep;

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void* p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// 2-D map over [n rows, dim] with a box of `box_rows` rows x 128 bytes
int make_map(CUtensorMap* m, const void* base, int64_t n, int dim, int esize, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return abi::fail(SWB_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    const CUtensorMapDataType dt = (esize == 2) ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    cuuint64_t dims[2] = {(cuuint64_t)dim, (cuuint64_t)n};
    cuuint64_t strides[1] = {(cuuint64_t)dim * esize};
    cuuint32_t box[2] = {(cuuint32_t)(ROW_BYTES / esize), (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return abi::fail(SWB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return SWB_OK;
}

// rows of the workspace's per-row lists: a whole number of CTA pairs
int64_t padded_rows(int64_t rows) { return (rows + 2 * BM - 1) / (2 * BM) * (2 * BM); }

template <int MODE, bool PAIR>
int launch_sweep(const void* a_hi, const void* a_lo, int64_t n, int dim, const float* norms, int64_t row0,
                 int64_t rows, int C, int metric, int32_t* idx, float* dst, void* ws, int32_t* status,
                 cudaStream_t st) {
    using Ly = Layout<MODE, PAIR>;
    const int esize = (MODE == MODE_F16) ? 2 : 4;
    CUtensorMap mA, mA2, mB, mB2;
    int rc = make_map(&mA, a_hi, n, dim, esize, BM);
    if (!rc) rc = make_map(&mB, a_hi, n, dim, esize, Ly::B_ROWS);
    if (!rc) rc = make_map(&mA2, a_lo ? a_lo : a_hi, n, dim, esize, BM);
    if (!rc) rc = make_map(&mB2, a_lo ? a_lo : a_hi, n, dim, esize, Ly::B_ROWS);
    if (rc) return rc;
    Params P;
    P.n = n;
    P.row0 = row0;
    P.rows = rows;
    P.dim = dim;
    P.C = C;
    P.metric = metric;
    P.norms = norms;
    P.best_d = reinterpret_cast<float*>(ws);
    P.best_i = reinterpret_cast<int32_t*>(reinterpret_cast<char*>(ws) + (size_t)padded_rows(rows) * 2 * C * 4);
    P.idx = idx;
    P.dst = dst;
    P.status = status;
    const int smem = Ly::ALLOC;
    cudaError_t e = cudaFuncSetAttribute(sweep_kernel<MODE, PAIR>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return abi::cuda_fail(e, "cudaFuncSetAttribute(sweep)");
    unsigned blocks = (unsigned)((rows + BM - 1) / BM);
    if (!PAIR) {
        sweep_kernel<MODE, false><<<blocks, NTHREADS, smem, st>>>(mA, mA2, mB, mB2, P);
        return abi::cuda_check("sweep launch");
    }
    blocks += blocks & 1u;   // whole pairs; a spare CTA has no live rows
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks);
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, sweep_kernel<MODE, true>, mA, mA2, mB, mB2, P);
    if (e != cudaSuccess) return abi::cuda_fail(e, "sweep launch (CTA pairs)");
    return abi::cuda_check("sweep launch");
}

}  // namespace

extern "C" uint64_t swb_sweep_workspace(int64_t n, int64_t rows, int C, int x_dtype) {
    uint64_t b = (uint64_t)padded_rows(rows) * 2 * C * 8;      // ping-pong best lists
    if (x_dtype == SWB_F32) b += 2 * (uint64_t)n * 0;          // hi / lo planes are caller-provided
    (void)n;
    return b;
}

extern "C" int swb_split_tf32(const float* X, int64_t count, float* hi, float* lo, void* stream) {
    if (!X || !hi || !lo) return abi::fail(SWB_ERR_ARG, "null buffer");
    if (count <= 0) return SWB_OK;
    split_tf32_kernel<<<(unsigned)((count + 255) / 256), 256, 0, (cudaStream_t)stream>>>(X, count, hi, lo);
    return abi::cuda_check("split launch");
}

extern "C" int swb_sweep_topc(const void* X, const void* X_lo, int x_dtype, int64_t n, int dim, const float* norms,
                              int64_t row0, int64_t rows, int C, int metric, int32_t* idx, float* dst,
                              void* workspace, uint64_t ws_bytes, int32_t* status, void* stream) {
    if (!X || !idx || !dst || !workspace) return abi::fail(SWB_ERR_ARG, "null buffer");
    if (C < 1 || C > 32 * PER_MAX) return abi::fail(SWB_ERR_ARG, "C must be 1..%d", 32 * PER_MAX);
    if (rows <= 0) return SWB_OK;
    if (row0 < 0 || row0 + rows > n) return abi::fail(SWB_ERR_ARG, "row range outside the corpus");
    if (n >= ((int64_t)1 << 31)) return abi::fail(SWB_ERR_ARG, "at most 2^31 - 1 rows");
    if (metric == SWB_METRIC_L2 && !norms) return abi::fail(SWB_ERR_ARG, "l2 needs row norms");
    if (ws_bytes < swb_sweep_workspace(n, rows, C, x_dtype)) return abi::fail(SWB_ERR_ARG, "workspace too small");
    if (reinterpret_cast<uintptr_t>(X) % 16 || (X_lo && reinterpret_cast<uintptr_t>(X_lo) % 16))
        return abi::fail(SWB_ERR_ARG, "rows must be 16-byte aligned");
    cudaStream_t st = (cudaStream_t)stream;
    // CTA pairs (M = 256 across two SMs) by default; SWB_SWEEP_PAIR=0 runs one CTA per 128 rows
    const bool pair = abi::env_int("SWB_SWEEP_PAIR", 1) != 0;
    if (x_dtype == SWB_F16) {
        if (dim % 64) return abi::fail(SWB_ERR_ARG, "the tensor-core sweep needs dim %% 64 == 0 for fp16 rows");
        return pair ? launch_sweep<MODE_F16, true>(X, nullptr, n, dim, norms, row0, rows, C, metric, idx, dst,
                                                   workspace, status, st)
                    : launch_sweep<MODE_F16, false>(X, nullptr, n, dim, norms, row0, rows, C, metric, idx, dst,
                                                    workspace, status, st);
    }
    if (!X_lo) return abi::fail(SWB_ERR_ARG, "fp32 rows need their tf32 low parts (swb_split_tf32)");
    if (dim % 32) return abi::fail(SWB_ERR_ARG, "the tensor-core sweep needs dim %% 32 == 0 for fp32 rows");
    return pair ? launch_sweep<MODE_TF32X3, true>(X, X_lo, n, dim, norms, row0, rows, C, metric, idx, dst, workspace,
                                                  status, st)
                : launch_sweep<MODE_TF32X3, false>(X, X_lo, n, dim, norms, row0, rows, C, metric, idx, dst, workspace,
                                                   status, st);
}
