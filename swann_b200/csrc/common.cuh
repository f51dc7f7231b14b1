// common.cuh -- device helpers shared by the search and build kernels (sm_100a):
// mbarrier primitives (every wait bounded), the (distance, id) order, and the
// reference's distance arithmetic over 16-byte row chunks.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <float.h>
#include <stdint.h>

namespace swb {

constexpr int NCTR = 10;        // counters per branch (local_search.cu:35-41)
constexpr int CPROBE = 32;      // probes into the per-query table before giving up
constexpr int MAXL = 512;       // queue width limit
constexpr int MAXD = 128;       // graph out-degree limit
constexpr int MAXV = 128;       // seeds per branch limit
constexpr int METRIC_IP = 0;
constexpr int METRIC_L2 = 1;
constexpr int POLICY_BEST = 0;
constexpr int POLICY_RR = 1;
constexpr uint32_t FLT_MAX_BITS = 0x7f7fffffu;
constexpr unsigned FULL = 0xffffffffu;
constexpr int ERR_TIMEOUT = 6;  // SWB_ERR_TIMEOUT

// (distance, id) total order (local_search.cu:87-89)
__device__ __forceinline__ bool key_lt(float da, int ia, float db, int ib) {
    return (da < db) || (da == db && ia < ib);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait with a suspend-time hint: a thread whose phase is not complete is
// suspended (it issues nothing) until the phase completes or about `ns`
// nanoseconds pass, instead of returning at once to spin
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
        : "memory");
    return ok != 0;
}

// Bounded wait for phase `parity` of `bar` to complete: gives up after about
// two seconds of SM clock and returns false (the caller records a status).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (;;) {
        for (int i = 0; i < 64; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (clock64() - t0 > (1ll << 32)) return false;
    }
}

// The same bound, with the waiting thread suspended between checks (for
// warps that share a scheduler with warps doing work).
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (;;) {
        if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
        if (clock64() - t0 > (1ll << 32)) return false;
    }
}

__device__ __forceinline__ float ld_volatile_f32(const float* p) {
    return *reinterpret_cast<const volatile float*>(p);
}

__device__ __forceinline__ void st_volatile_u64(uint64_t* p, uint64_t v) {
    *reinterpret_cast<volatile unsigned long long*>(p) = static_cast<unsigned long long>(v);
}

__device__ __forceinline__ unsigned lanemask_lt() {
    unsigned m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

// bar.sync on named barrier `id` (1..15; 0 is __syncthreads') for `threads`
// threads, a multiple of 32, called by whole warps; orders shared-memory
// accesses like __syncthreads
__device__ __forceinline__ void named_barrier(int id, int threads) {
    __syncwarp();
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// -- distances ------------------------------------------------------------
//
// The reference fixes the arithmetic (local_search.cu:185-203, _refcpu.py:21-48):
// lane l of a TEAM-wide team owns the 16-byte chunks l, l + TEAM, l + 2*TEAM,
// ... of the row (4 fp32 or 8 fp16 elements each), sums product terms into one
// fp32 accumulator with the multiply and the add rounded separately, and the
// team folds its lanes with a shuffle-down tree.  The products of neighbouring
// elements are formed in pairs (sm_100's mul.rn.f32x2, each half rounded on its
// own); the sum stays a chain of scalar add.rn, which no compiler pass may fuse
// with the multiply.  (Chains of packed adds fed by packed multiplies came out
// of ptxas, in some code shapes, different from separately rounded operations,
// .rn modifiers and -fmad=false notwithstanding, while each packed operation on
// its own rounded exactly: measured, so the adds stay scalar.)

template <typename XT>
struct VecN;
template <>
struct VecN<float> {
    static constexpr int N = 4;
};
template <>
struct VecN<__half> {
    static constexpr int N = 8;
};

// Where the query sits in shared memory.  fp32 rows: in order.  fp16 rows (8
// elements a 16-byte chunk): as two planes, plane h holding elements
// 8c + 4h .. 8c + 4h + 3 of every chunk c at float offset h * dim / 2 + 4c.
// The lanes of a team read consecutive chunks, so every 16-byte read of a
// plane is contiguous across the team; in order, lanes sat 32 bytes apart and
// each read was a 2-way bank conflict.  part() is the 4 floats for elements
// c * VecN + 4h ..; pos() the place of element i.
template <typename XT>
struct QLay;
template <>
struct QLay<float> {
    static __device__ __forceinline__ const float* part(const float* sq, int, int c, int) { return sq + 4 * c; }
    static __device__ __forceinline__ int pos(int, int i) { return i; }
};
template <>
struct QLay<__half> {
    static __device__ __forceinline__ const float* part(const float* sq, int dim, int c, int h) {
        return sq + h * (dim >> 1) + 4 * c;
    }
    static __device__ __forceinline__ int pos(int dim, int i) {
        return ((i >> 2) & 1) * (dim >> 1) + ((i >> 3) << 2) + (i & 3);
    }
};

__device__ __forceinline__ void widen16(const float* p, float* out) {
    const float4 v = *reinterpret_cast<const float4*>(p);
    out[0] = v.x; out[1] = v.y; out[2] = v.z; out[3] = v.w;
}
__device__ __forceinline__ void widen16(const __half* p, float* out) {
    const uint4 raw = *reinterpret_cast<const uint4*>(p);
    const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h[i]);
        out[2 * i] = f.x;
        out[2 * i + 1] = f.y;
    }
}

// a 16-byte chunk held in registers, widened to fp32
template <typename XT>
__device__ __forceinline__ void widen_u4(const uint4 v, float* out);
template <>
__device__ __forceinline__ void widen_u4<float>(const uint4 v, float* out) {
    out[0] = __uint_as_float(v.x); out[1] = __uint_as_float(v.y);
    out[2] = __uint_as_float(v.z); out[3] = __uint_as_float(v.w);
}
template <>
__device__ __forceinline__ void widen_u4<__half>(const uint4 v, float* out) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        union { uint32_t u; __half2 h; } c;
        c.u = w[i];
        const float2 f = __half22float2(c.h);
        out[2 * i] = f.x;
        out[2 * i + 1] = f.y;
    }
}

// packed fp32 pairs, each half rounded to nearest on its own
__device__ __forceinline__ unsigned long long f2_bits(float2 a) {
    return *reinterpret_cast<const unsigned long long*>(&a);
}
__device__ __forceinline__ float2 f2_mul(float2 a, float2 b) {
    float2 d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(*reinterpret_cast<unsigned long long*>(&d)) : "l"(f2_bits(a)), "l"(f2_bits(b)));
    return d;
}
__device__ __forceinline__ float2 f2_sub(float2 a, float2 b) {
    float2 d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(*reinterpret_cast<unsigned long long*>(&d)) : "l"(f2_bits(a)), "l"(f2_bits(b)));
    return d;
}

// all 32 lanes call this; each TEAM-wide segment folds independently
template <int TEAM>
__device__ __forceinline__ float team_reduce(float acc) {
#pragma unroll
    for (int off = TEAM / 2; off > 0; off >>= 1) acc = __fadd_rn(acc, __shfl_down_sync(FULL, acc, off, TEAM));
    return acc;
}

// Chunks of each row in flight per lane (a segment); a row's later segments
// are L2 hits after its whole-row prefetch, so short segments cost little and
// leave registers for occupancy.
#ifndef SWB_LDG_SEG
#define SWB_LDG_SEG 1
#endif
// One 16-byte chunk of a corpus row, read without allocating in L1: a row is
// read once per query, and L1 is worth more to the spilled registers (2% on
// the C3 search, measured; an L2 evict-first policy on top measured slower --
// hub rows are re-read by other queries from L2).
__device__ __forceinline__ uint4 ld_row16(const uint4* p) {
    uint4 v;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
        : "l"(p));
    return v;
}

// Asynchronous 16-byte global -> shared copy (cp.async, cached in L2 only):
// the bytes travel without occupying a register; the issuing thread waits for
// them with cp_async_wait.  Both addresses 16-byte aligned.
__device__ __forceinline__ void cp_async16(uint32_t smem_dst, const void* gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_dst), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// wait until at most N of this thread's committed groups are still in flight
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// A whole row into L2 with one instruction (16-byte aligned, size a multiple
// of 16): issued as a team starts a row, it turns the row's later segments
// into L2 hits instead of dependent DRAM round trips.
__device__ __forceinline__ void prefetch_row_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Elements 4h .. 4h+3 of a 16-byte chunk held in registers, widened to fp32
template <typename XT>
__device__ __forceinline__ void widen_part(const uint4& v, int h, float* out);
template <>
__device__ __forceinline__ void widen_part<float>(const uint4& v, int, float* out) {
    out[0] = __uint_as_float(v.x); out[1] = __uint_as_float(v.y);
    out[2] = __uint_as_float(v.z); out[3] = __uint_as_float(v.w);
}
template <>
__device__ __forceinline__ void widen_part<__half>(const uint4& v, int h, float* out) {
    union { uint32_t u; __half2 h2; } c0, c1;
    c0.u = h ? v.z : v.x;
    c1.u = h ? v.w : v.y;
    const float2 f0 = __half22float2(c0.h2), f1 = __half22float2(c1.h2);
    out[0] = f0.x; out[1] = f0.y; out[2] = f1.x; out[3] = f1.y;
}

// R rows at once on one team, read straight from global memory: lane tl's
// partial sum of each row r < nrows into acc[r], every row its own chain in
// the reference's order (lane tl owns chunks tl, tl + TEAM, ...; within a
// chunk, elements in order).  The loads of all R rows' segments go out
// together (the first, DRAM-bound segment of R rows in one round trip) and the
// R add chains advance in turn, one add each.  Rows r >= nrows are neither
// read nor meaningful.
template <int TEAM, typename XT, int R, int SEG>
__device__ __forceinline__ void team_partial_rows(const float* __restrict__ sq, const XT* const (&rows)[R],
                                                  int nrows, int dim, int metric, int tl, float (&acc)[R]) {
    constexpr int V = VecN<XT>::N;
    const int nch = dim / V;
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.f;
    for (int s0 = tl; s0 < nch; s0 += TEAM * SEG) {
        uint4 raw[R][SEG];
#pragma unroll
        for (int u = 0; u < SEG; ++u) {
            const int c = s0 + u * TEAM;
#pragma unroll
            for (int r = 0; r < R; ++r)
                raw[r][u] = (c < nch && r < nrows) ? ld_row16(reinterpret_cast<const uint4*>(rows[r]) + c)
                                                   : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < SEG; ++u) {
            const int c = s0 + u * TEAM;
            if (c < nch) {
#pragma unroll
                for (int h = 0; h < V / 4; ++h) {
                    const float4 q4 = *reinterpret_cast<const float4*>(QLay<XT>::part(sq, dim, c, h));
                    const float2 q01 = make_float2(q4.x, q4.y), q23 = make_float2(q4.z, q4.w);
                    float p[R][4];
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        float x[4];
                        widen_part<XT>(raw[r][u], h, x);
                        const float2 x01 = make_float2(x[0], x[1]), x23 = make_float2(x[2], x[3]);
                        float2 p01, p23;
                        if (metric == METRIC_IP) {
                            p01 = f2_mul(q01, x01);
                            p23 = f2_mul(q23, x23);
                        } else {
                            const float2 d01 = f2_sub(q01, x01), d23 = f2_sub(q23, x23);
                            p01 = f2_mul(d01, d01);
                            p23 = f2_mul(d23, d23);
                        }
                        p[r][0] = p01.x; p[r][1] = p01.y; p[r][2] = p23.x; p[r][3] = p23.y;
                    }
                    // the rows' chains advance in turn, one add each
#pragma unroll
                    for (int e = 0; e < 4; ++e)
#pragma unroll
                        for (int r = 0; r < R; ++r) acc[r] = __fadd_rn(acc[r], p[r][e]);
                }
            }
        }
    }
}

}  // namespace swb
