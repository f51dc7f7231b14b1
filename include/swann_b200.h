/*
 * swann_b200.h -- C ABI of the B200 (sm_100a) SWANN search and graph build.
 *
 * Plain pointers, sizes, knobs and a cudaStream_t (passed as void*); no torch
 * types.  Every buffer is caller-owned device memory unless a comment says
 * otherwise; the calls are asynchronous on `stream` and never synchronise.
 * Each returns SWB_OK or an SWB_ERR_* code; swb_last_error() describes the
 * last failure on the calling thread.
 *
 * Each entry point names the reference interface it replaces (paths inside
 * geniussyn/SWANN).  The reference binds its kernels through pybind
 * (swann/csrc/local_search.cu:950-955) and torch (swann/build.py); a
 * maintainer binds these through ctypes instead: swann_b200/_lib.py declares
 * every signature below, and swann_b200/refext.py keeps the reference's own
 * pybind argument lists on top of them.
 */
#ifndef SWANN_B200_H
#define SWANN_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define SWB_API __attribute__((visibility("default")))
#else
#define SWB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define SWB_OK 0
#define SWB_ERR_ARG 1       /* a shape, size, pointer or knob is invalid */
#define SWB_ERR_TEAM 2      /* team size is not 4, 8, 16 or 32 */
#define SWB_ERR_SMEM 3      /* the configuration needs more shared memory than a block may have */
#define SWB_ERR_BATCH 4     /* more than 65535 queries in one call */
#define SWB_ERR_CUDA 5      /* a CUDA runtime call or launch failed */
#define SWB_ERR_TIMEOUT 6   /* a bounded device-side wait gave up (read from the status word) */

/* element types of the corpus */
#define SWB_F32 0
#define SWB_F16 1

/* metrics and policies (swann/_engine.py:31-36) */
#define SWB_METRIC_IP 0     /* distance = 1 - <q, x>, rows L2-normalised */
#define SWB_METRIC_L2 1     /* distance = |q - x|^2 */
#define SWB_POLICY_BEST 0
#define SWB_POLICY_ROUND_ROBIN 1

#define SWB_NCTR 10         /* per-branch counters, local_search.cu:35-41 */

/* Limits of the kernels (the reference's MAXL, MAXD and lineage width). */
#define SWB_MAX_QUEUE 512
#define SWB_MAX_DEGREE 128
#define SWB_MAX_SEEDS 128
#define SWB_MAX_BATCH 65535

/* ---------------------------------------------------------------- search -- */

/* Replaces init_states (swann/csrc/local_search.cu:741-776, launched from
 * swann/_engine.py:219-278).  One state per (query, branch): scores the V seeds
 * of each branch, writes its queue, clears its visited table and counters, and
 * clears the per-query distance table and bound when they are given.
 *   X        [n, dim] SWB_F32 or SWB_F16 rows; dim % 4 == 0 (f32) or % 8 == 0 (f16)
 *   Qv       [Q, dim] float32 queries
 *   seeds    [Q, J, V] int32, -1 = empty
 *   ids/dist/expanded/lineage  [Q, J, L] int32 / float32 / uint8 / uint8 (out)
 *   visited  [Q, J, H] int32, H a power of two; H == 1 switches it off
 *   counters [Q, J, SWB_NCTR] int32 (out)
 *   cache    [Q, Hc] uint64 per-query distance table (key id+1 in the high word,
 *            float bits of the distance in the low word); NULL / Hc == 0 = off
 *   bound    [Q] float32 per-query k-th-best bound; NULL = off */
SWB_API int swb_search_init(const void* X, int x_dtype, int64_t n, int dim,
                    const float* Qv, const int32_t* seeds, int Q, int J, int V,
                    int32_t* ids, float* dist, uint8_t* expanded, uint8_t* lineage, int L,
                    int32_t* visited, int H, int32_t* counters,
                    int metric, int team,
                    uint64_t* cache, int Hc, float* bound,
                    void* stream);

/* Replaces advance (swann/csrc/local_search.cu:778-841, swann/_engine.py:281-317).
 * Advances every branch (or the `n_active` flattened q*J+j indices in
 * `active`) by up to `delta` expansions, in place; resumable: advance(a) then
 * advance(b) equals advance(a + b).
 *   G        [n, D] int32 adjacency, -1 = no edge, D <= SWB_MAX_DEGREE
 *   codes    optional sign-code prefilter (local_search.cu:205-243,560-572;
 *            the reference's advance(..., codes, alpha, cmu, margin)), inner
 *            product only: codes [n, code_words] int32, bit i set when
 *            x_i > mu_i, code_words = ceil(dim / 32); code_alpha [n] the
 *            per-node scale |x - mu|_1 / dim; code_mu [dim] the corpus mean.
 *            A neighbour whose estimated distance exceeds the step's expansion
 *            limit by more than code_margin is not read.  NULL = off.
 *   status   optional int32 device word, kept for symmetry with the build
 *            calls: the search kernels have no device-side waits, so they
 *            never write it (a caller may pass NULL) */
SWB_API int swb_search_advance(const void* X, int x_dtype, int64_t n, int dim,
                       const int32_t* G, int D, const float* Qv,
                       int32_t* ids, float* dist, uint8_t* expanded, uint8_t* lineage,
                       int Q, int J, int L,
                       int32_t* visited, int H, int32_t* counters,
                       int metric, int team, int delta, int max_expansions,
                       int policy, int V, float stop_eps, int kstop,
                       uint64_t* cache, int Hc, float* bound, int exclusive,
                       int stall_patience, float crowd_frac,
                       const int32_t* active, int n_active,
                       const int32_t* codes, const float* code_alpha, const float* code_mu,
                       float code_margin, int code_words,
                       int32_t* status, void* stream);

/* Replaces merge_branches (swann/csrc/local_search.cu:925-947, and the tensor
 * definition swann/_engine.py:377-402): per query, the k nearest of the J*kk
 * branch results by (distance, id), each id once; padding is (-1, +inf). */
SWB_API int swb_merge_branches(const int32_t* bids, const float* bdist, int Q, int J, int kk, int k,
                       int32_t* out_ids, float* out_dist, void* stream);

/* Replaces the torch.topk calls of select_nearest (swann/_select.py:93-130):
 * folds one slice of query x catalogue scores (scores[r * ld + c], catalogue
 * entries col0 .. col0+P-1) into each query's running E nearest, by the
 * reference's metric expressions (1 - s; (|v|^2 - 2s) + |q|^2 with vnorm [P]
 * and qnorm [rows]).  best_d / best_i [rows][E] hold the list sorted by
 * (distance, index), padding (+inf, -1); resume = 0 starts them fresh.
 * E <= 128. */
SWB_API int swb_select_topk(const float* scores, int64_t rows, int P, int64_t ld, const float* vnorm,
                    const float* qnorm, int metric, int E, int col0, float* best_d, int64_t* best_i,
                    int resume, void* stream);

/* Clears what a fused search shares per query: the distance table, the bound
 * and the per-query completion counter.  Launch before swb_search_fused on the
 * same stream.  Part of replacing init_kernel's clears (local_search.cu:302-313). */
SWB_API int swb_search_prepare(int Q, uint64_t* cache, int Hc, float* bound, int32_t* qdone,
                       void* stream);

/* Replaces the whole of swann/_engine.py:428-447 (search: init_states, advance
 * for the full budget, branch_topk, merge_branches) as one kernel, the path
 * swann/index.py:86-110 (Index.search) runs.  The last branch of each query to
 * finish merges that query's branches.
 *   branch_ids/branch_dist [Q, J, kk] int32/float32 scratch, kk = min(k, L)
 *   qdone    [Q] int32, cleared by swb_search_prepare
 *   out_ids/out_dist [Q, k] (out)
 *   ids/dist/expanded/lineage/counters: optional outputs of the final branch
 *   states (NULL to skip), shapes as in swb_search_init
 *   status: as in swb_search_advance (never written; NULL is fine)
 * Small batches run other forms of the kernel, with the same results: with
 * Q * J at most 16 an SM, one branch a CTA whose other three warps score its
 * rows with it; else with at most 16 CTAs an SM (a CTA holds 4 branches of
 * one query), eight rows a team in flight instead of two.  The environment
 * variables SWB_HELP_CTAS and SWB_WIDE_CTAS override those limits (0: never). */
SWB_API int swb_search_fused(const void* X, int x_dtype, int64_t n, int dim,
                     const int32_t* G, int D, const float* Qv, const int32_t* seeds,
                     int Q, int J, int V, int k, int L, int B,
                     int metric, int team, int policy, float stop_eps, int kstop,
                     int32_t* visited, int H,
                     uint64_t* cache, int Hc, float* bound, int exclusive,
                     int stall_patience, float crowd_frac,
                     int32_t* branch_ids, float* branch_dist, int32_t* qdone,
                     int32_t* out_ids, float* out_dist,
                     int32_t* ids, float* dist, uint8_t* expanded, uint8_t* lineage,
                     int32_t* counters, int32_t* status, void* stream);

/* No counterpart in the reference: the fused search above, for callers that
 * cannot hand this library device memory for its scratch -- a host runtime
 * whose memory manager owns the whole device heap and forbids raw cudaMalloc,
 * or a latency-critical serving thread that must never call an allocator (an
 * allocation can synchronise the device).  The caller passes only inputs and
 * outputs; the per-query distance tables, bounds, completion counters,
 * per-branch result lists and visited tables come from one fixed array of
 * SWB_STATIC_SCRATCH_BYTES compiled into the library (every GPU that loads the
 * library holds it until exit).  Nothing is allocated.
 *   - A configuration needing more scratch than the array holds
 *     (swb_search_static_bytes) is rejected with SWB_ERR_ARG; split the batch.
 *   - The first call on a device looks up the array's device address on that
 *     device (cudaGetSymbolAddress); make that first call before any stream
 *     capture.
 *   - Every call shares the one array and clears what must start empty on its
 *     own stream first.  Calls whose work overlaps on the GPU (other streams,
 *     other threads) race on the array and corrupt each other's results:
 *     serialise them.
 *   - One seed per branch (seeds [Q, J]), POLICY_BEST, no stall or crowd
 *     rules; shared_cache / shared_bound / exclusive / elide_visited as in
 *     swb_search_fused; Hc is the per-query table size (a power of two).
 *   - status is accepted for symmetry and never written (the search has no
 *     device-side waits); NULL is fine.
 *   - Q <= 65535, D <= SWB_MAX_DEGREE, L <= SWB_MAX_QUEUE and a visited table
 *     of at most 2^30 slots (B * D bounded) are checked before any sizing. */
#define SWB_STATIC_SCRATCH_BYTES (32u << 20)
SWB_API int swb_search_fused_static(const void* X, int x_dtype, int64_t n, int dim,
                            const int32_t* G, int D, const float* Qv, const int32_t* seeds,
                            int Q, int J, int k, int L, int B, int metric, int team,
                            float stop_eps, int shared_cache, int shared_bound, int exclusive,
                            int elide_visited, int Hc, int32_t* out_ids, float* out_dist,
                            int32_t* status, void* stream);
/* Scratch bytes swb_search_fused_static needs for a configuration. */
SWB_API uint64_t swb_search_static_bytes(int Q, int J, int k, int L, int B, int D, int Hc,
                                 int shared_cache, int exclusive, int elide_visited);

/* ----------------------------------------------------------------- build -- */

/* Replaces the selection half of knn_candidates (swann/build.py:36-42:
 * pairwise, the 3.4e38 diagonal, torch.topk): folds a block of dot products
 * dots[r * ld + c] = <x_{row0+r}, x_{col0+c}> (rows x ncols) into each row's
 * running C nearest, ascending by (distance, id).  resume = 0 starts the lists;
 * resume = 1 continues the lists idx/dst already hold (column blocking).
 *   ip: 1 - <a, b>      l2: max((|b|^2 - 2<a, b>) + |a|^2, 0)
 *   norms    [n] float32 squared row norms (l2 only; NULL for ip)
 *   idx/dst  [rows, C] int32 / float32, C <= 256 */
SWB_API int swb_topc_block(const float* dots, int64_t rows, int64_t ld, int64_t ncols, int64_t row0,
                   int64_t col0, const float* norms, int metric, int C, int32_t* idx, float* dst,
                   int resume, void* stream);

/* Replaces knn_candidates (swann/build.py:30-43) whole: for rows
 * [row0, row0 + rows) of X, the C nearest rows of X by the metric, ascending by
 * (distance, id), the row itself carrying 3.4e38 -- X x X^T on tcgen05 (TMEM
 * accumulators, TMA-fed) with the per-row top-C selection in the epilogue.
 *   SWB_F16 rows: X fp16 [n, dim], dim % 64 == 0, X_lo = NULL (exact products)
 *   SWB_F32 rows: X = tf32 high parts, X_lo = low parts (swb_split_tf32),
 *                 dim % 32 == 0 (3xTF32: hi*hi + hi*lo + lo*hi)
 *   norms [n] float32 squared row norms (l2 only)
 *   idx/dst [rows, C] int32 / float32 (out), C <= 256
 *   workspace: at least swb_sweep_workspace() bytes
 *   status: optional int32 device word, SWB_ERR_TIMEOUT if a wait ran out */
SWB_API int swb_sweep_topc(const void* X, const void* X_lo, int x_dtype, int64_t n, int dim,
                   const float* norms, int64_t row0, int64_t rows, int C, int metric,
                   int32_t* idx, float* dst, void* workspace, uint64_t ws_bytes,
                   int32_t* status, void* stream);
SWB_API uint64_t swb_sweep_workspace(int64_t n, int64_t rows, int C, int x_dtype);

/* fp32 -> (hi, lo): hi = x rounded to tf32 precision, lo = x - hi (exact). */
SWB_API int swb_split_tf32(const float* X, int64_t count, float* hi, float* lo, void* stream);

/* Squared norms of the rows of X in sequential-fmaf order (the build's l2 norms). */
SWB_API int swb_row_norms(const void* X, int x_dtype, int64_t n, int dim, float* norms, void* stream);

/* Replaces robust_prune (swann/build.py:48-91): keeps candidate i of node u
 * unless an already-kept j has alpha * pair(j, i) <= cdist[u, i]; at most `deg`
 * kept, written in candidate order and padded with -1.
 *   X [n, dim] f32 rows (fp16 corpora are built in fp32, build.py:165-166)
 *   cand/cdist [rows, C] int32 / float32, C <= 128;  out [rows, deg] int32
 *   deg_per_node  optional int32 [rows]: node u keeps at most min(deg_per_node[u],
 *                 deg) (robust_prune's deg_per_node; deg is then the widest)
 *   protect       optional uint8 [rows, C]: a set entry exempts that candidate
 *                 from the detour test (robust_prune's protect, mutual pairs) */
SWB_API int swb_prune(const float* X, int64_t n, int dim, const int32_t* cand, const float* cdist,
              int64_t rows, int C, int deg, float alpha, int metric,
              const int32_t* deg_per_node, const uint8_t* protect, int32_t* out, void* stream);

/* Replaces robust_prune (swann/build.py:48-91) as swb_prune does, with the
 * pair distances on the tensor cores and the same output, bit for bit: each
 * node's 128 x 128 candidate Gram matrix is formed with tcgen05 (kind::f16
 * for fp16-valued rows, 3xTF32 otherwise), every detour test that clears its
 * threshold by more than a rigorous bound on the tensor-core value's gap to
 * the dimension-ordered fmaf chain is decided from it, and the pairs within
 * the bound are recomputed with that fmaf chain.
 *   A        tensor-core operand rows [n, adim]: a_dtype SWB_F16 -> the rows in
 *            fp16 (they must be fp16-valued), SWB_F32 -> their tf32 high parts
 *            with A_lo the low parts (swb_split_tf32); zero-padded to adim, a
 *            multiple of 64 (f16) or 32 (f32); 16-byte aligned
 *   X        the fp32 rows [n, dim] (the exact recompute)
 *   norms    [n] squared norms of X by swb_row_norms (both metrics)
 *   recomputed optional device uint64: += the pairs recomputed exactly
 *   status   optional int32 device word: SWB_ERR_TIMEOUT if a wait ran out
 *   other arguments as swb_prune */
SWB_API int swb_prune_tc(const float* X, const void* A, const void* A_lo, int a_dtype, int adim,
                 const float* norms, int64_t n, int dim, const int32_t* cand, const float* cdist,
                 int64_t rows, int C, int deg, float alpha, int metric, const int32_t* deg_per_node,
                 const uint8_t* protect, int32_t* out, unsigned long long* recomputed, int32_t* status,
                 void* stream);

/* Replaces add_reverse (swann/build.py:96-150): offers every edge of G back to
 * its target (first `max_in` offers per target in source order), merges with
 * the target's own row, drops self and duplicates, scores, keeps the nearest
 * 128 and re-prunes to `deg` -- for rows [row0, row0 + rows) (a rank's row
 * block; the whole graph is row0 = 0, rows = n).
 *   G [n, deg] int32;  out [rows, deg] int32 (must not alias G)
 *   deg_per_node  optional int32 [n] per-node caps of the re-prune (add_reverse's
 *                 deg_per_node), indexed by node id
 *   workspace: at least swb_reverse_workspace(n, rows, deg, max_in) bytes */
SWB_API int swb_reverse(const float* X, int64_t n, int dim, const int32_t* G, int deg, float alpha,
                int max_in, int metric, const int32_t* deg_per_node, int64_t row0, int64_t rows,
                int32_t* out, void* workspace, uint64_t ws_bytes, void* stream);
SWB_API uint64_t swb_reverse_workspace(int64_t n, int64_t rows, int deg, int max_in);
/* swb_reverse with its re-prune on the tensor cores (swb_prune_tc's operands
 * and guarantee: the same output as swb_reverse, bit for bit). */
SWB_API int swb_reverse_tc(const float* X, const void* A, const void* A_lo, int a_dtype, int adim,
                   const float* norms, int64_t n, int dim, const int32_t* G, int deg, float alpha,
                   int max_in, int metric, const int32_t* deg_per_node, int64_t row0, int64_t rows,
                   int32_t* out, void* workspace, uint64_t ws_bytes, unsigned long long* recomputed,
                   int32_t* status, void* stream);

/* ------------------------------------------------- offline builder extras -- */

/* Replaces candidates_from_graph (offline/build_graph.py:73-99): node u's
 * first C entries of an existing graph Gc [n, gc_width], with exact distances
 * (dimension-ordered fmaf), -1 entries and u itself at 3.4e38, ordered by
 * (distance, position).  X [n, dim] f32; idx [n, C] int32, dst [n, C] f32. */
SWB_API int swb_graph_candidates(const float* X, int64_t n, int dim, const int32_t* Gc, int gc_width, int C,
                         int metric, int32_t* idx, float* dst, void* stream);

/* Replaces mutual_rank (offline/build_graph.py:102-130): out[u, i] = 1 when
 * i < M, cand[u, i] >= 0 and u is among the first M entries of
 * cand[cand[u, i]]; cand [n, C] int32, out [n, C] uint8. */
SWB_API int swb_mutual_rank(const int32_t* cand, int64_t n, int C, int M, uint8_t* out, void* stream);

/* Replaces fill_degree (offline/build_graph.py:133-202), in place on G [n, W]:
 * rule 0 "near", 1 "far", 2 "bridge"; rows `chunk` at a time, each chunk
 * seeing the earlier chunks' fills; tmp [chunk, W] int32 scratch. */
SWB_API int swb_fill_degree(int32_t* G, int64_t n, int W, const int32_t* cand, int C, int rule, int chunk,
                    int32_t* tmp, void* stream);

/* Replaces enforce_min_in (offline/build_graph.py:309-386), in place on G
 * [n, W]: up to `rounds` rounds of offering nodes below `min_in` in-edges to
 * their candidates (cand [n, C]).  Synchronous (it stops when the floor is
 * met).  stats: optional host int32 [rounds][4] (nodes below, edges to place,
 * placed, already linked); rounds_run: optional host int. */
SWB_API uint64_t swb_min_in_workspace(int64_t n);
SWB_API int swb_enforce_min_in(int32_t* G, int64_t n, int W, const int32_t* cand, int C, int min_in, int rounds,
                       void* workspace, uint64_t ws_bytes, int32_t* stats, int* rounds_run, void* stream);

/* --------------------------------------------------------------- utility -- */

SWB_API const char* swb_last_error(void);
SWB_API int swb_version(void);

#ifdef __cplusplus
}
#endif
#endif /* SWANN_B200_H */
