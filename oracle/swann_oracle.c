/*
 * swann_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C, CPU-only restatement of the reference algorithms for the two
 * hot paths this repository accelerates.  It is the checker the GPU kernels are
 * compared against and the timed CPU baseline in bench.py; nothing in the
 * product (swann_b200/) links, loads or calls it.
 *
 * What it restates (paths are inside the reference project, geniussyn/SWANN):
 *   search  swann/_refcpu.py:21-48    team_distance (lane-strided order, fp32,
 *                                     multiply and add rounded separately)
 *           swann/_refcpu.py:58-143   init_state / advance (one branch)
 *           swann/csrc/local_search.cu:451-683  the kernel's step, for the
 *                                     shared-table / bound / exclusive modes
 *                                     that _refcpu does not model
 *           swann/csrc/local_search.cu:637-650  merge-path tie rule
 *           swann/csrc/local_search.cu:659-682  crowd and stall rules (the
 *                                     kernel's only; _refcpu has neither)
 *           swann/csrc/local_search.cu:863-919  merge of branch results
 *   build   swann/build.py:14-43      pairwise + knn_candidates
 *           swann/build.py:48-91      robust_prune
 *           swann/build.py:96-150     add_reverse
 *
 * Parity pins: tests/golden/ holds vectors produced by running the reference's
 * own _refcpu.py and build.py (the generating script sits beside them); the
 * CPU test-suite checks this file against every one of them.
 *
 * Arithmetic conventions (chosen so a GPU kernel can reproduce them bit for bit):
 *   - search distances follow _refcpu exactly: per-lane fp32 accumulation of
 *     separately rounded products, then the halving tree;
 *   - build dot products are sequential fmaf over the dimension (the reference
 *     leaves this order to BLAS, which specifies none); the exact candidate
 *     sweep uses double precision so that it is the "truth" ties are measured against.
 *
 * Build: gcc -O2 -fPIC -shared -ffp-contract=off -fno-builtin-powf -fopenmp
 * (oracle/build_oracle.py).
 * -ffp-contract=off matters: a fused multiply-add in team_distance would change
 * the rounding the reference defines.
 */
#include <float.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define OR_METRIC_IP 0
#define OR_METRIC_L2 1
#define OR_POLICY_BEST 0
#define OR_POLICY_RR 1
#define OR_NCTR 10

/* ------------------------------------------------------------------------ */
/* distances                                                                 */
/* ------------------------------------------------------------------------ */

/* How an L2 term is squared.  The kernel multiplies, df * df, rounded once
 * (local_search.cu:197).  _refcpu.py:39 writes F32(q - x) ** 2, which numpy
 * evaluates with libm powf; powf(df, 2) is not always the correctly rounded
 * square and differs from the multiply on about 0.07% of float32 inputs.  Mode
 * 0 (default) is the kernel's definition, the one GPU parity is held to; mode 1
 * reproduces _refcpu bit for bit and is what the golden vectors are pinned in. */
static int g_square_mode = 0;
void or_set_square_mode(int mode) { g_square_mode = mode; }

/* swann/_refcpu.py:21-48 (and the kernel's team_dist, local_search.cu:185-203):
 * lane `l` of a `team`-wide team sums elements l*vec .. l*vec+vec-1, then
 * strides by team*vec; the lanes are folded by a halving tree. */
float or_team_distance(const float* q, const float* x, int d, int metric,
                       int team, int vec) {
    float lanes[32];
    for (int lane = 0; lane < team; ++lane) {
        float acc = 0.0f;
        for (int base = lane * vec; base < d; base += team * vec) {
            for (int i = 0; i < vec; ++i) {
                int t = base + i;
                if (t >= d) break;
                float term;
                if (metric == OR_METRIC_IP) {
                    term = q[t] * x[t];
                } else {
                    float df = q[t] - x[t];
                    term = g_square_mode ? powf(df, 2.0f) : df * df;
                }
                acc = acc + term;
            }
        }
        lanes[lane] = acc;
    }
    for (int off = team / 2; off > 0; off >>= 1)
        for (int lane = 0; lane < off; ++lane) lanes[lane] = lanes[lane] + lanes[lane + off];
    return metric == OR_METRIC_IP ? 1.0f - lanes[0] : lanes[0];
}

/* ------------------------------------------------------------------------ */
/* one branch of the search                                                  */
/* ------------------------------------------------------------------------ */

typedef struct {
    int id;
    float d;
    uint8_t e; /* expanded */
    uint8_t l; /* lineage */
} entry_t;

static int key_lt(float da, int ia, float db, int ib) {
    return (da < db) || (da == db && ia < ib);
}

static int entry_cmp(const void* a, const void* b) {
    const entry_t* x = (const entry_t*)a;
    const entry_t* y = (const entry_t*)b;
    if (key_lt(x->d, x->id, y->d, y->id)) return -1;
    if (key_lt(y->d, y->id, x->d, x->id)) return 1;
    return 0;
}

/* An exact integer set (open addressing, grows never: sized for the most
 * inserts a branch can make).  Stands in for both the per-branch visited
 * table and the per-query distance table; the emulation never loses an
 * insert, where the GPU's bounded probes can. */
typedef struct {
    int* key;   /* id + 1, 0 = empty */
    float* val; /* distance, for the per-query table */
    uint32_t mask;
} iset_t;

static void iset_init(iset_t* s, int64_t want, int with_val) {
    uint32_t h = 16;
    while ((int64_t)h < 2 * want + 2) h <<= 1;
    s->key = (int*)calloc(h, sizeof(int));
    s->val = with_val ? (float*)malloc(sizeof(float) * h) : NULL;
    s->mask = h - 1;
}
static void iset_free(iset_t* s) {
    free(s->key);
    free(s->val);
}
/* returns slot index; *found = 1 if the key was already present */
static uint32_t iset_insert(iset_t* s, int key, int* found) {
    uint32_t pos = (2654435761u * (uint32_t)key) & s->mask;
    for (;;) {
        if (s->key[pos] == key + 1) {
            *found = 1;
            return pos;
        }
        if (s->key[pos] == 0) {
            s->key[pos] = key + 1;
            *found = 0;
            return pos;
        }
        pos = (pos + 1) & s->mask;
    }
}

typedef struct {
    /* problem */
    const float* X;
    int d;
    const int* G;
    int D;
    const float* q;
    int metric, team, vec;
    /* knobs */
    int L, B, V, policy, kstop;
    float stop_eps;
    int stall_patience; /* stop after this many steps without a better k-th best; 0 = off */
    float crowd_frac;   /* retire a lineage after two steps this crowded; 0 = off */
    int use_visited;   /* H > 1 in the kernel */
    /* state */
    entry_t* queue;    /* L slots, empty = (-1, FLT_MAX, 1, 0) */
    entry_t* cand;     /* D */
    entry_t* merged;   /* L */
    iset_t visited;
    int ctr[OR_NCTR];
    uint32_t retired[8];
    /* per-advance-call rule state (local_search.cu:396-415: reset every call) */
    float best_k;
    int stall, crowd_run;
    int done;
} branch_t;

/* shared per-query context for the lockstep emulation */
typedef struct {
    int shared_cache, shared_bound, exclusive;
    iset_t cache;
    float bound;
} qshared_t;

static void branch_alloc(branch_t* b) {
    b->queue = (entry_t*)malloc(sizeof(entry_t) * (size_t)b->L);
    b->merged = (entry_t*)malloc(sizeof(entry_t) * (size_t)b->L);
    b->cand = (entry_t*)malloc(sizeof(entry_t) * (size_t)(b->D > b->V ? b->D : b->V) + sizeof(entry_t));
    if (b->use_visited) iset_init(&b->visited, (int64_t)b->V + (int64_t)b->B * b->D + 1, 0);
    memset(b->ctr, 0, sizeof(b->ctr));
    memset(b->retired, 0, sizeof(b->retired));
    b->best_k = FLT_MAX;
    b->stall = 0;
    b->crowd_run = 0;
    b->done = 0;
}
static void branch_free(branch_t* b) {
    free(b->queue);
    free(b->merged);
    free(b->cand);
    if (b->use_visited) iset_free(&b->visited);
}

/* swann/_refcpu.py:58-79 (init_state); kernel init: local_search.cu:318-350.
 * Seeds are deduplicated first-occurrence-wins (as _refcpu's `seen` set). */
static void branch_init(branch_t* b, const int* seeds) {
    int nc = 0;
    for (int i = 0; i < b->V; ++i) {
        int s = seeds[i];
        if (s < 0) continue;
        if (b->use_visited) {
            int found;
            iset_insert(&b->visited, s, &found);
            if (found) continue;
        } else {
            int dup = 0;
            for (int j = 0; j < nc; ++j) dup |= (b->cand[j].id == s);
            if (dup) continue;
        }
        b->cand[nc].id = s;
        b->cand[nc].d = or_team_distance(b->q, b->X + (size_t)s * b->d, b->d, b->metric, b->team, b->vec);
        b->cand[nc].e = 0;
        b->cand[nc].l = (uint8_t)i;
        ++nc;
        b->ctr[1] += 1;
    }
    qsort(b->cand, (size_t)nc, sizeof(entry_t), entry_cmp);
    for (int i = 0; i < b->L; ++i) {
        if (i < nc) b->queue[i] = b->cand[i];
        else { b->queue[i].id = -1; b->queue[i].d = FLT_MAX; b->queue[i].e = 1; b->queue[i].l = 0; }
    }
}

static int retired_has(const branch_t* b, unsigned li) { return (b->retired[li >> 5] >> (li & 31)) & 1u; }
static void retired_set(branch_t* b, unsigned li) { b->retired[li >> 5] |= (1u << (li & 31)); }

/* One expansion.  swann/_refcpu.py:93-142 for the selection, the stop rule and
 * the expansion; swann/csrc/local_search.cu:451-658 for the table, bound and
 * exclusive semantics and for the merge (which equals _refcpu's two-pointer
 * merge whenever keys are distinct).  Returns 0 when the branch stops. */
static int branch_step(branch_t* b, qshared_t* sh) {
    const int L = b->L;
    if (b->ctr[0] >= b->B) return 0;
    const int early = (b->stop_eps >= 0.0f);
    /* the kernel reads the min(kstop, L)-th entry (local_search.cu:464); _refcpu
     * reads the kstop-th and so agrees whenever kstop <= L */
    const int kr = (b->kstop < L) ? b->kstop : L;
    float radius = (kr > 0 && b->queue[kr - 1].id >= 0) ? b->queue[kr - 1].d : FLT_MAX;
    if (sh && sh->shared_bound && sh->bound < radius) radius = sh->bound;
    const float limit = (radius == FLT_MAX) ? FLT_MAX : radius * (1.0f + b->stop_eps);

    int slot = -1;
    if (b->policy == OR_POLICY_RR && b->V > 1) {
        for (int turn = 0; turn < b->V && slot < 0; ++turn) {
            const int want = (b->ctr[0] + turn) % b->V;
            if (retired_has(b, (unsigned)want)) continue;
            int found = -1;
            for (int i = 0; i < L; ++i)
                if (b->queue[i].id >= 0 && b->queue[i].e == 0 && b->queue[i].l == want) { found = i; break; }
            if (found < 0) { retired_set(b, (unsigned)want); continue; }
            if (early && b->queue[found].d > limit) { retired_set(b, (unsigned)want); continue; }
            slot = found;
        }
        if (slot < 0 && !early) {
            for (int i = 0; i < L; ++i)
                if (b->queue[i].id >= 0 && b->queue[i].e == 0) { slot = i; break; }
        }
    } else {
        for (int i = 0; i < L; ++i)
            if (b->queue[i].id >= 0 && b->queue[i].e == 0) {
                if (retired_has(b, b->queue[i].l)) continue;
                if (!early || b->queue[i].d <= limit) slot = i;
                break;
            }
    }
    if (slot < 0) {
        b->ctr[3] = 1;
        return 0;
    }
    b->queue[slot].e = 1;
    const int p = b->queue[slot].id;
    const uint8_t plin = b->queue[slot].l;
    b->ctr[0] += 1;

    /* expand p, candidates in G's slot order; nbr counts the neighbours and
     * cov those already covered -- in this branch's visited set, or claimed
     * and scored by another branch (local_search.cu:533-585) */
    int nc = 0, nbr = 0, cov = 0;
    for (int s = 0; s < b->D; ++s) {
        const int v = b->G[(size_t)p * b->D + s];
        if (v < 0) continue;
        ++nbr;
        if (b->use_visited) {
            int found;
            iset_insert(&b->visited, v, &found);
            if (found) { ++cov; continue; }
        }
        float dv = FLT_MAX;
        int have = 0, taken = 0;
        if (sh && sh->shared_cache) {
            int found;
            uint32_t pos = iset_insert(&sh->cache, v, &found);
            if (found) {
                dv = sh->cache.val[pos];
                have = 1;
                if (sh->exclusive) taken = 1;
                b->ctr[4] += 1;
            } else {
                dv = or_team_distance(b->q, b->X + (size_t)v * b->d, b->d, b->metric, b->team, b->vec);
                sh->cache.val[pos] = dv;
                b->ctr[5] += 1;
                b->ctr[1] += 1;
                have = 1;
            }
        }
        if (!have) {
            dv = or_team_distance(b->q, b->X + (size_t)v * b->d, b->d, b->metric, b->team, b->vec);
            b->ctr[1] += 1;
        }
        if (taken) { ++cov; continue; }
        b->cand[nc].id = v;
        b->cand[nc].d = dv;
        b->cand[nc].e = 0;
        b->cand[nc].l = plin;
        ++nc;
    }
    /* keep only what can still enter the queue (kernel: local_search.cu:607-625) */
    const float worst = (b->queue[L - 1].id >= 0) ? b->queue[L - 1].d : FLT_MAX;
    int nk = 0;
    for (int i = 0; i < nc; ++i)
        if (worst == FLT_MAX || b->cand[i].d <= worst) b->cand[nk++] = b->cand[i];
    b->ctr[8] += nk;
    b->ctr[9] += 1;
    qsort(b->cand, (size_t)nk, sizeof(entry_t), entry_cmp);

    /* merge-path, one output slot at a time (local_search.cu:637-650) */
    for (int o = 0; o < L; ++o) {
        int lo = (o - nk) > 0 ? (o - nk) : 0, hi = o < L ? o : L;
        while (lo < hi) {
            const int i = (lo + hi) >> 1, j = o - i;
            if (j > 0 && !key_lt(b->cand[j - 1].d, b->cand[j - 1].id, b->queue[i].d, b->queue[i].id)) lo = i + 1;
            else hi = i;
        }
        const int i = lo, j = o - i;
        const int takeA = (j >= nk) || (i < L && key_lt(b->queue[i].d, b->queue[i].id, b->cand[j].d, b->cand[j].id));
        entry_t out;
        if (takeA) out = b->queue[i];
        else { out = b->cand[j]; out.e = 0; }
        if (out.id < 0) { out.d = FLT_MAX; out.e = 1; out.l = 0; }
        b->merged[o] = out;
    }
    memcpy(b->queue, b->merged, sizeof(entry_t) * (size_t)L);
    if (sh && sh->shared_bound && kr > 0 && b->queue[kr - 1].id >= 0 && b->queue[kr - 1].d < sh->bound)
        sh->bound = b->queue[kr - 1].d;
    /* crowding (local_search.cu:659-671): a lineage whose expansions land on
     * covered ground two steps in a row is retired */
    if (b->crowd_frac > 0.0f) {
        const float cv = (nbr > 0) ? ((float)cov / (float)nbr) : 0.0f;
        if (cv >= b->crowd_frac) {
            if (++b->crowd_run >= 2) {
                retired_set(b, (unsigned)plin);
                b->ctr[7] += 1;
                b->crowd_run = 0;
            }
        } else {
            b->crowd_run = 0;
        }
    }
    /* stalling (local_search.cu:672-682): stop once the k-th best has not
     * improved for stall_patience steps */
    if (b->stall_patience > 0) {
        const float bk = (kr > 0 && b->queue[kr - 1].id >= 0) ? b->queue[kr - 1].d : FLT_MAX;
        if (bk < b->best_k) { b->best_k = bk; b->stall = 0; }
        else b->stall += 1;
        if (b->stall >= b->stall_patience) {
            b->ctr[6] = 1;
            return 0;
        }
    }
    return 1;
}

static void branch_export(const branch_t* b, int* ids, float* dist, uint8_t* expd, uint8_t* lin, int* ctr) {
    for (int i = 0; i < b->L; ++i) {
        if (ids) ids[i] = b->queue[i].id;
        if (dist) dist[i] = b->queue[i].d;
        if (expd) expd[i] = b->queue[i].e;
        if (lin) lin[i] = b->queue[i].l;
    }
    if (ctr) memcpy(ctr, b->ctr, sizeof(int) * OR_NCTR);
}

/* swann/_refcpu.py:146-151 (run = init + one advance of `delta` expansions),
 * for one branch seeded with V entries.  Outputs are the kernel's L slots. */
int or_branch_run(const float* X, int d, const int* G, int D, const float* q,
                  const int* seeds, int V, int L, int B, int metric, int team, int vec,
                  int policy, float stop_eps, int kstop, int stall_patience, float crowd_frac, int delta,
                  int* ids, float* dist, uint8_t* expd, uint8_t* lin, int* ctr) {
    branch_t b;
    memset(&b, 0, sizeof(b));
    b.X = X; b.d = d; b.G = G; b.D = D; b.q = q;
    b.metric = metric; b.team = team; b.vec = vec;
    b.L = L; b.B = B; b.V = V; b.policy = policy; b.kstop = kstop; b.stop_eps = stop_eps;
    b.stall_patience = stall_patience; b.crowd_frac = crowd_frac;
    b.use_visited = 1;
    branch_alloc(&b);
    branch_init(&b, seeds);
    for (int s = 0; s < delta; ++s)
        if (!branch_step(&b, NULL)) break;
    branch_export(&b, ids, dist, expd, lin, ctr);
    branch_free(&b);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* merging branch results (local_search.cu:863-919; _engine.py:377-402)       */
/* ------------------------------------------------------------------------ */

typedef struct { float d; int id; } pair_t;
static int pair_cmp(const void* a, const void* b) {
    const pair_t* x = (const pair_t*)a;
    const pair_t* y = (const pair_t*)b;
    if (x->d < y->d) return -1;
    if (x->d > y->d) return 1;
    return (x->id > y->id) - (x->id < y->id);
}

/* n entries (ids, dist) -> k deduplicated nearest by (distance, id);
 * invalid ids (< 0) sort last, output padding is (-1, +inf). */
void or_merge_one(const int* ids, const float* dist, int n, int k, int* out_ids, float* out_dist) {
    pair_t* p = (pair_t*)malloc(sizeof(pair_t) * (size_t)(n > 0 ? n : 1));
    for (int i = 0; i < n; ++i) {
        const int valid = ids[i] >= 0;
        p[i].id = valid ? ids[i] : INT32_MAX;
        p[i].d = valid ? dist[i] : INFINITY;
    }
    qsort(p, (size_t)n, sizeof(pair_t), pair_cmp);
    int w = 0;
    for (int i = 0; i < n && w < k; ++i) {
        if (p[i].id == INT32_MAX) break;
        if (i > 0 && p[i].id == p[i - 1].id) continue;
        out_ids[w] = p[i].id;
        out_dist[w] = p[i].d;
        ++w;
    }
    for (; w < k; ++w) { out_ids[w] = -1; out_dist[w] = INFINITY; }
    free(p);
}

void or_merge_branches(const int* ids, const float* dist, int Q, int J, int kk, int k,
                       int* out_ids, float* out_dist) {
    for (int q = 0; q < Q; ++q)
        or_merge_one(ids + (size_t)q * J * kk, dist + (size_t)q * J * kk, J * kk, k,
                     out_ids + (size_t)q * k, out_dist + (size_t)q * k);
}

/* ------------------------------------------------------------------------ */
/* whole searches                                                            */
/* ------------------------------------------------------------------------ */

/* J branches per query, either independent (shared_* = 0: _refcpu per branch,
 * which is the kernel with the per-query table on or off) or advanced in
 * lockstep -- branch 0, 1, ..., J-1 one expansion each, round after round --
 * sharing the per-query table, the bound and the claims the way the kernel's
 * branches do.  The lockstep order is one legal interleaving of the kernel's
 * concurrent branches; results of those modes agree with the GPU in
 * distribution (recall, work), not bit for bit.
 *
 * seeds: [nq, J, V] int32.  out_ids/out_dist: [nq, k].  out_ctr (optional):
 * [nq, J, OR_NCTR].  Returns 0. */
int or_search(const float* X, int64_t n, int d, const int* G, int D,
              const float* Q, int nq, const int* seeds, int J, int V,
              int k, int L, int B, int metric, int team, int vec, int policy,
              float stop_eps, int kstop, int shared_cache, int shared_bound,
              int exclusive, int elide_visited, int stall_patience, float crowd_frac, int nthreads,
              int* out_ids, float* out_dist, int* out_ctr) {
    (void)n;
    const int kk = k < L ? k : L;
    const int excl = exclusive && shared_cache && J > 1;
    const int cache_on = shared_cache && J > 1;
    const int bound_on = shared_bound && J > 1;
    const int elide = elide_visited && excl && cache_on && J > 1 && V == 1;
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1)
#endif
    for (int qi = 0; qi < nq; ++qi) {
        branch_t* br = (branch_t*)calloc((size_t)J, sizeof(branch_t));
        qshared_t sh;
        memset(&sh, 0, sizeof(sh));
        sh.shared_cache = cache_on;
        sh.shared_bound = bound_on;
        sh.exclusive = excl;
        sh.bound = FLT_MAX;
        if (cache_on) iset_init(&sh.cache, (int64_t)J * ((int64_t)V + (int64_t)B * D) + 1, 1);
        for (int j = 0; j < J; ++j) {
            branch_t* b = &br[j];
            b->X = X; b->d = d; b->G = G; b->D = D; b->q = Q + (size_t)qi * d;
            b->metric = metric; b->team = team; b->vec = vec;
            b->L = L; b->B = B; b->V = V; b->policy = policy; b->kstop = kstop; b->stop_eps = stop_eps;
            b->stall_patience = stall_patience; b->crowd_frac = crowd_frac;
            b->use_visited = !elide;
            branch_alloc(b);
            branch_init(b, seeds + ((size_t)qi * J + j) * V);
        }
        if (cache_on || bound_on) {
            int live = J;
            while (live > 0) {
                live = 0;
                for (int j = 0; j < J; ++j) {
                    if (br[j].done) continue;
                    if (!branch_step(&br[j], &sh)) br[j].done = 1;
                    else ++live;
                }
            }
        } else {
            for (int j = 0; j < J; ++j)
                while (branch_step(&br[j], NULL)) {}
        }
        int* bi = (int*)malloc(sizeof(int) * (size_t)J * kk);
        float* bd = (float*)malloc(sizeof(float) * (size_t)J * kk);
        for (int j = 0; j < J; ++j) {
            for (int t = 0; t < kk; ++t) {
                bi[j * kk + t] = br[j].queue[t].id;
                bd[j * kk + t] = br[j].queue[t].d;
            }
            if (out_ctr) memcpy(out_ctr + ((size_t)qi * J + j) * OR_NCTR, br[j].ctr, sizeof(int) * OR_NCTR);
            branch_free(&br[j]);
        }
        or_merge_one(bi, bd, J * kk, k, out_ids + (size_t)qi * k, out_dist + (size_t)qi * k);
        free(bi);
        free(bd);
        if (cache_on) iset_free(&sh.cache);
        free(br);
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* graph build                                                               */
/* ------------------------------------------------------------------------ */

/* Exact top-C neighbours by the metric, self excluded, ascending by
 * (distance, id).  swann/build.py:14-43.  The reference evaluates
 * 1 - <a,b> (ip) or (|b|^2 - 2<a,b>) + |a|^2 clamped at 0 (l2) from an fp32
 * GEMM and marks the diagonal 3.4e38; here the same expressions are evaluated
 * in double, so these lists are the exact answer that fp32 results are
 * compared with.  Rows [r0, r1) only (a row sample of a large sweep). */
typedef struct { double d; int id; } dpair_t;
static int dpair_cmp(const void* a, const void* b) {
    const dpair_t* x = (const dpair_t*)a;
    const dpair_t* y = (const dpair_t*)b;
    if (x->d < y->d) return -1;
    if (x->d > y->d) return 1;
    return (x->id > y->id) - (x->id < y->id);
}

int or_knn_candidates(const float* X, int64_t n, int d, int C, int metric,
                      int64_t r0, int64_t r1, int nthreads, int* idx, float* dst, double* dst64) {
    double* norms = (double*)malloc(sizeof(double) * (size_t)n);
    for (int64_t j = 0; j < n; ++j) {
        double s = 0.0;
        const float* b = X + (size_t)j * d;
        for (int t = 0; t < d; ++t) s += (double)b[t] * (double)b[t];
        norms[j] = s;
    }
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 4)
#endif
    for (int64_t i = r0; i < r1; ++i) {
        dpair_t* row = (dpair_t*)malloc(sizeof(dpair_t) * (size_t)n);
        const float* a = X + (size_t)i * d;
        for (int64_t j = 0; j < n; ++j) {
            const float* b = X + (size_t)j * d;
            double dot = 0.0;
            for (int t = 0; t < d; ++t) dot += (double)a[t] * (double)b[t];
            double v;
            if (metric == OR_METRIC_IP) v = 1.0 - dot;
            else { v = (norms[j] - 2.0 * dot) + norms[i]; if (v < 0.0) v = 0.0; }
            if (j == i) v = (double)3.4e38f;
            row[j].d = v;
            row[j].id = (int)j;
        }
        qsort(row, (size_t)n, sizeof(dpair_t), dpair_cmp);
        for (int c = 0; c < C; ++c) {
            idx[(size_t)(i - r0) * C + c] = row[c].id;
            dst[(size_t)(i - r0) * C + c] = (float)row[c].d;
            if (dst64) dst64[(size_t)(i - r0) * C + c] = row[c].d;
        }
        free(row);
    }
    free(norms);
    return 0;
}

/* sequential fmaf dot product: the order the GPU prune/reverse kernels use */
static float dot_seq(const float* a, const float* b, int d) {
    float acc = 0.0f;
    for (int t = 0; t < d; ++t) acc = fmaf(a[t], b[t], acc);
    return acc;
}
static float l2_seq(const float* a, const float* b, int d) {
    float acc = 0.0f;
    for (int t = 0; t < d; ++t) {
        const float df = a[t] - b[t];
        acc = fmaf(df, df, acc);
    }
    return acc;
}

/* swann/build.py:48-91, one node.  Candidate i is kept unless an already-kept
 * j has alpha*pair(j,i) <= du[i]; at most `deg` are kept; output is the kept
 * candidates in candidate order, -1 padded to `width`.
 * pair(j,i) = 1 - <v_j,v_i> (ip) or ((|v_i|^2 - 2<v_j,v_i>) + |v_j|^2) clamped
 * at 0 (l2) -- the reference's expression, element [j][i] of its bmm form.
 * alpha is applied in fp32, as torch does for a python scalar. */
/* deg: this node's cap; width: the output row's width; prot (optional): a set
 * entry exempts that candidate from the detour test (robust_prune's protect,
 * offline/build_graph.py:230-232) */
static void prune_one(const float* X, int d, const int* cand, const float* du, int C,
                      int deg, int width, float alpha, int metric, const uint8_t* prot, int* out,
                      float* vn, uint8_t* kept) {
    for (int i = 0; i < C; ++i) {
        vn[i] = 0.0f;
        kept[i] = 0;
        if (cand[i] >= 0) {
            const float* v = X + (size_t)cand[i] * d;
            vn[i] = dot_seq(v, v, d);
        }
    }
    int nk = 0;
    for (int i = 0; i < C && nk < deg; ++i) {
        if (cand[i] < 0) continue;
        const float* vi = X + (size_t)cand[i] * d;
        int viol = 0;
        for (int j = 0; j < i && !viol; ++j) {
            if (!kept[j]) continue;
            const float dot = dot_seq(X + (size_t)cand[j] * d, vi, d);
            float pr;
            if (metric == OR_METRIC_IP) pr = 1.0f - dot;
            else {
                pr = (vn[i] - 2.0f * dot) + vn[j];
                if (pr < 0.0f) pr = 0.0f;
            }
            if (alpha * pr <= du[i]) viol = 1;
        }
        if (prot && prot[i]) viol = 0;
        if (!viol) { kept[i] = 1; ++nk; }
    }
    int w = 0;
    for (int i = 0; i < C && w < width; ++i)
        if (kept[i]) out[w++] = cand[i];
    for (; w < width; ++w) out[w] = -1;
}

/* deg is the output width; dpn (optional) caps node u at min(dpn[u], deg) */
int or_robust_prune(const float* X, int64_t n, int d, const int* cand, const float* cdist, int C,
                    int deg, float alpha, int metric, const int* dpn, const uint8_t* prot, int nthreads,
                    int* out) {
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel
#endif
    {
        float* vn = (float*)malloc(sizeof(float) * (size_t)C);
        uint8_t* kept = (uint8_t*)malloc((size_t)C);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 16)
#endif
        for (int64_t u = 0; u < n; ++u)
            prune_one(X, d, cand + (size_t)u * C, cdist + (size_t)u * C, C,
                      dpn ? (dpn[u] < deg ? dpn[u] : deg) : deg, deg, alpha, metric,
                      prot ? prot + (size_t)u * C : NULL, out + (size_t)u * deg, vn, kept);
        free(vn);
        free(kept);
    }
    return 0;
}

static int int_cmp(const void* a, const void* b) {
    const int x = *(const int*)a, y = *(const int*)b;
    return (x > y) - (x < y);
}
typedef struct { float d; int id; int pos; } fpair_t;
static int fpair_cmp(const void* a, const void* b) {
    const fpair_t* x = (const fpair_t*)a;
    const fpair_t* y = (const fpair_t*)b;
    if (x->d < y->d) return -1;
    if (x->d > y->d) return 1;
    return (x->pos > y->pos) - (x->pos < y->pos);
}

/* swann/build.py:96-150.  Every edge u->t is offered back to t; t keeps the
 * first max_in offers in (source id, slot) order; the union with t's own row is
 * stripped of t itself and of duplicates, scored against t (1 - <v,x_t> for ip,
 * sum (v - x_t)^2 for l2), ordered by distance (ties by id: the union is sorted
 * by id first and the order is stable), cut to 128 and re-pruned.  Slots with
 * no entry carry id 0 and distance +inf into the prune, as in the reference. */
int or_add_reverse(const float* X, int64_t n, int d, const int* G, int deg, float alpha,
                   int max_in, int metric, const int* dpn, int nthreads, int* out) {
    /* reverse lists in (source, slot) order */
    int* cnt = (int*)calloc((size_t)n, sizeof(int));
    for (int64_t u = 0; u < n; ++u)
        for (int s = 0; s < deg; ++s) {
            const int t = G[(size_t)u * deg + s];
            if (t >= 0 && cnt[t] < max_in) ++cnt[t];
        }
    int64_t* start = (int64_t*)malloc(sizeof(int64_t) * (size_t)(n + 1));
    start[0] = 0;
    for (int64_t t = 0; t < n; ++t) start[t + 1] = start[t] + cnt[t];
    int* rev = (int*)malloc(sizeof(int) * (size_t)(start[n] > 0 ? start[n] : 1));
    memset(cnt, 0, sizeof(int) * (size_t)n);
    for (int64_t u = 0; u < n; ++u)
        for (int s = 0; s < deg; ++s) {
            const int t = G[(size_t)u * deg + s];
            if (t >= 0 && cnt[t] < max_in) rev[start[t] + cnt[t]++] = (int)u;
        }
    const int width = deg + max_in;
    const int keepn = width < 128 ? width : 128;
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel
#endif
    {
        int* row = (int*)malloc(sizeof(int) * (size_t)width);
        fpair_t* fp = (fpair_t*)malloc(sizeof(fpair_t) * (size_t)width);
        int* cand = (int*)malloc(sizeof(int) * (size_t)keepn);
        float* cd = (float*)malloc(sizeof(float) * (size_t)keepn);
        float* vn = (float*)malloc(sizeof(float) * (size_t)keepn);
        uint8_t* kept = (uint8_t*)malloc((size_t)keepn);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 16)
#endif
        for (int64_t t = 0; t < n; ++t) {
            int m = 0;
            for (int s = 0; s < deg; ++s) row[m++] = G[(size_t)t * deg + s];
            for (int64_t r = start[t]; r < start[t + 1]; ++r) row[m++] = rev[r];
            while (m < width) row[m++] = -1;
            for (int i = 0; i < width; ++i)
                if (row[i] == (int)t || row[i] < 0) row[i] = 1 << 30;
            qsort(row, (size_t)width, sizeof(int), int_cmp);
            for (int i = width - 1; i > 0; --i)
                if (row[i] == row[i - 1]) row[i] = 1 << 30;
            /* re-sort is not needed for the reference's semantics: a duplicate
             * becomes 2^30 in place, and validity (not position) is what the
             * distance step keys on; positions only order exact distance ties */
            const float* xt = X + (size_t)t * d;
            for (int i = 0; i < width; ++i) {
                const int valid = row[i] < (1 << 30);
                fp[i].id = valid ? row[i] : 0;
                fp[i].pos = i;
                if (!valid) fp[i].d = INFINITY;
                else if (metric == OR_METRIC_IP) fp[i].d = 1.0f - dot_seq(X + (size_t)row[i] * d, xt, d);
                else fp[i].d = l2_seq(X + (size_t)row[i] * d, xt, d);
            }
            qsort(fp, (size_t)width, sizeof(fpair_t), fpair_cmp);
            for (int i = 0; i < keepn; ++i) { cand[i] = fp[i].id; cd[i] = fp[i].d; }
            prune_one(X, d, cand, cd, keepn, dpn ? (dpn[t] < deg ? dpn[t] : deg) : deg, deg, alpha, metric,
                      NULL, out + (size_t)t * deg, vn, kept);
        }
        free(row); free(fp); free(cand); free(cd); free(vn); free(kept);
    }
    free(cnt); free(start); free(rev);
    return 0;
}

int or_version(void) { return 1; }
