"""Generate the golden vectors by running the REFERENCE's own code.

Runs only where the reference tree is mounted (its Python modules are
importable there; they do not travel to the GPU box).  Imports, read-only:

  swann/_refcpu.py   team_distance, init_state, advance, run
  swann/_engine.py   _merge_branches_tensor (the merge's tensor definition)
  swann/_select.py   select_nearest (on CPU tensors, fp32)
  swann/build.py     knn_candidates, robust_prune, add_reverse (on CPU tensors)

and writes outputs (plus input digests) to tests/golden/*.npz.

    python tests/golden/make_golden.py [--ref REFERENCE_ROOT] [--skip-c1]
"""
from __future__ import annotations

import argparse
import os
import functools
import multiprocessing as mp
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import cases  # noqa: E402

REF = None


def _import_ref(path):
    sys.path.insert(0, str(path))
    import swann._refcpu as refcpu  # noqa: F401
    return refcpu


def gen_distances(refcpu):
    out = {}
    for (d, team, vec, metric) in cases.DIST_GRID:
        q, x = cases.distance_pairs(d, seed=d * 131 + team * 7 + vec + metric)
        vals = np.array([refcpu.team_distance(q[i], x[i], metric, team, vec) for i in range(q.shape[0])],
                        np.float32)
        out[f"{d}_{team}_{vec}_{metric}"] = vals
        out[f"{d}_{team}_{vec}_{metric}_digest"] = np.array(cases.digest(q, x))
    np.savez_compressed(HERE / "team_distance.npz", **out)
    print("team_distance:", len(cases.DIST_GRID), "cases")


def _queue_arrays(st, L):
    ids = np.full(L, -1, np.int32)
    dist = np.full(L, np.finfo(np.float32).max, np.float32)
    expd = np.ones(L, np.uint8)
    lin = np.zeros(L, np.uint8)
    for i, e in enumerate(st["queue"]):
        ids[i], dist[i], expd[i], lin[i] = e[0], np.float32(e[1]), int(e[2]), int(e[3])
    c = st["counters"]
    return ids, dist, expd, lin, np.array([c["expansions"], c["dist_evals"], c["exhausted"]], np.int32)


def gen_branches(refcpu):
    """Single-branch runs: the shapes of the reference engine tests."""
    out = {}
    runs = []
    # teams x metrics, one seed per branch (test_engine.py:42-78's shape)
    for metric in (0, 1):
        X, G = cases.toy(metric=metric)
        rng = np.random.default_rng(7)
        nq, J, L, budget = 5, 3, 16, 12
        Qv = rng.standard_normal((nq, X.shape[1]), dtype=np.float32)
        if metric == 0:
            Qv /= np.linalg.norm(Qv, axis=1, keepdims=True)
        seeds = rng.integers(0, X.shape[0], size=(nq, J)).astype(np.int32)
        for team in (4, 8, 16, 32):
            runs.append(dict(name=f"team{team}_m{metric}", X=X, G=G, Q=Qv, seeds=seeds[:, :, None],
                             L=L, B=budget, metric=metric, team=team, policy=0, eps=-1.0, kstop=10,
                             delta=budget, vec=4, toy_metric=metric, toy_seed=0))
    # several seeds per branch, both policies (test_engine.py:263-288)
    X, G = cases.toy(seed=53)
    rng = np.random.default_rng(59)
    Qv = cases.unit_queries(4, X.shape[1], 59)
    seeds = rng.integers(0, X.shape[0], (4, 1, 6)).astype(np.int32)
    for policy in (0, 1):
        runs.append(dict(name=f"multiseed_p{policy}", X=X, G=G, Q=Qv, seeds=seeds, L=32, B=20,
                         metric=0, team=32, policy=policy, eps=-1.0, kstop=10, delta=20, vec=4,
                         toy_metric=0, toy_seed=53))
    # per-lineage early stop (test_engine.py:291-316)
    X, G = cases.toy(seed=71)
    rng = np.random.default_rng(73)
    Qv = cases.unit_queries(4, X.shape[1], 73)
    seeds = rng.integers(0, X.shape[0], (4, 1, 4)).astype(np.int32)
    for eps in (0.0, 0.1, 0.25):
        runs.append(dict(name=f"early_{eps}", X=X, G=G, Q=Qv, seeds=seeds, L=32, B=64, metric=0,
                         team=32, policy=1, eps=eps, kstop=10, delta=64, vec=4,
                         toy_metric=0, toy_seed=71))
    # POLICY_BEST with early stop, kstop < L, and a partial advance
    X, G = cases.toy(seed=5, metric=1)
    Qv = cases.unit_queries(3, X.shape[1], 5) * 3.0
    seeds = np.random.default_rng(5).integers(0, X.shape[0], (3, 2, 1)).astype(np.int32)
    runs.append(dict(name="best_eps_l2", X=X, G=G, Q=Qv, seeds=seeds, L=12, B=64, metric=1,
                     team=16, policy=0, eps=0.05, kstop=10, delta=64, vec=4, toy_metric=1, toy_seed=5))
    runs.append(dict(name="partial_delta", X=X, G=G, Q=Qv, seeds=seeds, L=12, B=64, metric=1,
                     team=8, policy=0, eps=-1.0, kstop=10, delta=5, vec=4, toy_metric=1, toy_seed=5))
    # fp16-widened corpus: vec = 8 (the kernel's 16-byte fp16 loads)
    X, G = cases.toy(seed=41)
    Xh = X.astype(np.float16).astype(np.float32)
    Qv = cases.unit_queries(3, X.shape[1], 41)
    seeds = np.random.default_rng(41).integers(0, X.shape[0], (3, 2, 1)).astype(np.int32)
    for team in (4, 16):
        runs.append(dict(name=f"fp16_team{team}", X=Xh, G=G, Q=Qv, seeds=seeds, L=16, B=16, metric=0,
                         team=team, policy=0, eps=-1.0, kstop=10, delta=16, vec=8, toy_metric=0,
                         toy_seed=41, half=True))

    orig = refcpu.team_distance
    for r in runs:
        refcpu.team_distance = functools.partial(orig, vec=r["vec"])
        nq, J, V = r["seeds"].shape
        L = r["L"]
        ids = np.empty((nq, J, L), np.int32); dist = np.empty((nq, J, L), np.float32)
        expd = np.empty((nq, J, L), np.uint8); lin = np.empty((nq, J, L), np.uint8)
        ctr = np.empty((nq, J, 3), np.int32)
        for qi in range(nq):
            for j in range(J):
                sd = [int(s) for s in r["seeds"][qi, j]]
                st = refcpu.init_state(r["X"], r["Q"][qi], sd if V > 1 else sd[0], L=L, B=r["B"],
                                       metric=r["metric"], team=r["team"], policy=r["policy"],
                                       stop_eps=r["eps"], kstop=r["kstop"])
                st = refcpu.advance(r["X"], r["G"], r["Q"][qi], st, r["delta"])
                ids[qi, j], dist[qi, j], expd[qi, j], lin[qi, j], ctr[qi, j] = _queue_arrays(st, L)
        p = r["name"]
        out[p + "_ids"], out[p + "_dist"], out[p + "_exp"], out[p + "_lin"], out[p + "_ctr"] = \
            ids, dist, expd, lin, ctr
        out[p + "_Q"], out[p + "_seeds"] = r["Q"], r["seeds"]
        out[p + "_knobs"] = np.array([r["L"], r["B"], r["metric"], r["team"], r["policy"], r["kstop"],
                                      r["delta"], r["vec"], r["toy_metric"], r["toy_seed"],
                                      int(r.get("half", False))], np.int64)
        out[p + "_eps"] = np.float32(r["eps"])
        out[p + "_digest"] = np.array(cases.digest(r["X"], r["G"]))
    refcpu.team_distance = orig
    out["names"] = np.array([r["name"] for r in runs])
    np.savez_compressed(HERE / "branches.npz", **out)
    print("branches:", len(runs), "runs")


def gen_merge():
    import torch
    from swann import _engine
    ids, dist = cases.merge_inputs()
    oi, od = _engine._merge_branches_tensor(torch.from_numpy(ids), torch.from_numpy(dist), 10)
    np.savez_compressed(HERE / "merge.npz", ids=oi.numpy(), dist=od.numpy(),
                        digest=np.array(cases.digest(ids, dist)))
    print("merge: done")


def gen_build():
    import torch
    from swann import build as B
    out = {}
    torch.set_num_threads(8)
    for metric, name in ((0, "ip"), (1, "l2")):
        X = cases.build_corpus(1000, 64, seed=11 + metric, metric=metric)
        Xt = torch.from_numpy(X)
        cand, cd = B.knn_candidates(Xt, 64, chunk=256, metric=name)
        G1 = B.robust_prune(Xt, cand, cd, 32, alpha=1.2, chunk=256, metric=name)
        G2 = B.add_reverse(Xt, G1, 32, alpha=1.2, metric=name)
        out[f"{name}_cand"], out[f"{name}_cdist"] = cand.numpy(), cd.numpy()
        out[f"{name}_prune"], out[f"{name}_graph"] = G1.numpy(), G2.numpy()
        out[f"{name}_digest"] = np.array(cases.digest(X))
    np.savez_compressed(HERE / "build.npz", **out)
    print("build: done")


def _c1_query(args):
    qi, seeds_row, X, G, Q, knobs = args
    import swann._refcpu as refcpu
    L, Bd, metric, team, eps, k = knobs
    pool = {}
    evals = 0
    for s in seeds_row:
        st = refcpu.run(X, G, Q[qi], int(s), L=L, B=Bd, metric=metric, team=team, stop_eps=eps,
                        kstop=min(k, L))
        evals += st["counters"]["dist_evals"]
        for i, d in refcpu.topk(st, min(k, L)):
            pool.setdefault(int(i), float(d))
    best = sorted(pool.items(), key=lambda kv: (kv[1], kv[0]))[:k]
    ids = [i for i, _ in best] + [-1] * (k - len(best))
    dd = [d for _, d in best] + [float("inf")] * (k - len(best))
    return qi, ids, dd, evals


def gen_c1(refpath):
    """BASELINE config 1 end to end: the reference build (CPU torch), catalogue
    and fp32 seed selection, then _refcpu search of every query's 32 branches."""
    import torch
    from swann import build as B
    from swann import _select as S
    torch.set_num_threads(8)
    X, Q = cases.c1_data()
    t = time.time()
    Xt = torch.from_numpy(X)
    cand, cd = B.knn_candidates(Xt, 128, metric="l2")
    G1 = B.robust_prune(Xt, cand, cd, 64, alpha=1.2, metric="l2")
    G = B.add_reverse(Xt, G1, 64, alpha=1.2, metric="l2").numpy()
    print(f"c1 build {time.time() - t:.1f}s")
    cat = cases.catalogue(X.shape[0])
    Vp = S.pool_vectors(Xt, torch.from_numpy(cat))
    ent = S.select_nearest(torch.from_numpy(Q), Vp, 32, metric=1, precision="fp32").numpy()
    seeds = cat[ent].astype(np.int32)
    knobs = (12, 64, 1, 16, 0.05, 10)
    t = time.time()
    ctx = mp.get_context("spawn")
    with ctx.Pool(8, initializer=_import_ref, initargs=(refpath,)) as pool:
        res = pool.map(_c1_query, [(qi, seeds[qi], X, G, Q, knobs) for qi in range(Q.shape[0])])
    print(f"c1 search {time.time() - t:.1f}s")
    ids = np.array([r[1] for r in sorted(res)], np.int32)
    dist = np.array([r[2] for r in sorted(res)], np.float32)
    evals = np.array([r[3] for r in sorted(res)], np.int64)
    np.savez_compressed(HERE / "c1.npz", graph=G.astype(np.int16), cand=cand.numpy()[:64],
                        cdist=cd.numpy()[:64], seeds=seeds, ids=ids, dist=dist, evals=evals,
                        digest=np.array(cases.digest(X, Q)), knobs=np.array(knobs[:4] + (10,), np.int64),
                        eps=np.float32(knobs[4]))
    print("c1: done")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("SWANN_REFERENCE"),
                    help="root of the reference project (default: $SWANN_REFERENCE)")
    ap.add_argument("--skip-c1", action="store_true")
    a = ap.parse_args()
    if not a.ref:
        ap.error("name the reference project's root with --ref or $SWANN_REFERENCE")
    refcpu = _import_ref(a.ref)
    gen_distances(refcpu)
    gen_branches(refcpu)
    gen_merge()
    gen_build()
    if not a.skip_c1:
        gen_c1(a.ref)


if __name__ == "__main__":
    main()
