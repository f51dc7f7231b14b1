"""The C oracle against golden vectors produced by the reference's own code.

The fixtures in tests/golden/ were written by make_golden.py, which ran the
reference's swann/_refcpu.py, swann/_engine.py (tensor merge), swann/_select.py
and swann/build.py.  These tests pin the oracle before anything is checked
against it.  CPU only.
"""
import numpy as np
import pytest

import cases
from oracle import oracle as O

GOLD = cases.__file__.rsplit("/", 1)[0]


def load(name):
    return np.load(f"{GOLD}/{name}.npz", allow_pickle=False)


def test_team_distance_bitwise():
    """Every (d, team, vec, metric) of the grid, bit for bit (_refcpu.py:21-48)."""
    g = load("team_distance")
    with O.square_mode("refcpu"):
        _check_distances(g)


def test_square_modes_differ_only_by_rounding():
    """The kernel squares an L2 term with one rounded multiply, _refcpu with
    numpy's float32 power (libm powf), which is not always correctly rounded.
    The two definitions give the same distance on most inputs and differ by a
    few ulps at most where they do not."""
    rng = np.random.default_rng(5)
    q, x = rng.standard_normal((2, 400, 64), dtype=np.float32)
    a = np.array([O.team_distance(q[i], x[i], 1, 16, 4) for i in range(400)], np.float32)
    with O.square_mode("refcpu"):
        b = np.array([O.team_distance(q[i], x[i], 1, 16, 4) for i in range(400)], np.float32)
    ulp = np.abs(a.view(np.int32).astype(np.int64) - b.view(np.int32).astype(np.int64))
    assert ulp.max() <= 64 and (ulp == 0).mean() > 0.8


def _check_distances(g):
    for (d, team, vec, metric) in cases.DIST_GRID:
        q, x = cases.distance_pairs(d, seed=d * 131 + team * 7 + vec + metric)
        key = f"{d}_{team}_{vec}_{metric}"
        assert str(g[key + "_digest"]) == cases.digest(q, x), "input generator drifted"
        got = np.array([O.team_distance(q[i], x[i], metric, team, vec) for i in range(q.shape[0])],
                       np.float32)
        assert np.array_equal(got.view(np.int32), g[key].view(np.int32)), key


def test_branch_runs_bitwise():
    """Queue ids, distances, expanded flags, lineage and counters of every
    single-branch run equal _refcpu's (engine-test shapes, both policies, early
    stop, partial advance, fp16-widened corpus)."""
    g = load("branches")
    for name in g["names"]:
        name = str(name)
        L, B, metric, team, policy, kstop, delta, vec, tm, ts, half = [int(v) for v in g[name + "_knobs"]]
        eps = float(g[name + "_eps"])
        X, G = cases.toy(seed=ts, metric=tm)
        if half:
            X = X.astype(np.float16).astype(np.float32)
        assert str(g[name + "_digest"]) == cases.digest(X, G), "toy corpus drifted"
        Q, seeds = g[name + "_Q"], g[name + "_seeds"]
        nq, J, V = seeds.shape
        for qi in range(nq):
            for j in range(J):
                with O.square_mode("refcpu"):
                        r = O.branch_run(X, G, Q[qi], seeds[qi, j], L=L, B=B, metric=metric, team=team,
                                     vec=vec, policy=policy, stop_eps=eps, kstop=kstop, delta=delta)
                tag = f"{name} q={qi} j={j}"
                assert np.array_equal(r["ids"], g[name + "_ids"][qi, j]), tag
                assert np.array_equal(r["dist"].view(np.int32), g[name + "_dist"][qi, j].view(np.int32)), tag
                assert np.array_equal(r["expanded"], g[name + "_exp"][qi, j]), tag
                assert np.array_equal(r["lineage"], g[name + "_lin"][qi, j]), tag
                exp_, evals, exh = g[name + "_ctr"][qi, j]
                assert r["counters"][0] == exp_ and r["counters"][1] == evals, tag
                assert r["counters"][3] == exh, tag


def test_merge_matches_reference_tensor_merge():
    g = load("merge")
    ids, dist = cases.merge_inputs()
    assert str(g["digest"]) == cases.digest(ids, dist)
    oi, od = O.merge_branches(ids, dist, 10)
    assert np.array_equal(oi, g["ids"])
    assert np.array_equal(od, g["dist"])


def _exact_dist(X, i, js, metric):
    a = X[i].astype(np.float64)
    B = X[js].astype(np.float64)
    if metric == 0:
        return 1.0 - B @ a
    return ((B - a) ** 2).sum(1)


def _tol(X, metric):
    # fp32 evaluation noise of the reference's BLAS path, a few ulps of the
    # magnitudes that cancel in the expression
    d = X.shape[1]
    scale = 1.0 if metric == 0 else 2.0 * float((X.astype(np.float64) ** 2).sum(1).max())
    return 4.0 * d * 2.0 ** -24 * scale


@pytest.mark.parametrize("metric", [0, 1])
def test_knn_candidates_match_except_ties(metric):
    """Exact top-C (oracle, double) vs the reference's fp32 sweep: every
    position agrees or the two entries there are a tie within fp32 noise."""
    name = "ip" if metric == 0 else "l2"
    g = load("build")
    X = cases.build_corpus(1000, 64, seed=11 + metric, metric=metric)
    assert str(g[f"{name}_digest"]) == cases.digest(X)
    ref = g[f"{name}_cand"]
    idx, _ = O.knn_candidates(X, ref.shape[1], metric)
    tol = _tol(X, metric)
    bad = 0
    for i in range(X.shape[0]):
        if np.array_equal(idx[i], ref[i]):
            continue
        de_o = _exact_dist(X, i, idx[i], metric)
        de_r = _exact_dist(X, i, ref[i], metric)
        bad += int(np.any(np.abs(de_o - de_r) > tol))
    assert bad == 0


def _near_tie_decisions(X, cand, du, alpha, metric, tol):
    """True when some prune decision of this row is within `tol` of flipping."""
    V = X[np.maximum(cand, 0)].astype(np.float64)
    dots = V @ V.T
    if metric == 0:
        pair = 1.0 - dots
    else:
        vn = (V * V).sum(1)
        pair = np.maximum(vn[None, :] - 2.0 * dots + vn[:, None], 0.0)
    marg = np.abs(np.float64(np.float32(alpha)) * pair - du.astype(np.float64)[None, :])
    return bool((marg <= tol).any())


@pytest.mark.parametrize("metric", [0, 1])
def test_robust_prune_bitexact_given_candidates(metric):
    """Oracle prune on the reference's own candidates equals the reference's
    prune on every row whose decisions are not within fp32 noise of a tie."""
    name = "ip" if metric == 0 else "l2"
    g = load("build")
    X = cases.build_corpus(1000, 64, seed=11 + metric, metric=metric)
    cand, cd, ref = g[f"{name}_cand"], g[f"{name}_cdist"], g[f"{name}_prune"]
    got = O.robust_prune(X, cand, cd, ref.shape[1], 1.2, metric)
    tol = _tol(X, metric)
    rows = np.nonzero((got != ref).any(1))[0]
    unexplained = [int(r) for r in rows if not _near_tie_decisions(X, cand[r], cd[r], 1.2, metric, tol)]
    assert not unexplained, unexplained[:10]
    assert len(rows) <= 0.02 * X.shape[0]


@pytest.mark.parametrize("metric", [0, 1])
def test_add_reverse_matches_except_ties(metric):
    name = "ip" if metric == 0 else "l2"
    g = load("build")
    X = cases.build_corpus(1000, 64, seed=11 + metric, metric=metric)
    G1, ref = g[f"{name}_prune"], g[f"{name}_graph"]
    got = O.add_reverse(X, G1, ref.shape[1], 1.2, 64, metric)
    rows = np.nonzero((got != ref).any(1))[0]
    tol = _tol(X, metric)
    unexplained = []
    for t in rows:
        # the union the row was re-pruned from, in exact distance order
        ids = set(int(v) for v in G1[t] if v >= 0 and v != t)
        ids |= set(int(u) for u in np.nonzero((G1 == t).any(1))[0] if u != t)
        ids = np.array(sorted(ids), np.int64)
        de = _exact_dist(X, int(t), ids, metric)
        o = np.argsort(de, kind="stable")
        ids, de = ids[o][:128], de[o][:128]
        close = np.any(np.diff(de) <= tol) if len(de) > 1 else False
        if not close and not _near_tie_decisions(X, ids.astype(np.int32), de.astype(np.float32), 1.2, metric, tol):
            unexplained.append(int(t))
    assert not unexplained, unexplained[:10]
    assert len(rows) <= 0.03 * X.shape[0]


def test_c1_search_matches_reference():
    """BASELINE config 1 end to end (n=10k, d=128, L2, 32 branches, queue 12,
    budget 64, stop_eps 0.05, team 16) on the reference's graph and seeds: the
    oracle's merged top-10 ids and distances equal _refcpu's, query by query,
    and so do the distance-evaluation counts."""
    g = load("c1")
    X, Q = cases.c1_data()
    assert str(g["digest"]) == cases.digest(X, Q)
    G = g["graph"].astype(np.int32)
    L, B, metric, team, k = [int(v) for v in g["knobs"]]
    with O.square_mode("refcpu"):
        ids, dist, ctr = O.search(X, G, Q, g["seeds"], k=k, L=L, B=B, metric=metric, team=team,
                                  stop_eps=float(g["eps"]), kstop=min(k, L), counters=True)
    assert np.array_equal(ids, g["ids"])
    assert np.array_equal(dist.view(np.int32), g["dist"].view(np.int32))
    assert np.array_equal(ctr[:, :, 1].sum(1), g["evals"])
