"""GPU parity of the search engine (swann_b200/_engine.py over csrc/search.cu).

Each check of the reference's own engine tests (tests/test_engine.py of
geniussyn/SWANN) is restated against two checkers:

  * the C oracle (oracle/swann_oracle.c), bit for bit, in the kernel's
    arithmetic (one rounded multiply per L2 term);
  * the reference's own kernels compiled for sm_100a (oracle/_ref), bit for
    bit, where that build is present.
"""
import numpy as np
import pytest
import torch

import cases
from oracle import oracle as O
from refcheck import DEV, ref_production, ref_run, same_state, to_gpu
from swann_b200 import _engine as E

pytestmark = pytest.mark.gpu
TEAMS = (4, 8, 16, 32)


def test_cpu_gpu_exact():
    """Same queue, same distances, bit for bit, at every team size (IP and L2)."""
    for metric in (E.METRIC_IP, E.METRIC_L2):
        X, G = cases.toy(metric=metric)
        rng = np.random.default_rng(7)
        nq, J, L, budget = 5, 3, 16, 12
        Qv = rng.standard_normal((nq, X.shape[1]), dtype=np.float32)
        if metric == E.METRIC_IP:
            Qv /= np.linalg.norm(Qv, axis=1, keepdims=True)
        seeds = rng.integers(0, X.shape[0], size=(nq, J)).astype(np.int32)
        Xg, Gg, Qg = to_gpu(X, G, Qv)
        for team in TEAMS:
            st = E.init_states(Xg, Qg, torch.from_numpy(seeds), L=L, B=budget, D=G.shape[1], metric=metric,
                               team_size=team)
            E.advance(Xg, Gg, Qg, st, budget)
            st.check()
            gi, gd = st.ids.cpu().numpy(), st.dist.cpu().numpy()
            ge, gc = st.expanded.cpu().numpy(), st.counters.cpu().numpy()
            for qi in range(nq):
                for j in range(J):
                    r = O.branch_run(X, G, Qv[qi], seeds[qi, j], L=L, B=budget, metric=metric, team=team)
                    tag = f"metric={metric} team={team} q={qi} j={j}"
                    assert np.array_equal(r["ids"], gi[qi, j]), tag
                    assert np.array_equal(r["dist"].view(np.int32), gd[qi, j].view(np.int32)), tag
                    assert np.array_equal(r["expanded"], ge[qi, j]), tag
                    assert gc[qi, j, 0] == r["counters"][0] and gc[qi, j, 1] == r["counters"][1], tag
            ref = ref_run(Xg, Gg, Qg, torch.from_numpy(seeds), L, budget, metric, team)
            if ref is not None:
                same_state(st, ref)


def test_resume_equivalence():
    """advance(a) then advance(b) is advance(a + b)."""
    X, G = cases.toy(seed=3)
    rng = np.random.default_rng(11)
    nq, J, L, budget = 8, 4, 32, 24
    Qv = cases.unit_queries(nq, X.shape[1], 11)
    seeds = torch.from_numpy(rng.integers(0, X.shape[0], (nq, J)).astype(np.int32))
    Xg, Gg, Qg = to_gpu(X, G, Qv)
    kw = dict(L=L, B=budget, D=G.shape[1], team_size=32)
    one = E.init_states(Xg, Qg, seeds, **kw)
    E.advance(Xg, Gg, Qg, one, budget)
    for split in (1, 2, 7, budget - 1):
        two = E.init_states(Xg, Qg, seeds, **kw)
        E.advance(Xg, Gg, Qg, two, split)
        E.advance(Xg, Gg, Qg, two, budget - split)
        assert torch.equal(one.ids, two.ids), split
        assert torch.equal(one.dist, two.dist), split
        assert torch.equal(one.expanded, two.expanded), split
        assert torch.equal(one.counters, two.counters), split


def test_budget_is_a_state_property():
    X, G = cases.toy(seed=5)
    rng = np.random.default_rng(13)
    Qv = cases.unit_queries(4, X.shape[1], 13)
    seeds = torch.from_numpy(rng.integers(0, X.shape[0], (4, 2)).astype(np.int32))
    Xg, Gg, Qg = to_gpu(X, G, Qv)
    st = E.init_states(Xg, Qg, seeds, L=16, B=10, D=G.shape[1])
    E.advance(Xg, Gg, Qg, st, 100)
    assert int(st.expansions.max()) == 10


def test_brute_force_on_complete_graph():
    """One expansion of a complete graph sees everything: exact top-10."""
    n, d, L = 96, 48, 16
    rng = np.random.default_rng(17)
    X = rng.standard_normal((n, d), dtype=np.float32)
    X /= np.linalg.norm(X, axis=1, keepdims=True)
    G = np.stack([np.delete(np.arange(n), i) for i in range(n)]).astype(np.int32)[:, :95]
    Qv = rng.standard_normal((6, d), dtype=np.float32)
    Qv /= np.linalg.norm(Qv, axis=1, keepdims=True)
    Xg, Gg, Qg = to_gpu(X, G, Qv)
    seeds = torch.zeros((6, 1), dtype=torch.int32)
    ids, dist, st = E.search(Xg, Gg, Qg, seeds, k=10, L=L, B=1)
    exact = 1.0 - (Qv @ X.T)
    want = np.argsort(exact, axis=1, kind="stable")[:, :10]
    assert (ids.cpu().numpy() == want).all()
    assert np.allclose(dist.cpu().numpy(), np.take_along_axis(exact, want, 1), atol=2e-6)


def test_dead_branch_and_exhaustion():
    n, d = 64, 16
    rng = np.random.default_rng(19)
    X = rng.standard_normal((n, d), dtype=np.float32)
    X /= np.linalg.norm(X, axis=1, keepdims=True)
    G = np.full((n, 8), -1, dtype=np.int32)
    Qv = rng.standard_normal((2, d), dtype=np.float32)
    Qv /= np.linalg.norm(Qv, axis=1, keepdims=True)
    Xg, Gg, Qg = to_gpu(X, G, Qv)
    seeds = torch.tensor([[0, -1], [5, -1]], dtype=torch.int32)
    st = E.init_states(Xg, Qg, seeds, L=16, B=16, D=8)
    E.advance(Xg, Gg, Qg, st, 16)
    st.check()
    assert int(st.expansions[0, 0]) == 1 and int(st.exhausted[0, 0]) == 1
    assert int(st.expansions[0, 1]) == 0 and int(st.exhausted[0, 1]) == 1
    assert int(st.ids[0, 1, 0]) == -1
    ids, _ = E.branch_topk(st, 10)
    assert int((ids >= 0).sum()) == 2


def test_visited_overflow_is_reported():
    X, G = cases.toy(n=1000, seed=23)
    Qv = cases.unit_queries(2, X.shape[1], 29)
    Xg, Gg, Qg = to_gpu(X, G, Qv)
    st = E.init_states(Xg, Qg, torch.zeros((2, 1), dtype=torch.int32), L=16, B=16, D=G.shape[1])
    st.visited = torch.zeros((2, 1, 64), dtype=torch.int32, device=DEV)   # far too small
    st.counters.zero_()
    E.advance(Xg, Gg, Qg, st, 16)
    assert int(st.hash_failures.sum()) > 0
    with pytest.raises(RuntimeError):
        st.check()


def test_merge_dedup():
    """The merged top-k is the exact best over the union of branch results, once each."""
    X, G = cases.toy(seed=31)
    rng = np.random.default_rng(37)
    nq, J, k = 6, 5, 10
    Qv = cases.unit_queries(nq, X.shape[1], 37)
    seeds = torch.from_numpy(rng.integers(0, X.shape[0], (nq, J)).astype(np.int32))
    Xg, Gg, Qg = to_gpu(X, G, Qv)
    ids, dist, st = E.search(Xg, Gg, Qg, seeds, k=k, L=16, B=16)
    bi, bd = E.branch_topk(st, k)
    bi, bd = bi.cpu().numpy(), bd.cpu().numpy()
    gi = ids.cpu().numpy()
    for q in range(nq):
        pool = {}
        for j in range(J):
            for t in range(k):
                if bi[q, j, t] >= 0:
                    pool.setdefault(int(bi[q, j, t]), float(bd[q, j, t]))
        want = [i for i, _ in sorted(pool.items(), key=lambda kv: (kv[1], kv[0]))[:k]]
        got = [int(i) for i in gi[q] if i >= 0]
        assert got == want
        assert len(set(got)) == len(got)


def test_merge_kernels_match_definition():
    """Standalone merge kernel and the tensor definition agree with the oracle
    on inputs with repeats across branches and empty slots."""
    ids, dist = cases.merge_inputs(Q=40, J=9, kk=12, seed=8)
    oi, od = O.merge_branches(ids, dist, 10)
    gi, gd = E.merge_branches(torch.from_numpy(ids).to(DEV), torch.from_numpy(dist).to(DEV), 10)
    assert np.array_equal(gi.cpu().numpy(), oi) and np.array_equal(gd.cpu().numpy(), od)
    ti, td = E._merge_branches_tensor(torch.from_numpy(ids).to(DEV), torch.from_numpy(dist).to(DEV), 10)
    assert np.array_equal(ti.cpu().numpy(), oi) and np.array_equal(td.cpu().numpy(), od)
    R = O.ref_kernels()
    if R is not None:
        ri, rd = R.merge_branches(torch.from_numpy(ids).to(DEV), torch.from_numpy(dist).to(DEV), 10)
        assert np.array_equal(ri.cpu().numpy(), oi) and np.array_equal(rd.cpu().numpy(), od)


def test_determinism():
    X, G = cases.toy(seed=41)
    rng = np.random.default_rng(43)
    Qv = cases.unit_queries(16, X.shape[1], 43)
    seeds = torch.from_numpy(rng.integers(0, X.shape[0], (16, 8)).astype(np.int32))
    Xg, Gg, Qg = to_gpu(X, G, Qv)
    ref = None
    for _ in range(5):
        ids, dist, st = E.search(Xg, Gg, Qg, seeds, k=10, L=16, B=16)
        now = (ids.cpu().numpy().copy(), dist.cpu().numpy().copy(), st.counters.cpu().numpy().copy())
        if ref is None:
            ref = now
        else:
            for a, b in zip(ref, now):
                assert (a == b).all()


def test_multiseed_matches_cpu():
    X, G = cases.toy(seed=53)
    rng = np.random.default_rng(59)
    nq, V, L, budget = 4, 6, 32, 20
    Qv = cases.unit_queries(nq, X.shape[1], 59)
    seeds = rng.integers(0, X.shape[0], (nq, 1, V)).astype(np.int32)
    Xg, Gg, Qg = to_gpu(X, G, Qv)
    for policy in (E.POLICY_BEST, E.POLICY_ROUND_ROBIN):
        st = E.init_states(Xg, Qg, torch.from_numpy(seeds), L=L, B=budget, D=G.shape[1], policy=policy)
        E.advance(Xg, Gg, Qg, st, budget)
        st.check()
        gi, gd, gl = st.ids.cpu().numpy(), st.dist.cpu().numpy(), st.lineage.cpu().numpy()
        for q in range(nq):
            r = O.branch_run(X, G, Qv[q], seeds[q, 0], L=L, B=budget, policy=policy)
            assert np.array_equal(r["ids"], gi[q, 0]), f"policy {policy}"
            assert np.array_equal(r["dist"], gd[q, 0])
            assert np.array_equal(r["lineage"], gl[q, 0])
        ref = ref_run(Xg, Gg, Qg, torch.from_numpy(seeds), L, budget, 0, 32, policy=policy)
        if ref is not None:
            same_state(st, ref)


def test_early_stop_matches_cpu():
    X, G = cases.toy(seed=71)
    rng = np.random.default_rng(73)
    nq, V, L, budget, k = 4, 4, 32, 64, 10
    Qv = cases.unit_queries(nq, X.shape[1], 73)
    seeds = rng.integers(0, X.shape[0], (nq, 1, V)).astype(np.int32)
    Xg, Gg, Qg = to_gpu(X, G, Qv)
    for eps in (0.0, 0.1, 0.25):
        st = E.init_states(Xg, Qg, torch.from_numpy(seeds), L=L, B=budget, D=G.shape[1],
                           policy=E.POLICY_ROUND_ROBIN, stop_eps=eps, kstop=k)
        E.advance(Xg, Gg, Qg, st, budget)
        st.check()
        gi, gd = st.ids.cpu().numpy(), st.dist.cpu().numpy()
        for q in range(nq):
            r = O.branch_run(X, G, Qv[q], seeds[q, 0], L=L, B=budget, policy=E.POLICY_ROUND_ROBIN,
                             stop_eps=eps, kstop=k)
            assert np.array_equal(r["ids"], gi[q, 0]), f"eps={eps}"
            assert np.array_equal(r["dist"], gd[q, 0])
            assert r["counters"][0] == int(st.expansions[q, 0])
        assert int(st.expansions.max()) < budget
        ref = ref_run(Xg, Gg, Qg, torch.from_numpy(seeds), L, budget, 0, 32, policy=1, stop_eps=eps, kstop=k)
        if ref is not None:
            same_state(st, ref)


def test_shared_cache_is_free_of_consequence():
    X, G = cases.toy(seed=79)
    rng = np.random.default_rng(83)
    nq, Ent, L, budget = 16, 24, 32, 12
    Qv = cases.unit_queries(nq, X.shape[1], 83)
    seeds = torch.from_numpy(rng.integers(0, X.shape[0], (nq, Ent)).astype(np.int32))
    Xg, Gg, Qg = to_gpu(X, G, Qv)
    plain = E.search(Xg, Gg, Qg, seeds, k=10, L=L, B=budget)
    cached = E.search(Xg, Gg, Qg, seeds, k=10, L=L, B=budget, shared_cache=True)
    assert torch.equal(plain[0], cached[0])
    assert torch.equal(plain[1], cached[1])
    assert torch.equal(plain[2].ids, cached[2].ids)
    assert torch.equal(plain[2].expansions, cached[2].expansions)
    a = float(plain[2].dist_evals.sum(1).float().mean())
    b = float(cached[2].dist_evals.sum(1).float().mean())
    hits = float(cached[2].cache_hits.sum(1).float().mean())
    assert b < a
    assert abs((a - b) - hits) < 1e-6


def test_shared_state_beats_split_branches_on_work():
    X, G = cases.toy(seed=61)
    rng = np.random.default_rng(67)
    nq, V, budget = 32, 8, 64
    Qv = cases.unit_queries(nq, X.shape[1], 67)
    seeds = rng.integers(0, X.shape[0], (nq, V)).astype(np.int32)
    Xg, Gg, Qg = to_gpu(X, G, Qv)
    L = 64
    split = E.init_states(Xg, Qg, torch.from_numpy(seeds), L=L, B=budget // V, D=G.shape[1])
    E.advance(Xg, Gg, Qg, split, budget // V)
    shared = E.init_states(Xg, Qg, torch.from_numpy(seeds).unsqueeze(1), L=L, B=budget, D=G.shape[1],
                           policy=E.POLICY_ROUND_ROBIN)
    E.advance(Xg, Gg, Qg, shared, budget)
    a = (split.dist_evals.sum(1).float() / split.expansions.sum(1).clamp(min=1).float()).mean()
    b = (shared.dist_evals[:, 0].float() / shared.expansions[:, 0].clamp(min=1).float()).mean()
    assert float(b) < float(a)


# -- beyond the reference's own tests ------------------------------------------

@pytest.mark.parametrize("metric,team,L,V,policy,eps", [
    (0, 16, 12, 1, 0, 0.05), (1, 8, 16, 1, 0, -1.0), (0, 32, 32, 4, 1, 0.1), (1, 4, 64, 3, 1, -1.0),
])
def test_fused_equals_init_advance(metric, team, L, V, policy, eps):
    """The fused kernel (init + walk + top-k + merge in one launch) returns
    exactly what init_states + advance + branch_topk + merge_branches return."""
    X, G = cases.toy(seed=97, metric=metric)
    rng = np.random.default_rng(101)
    nq, J, B, k = 9, 5, 24, 10
    Qv = cases.unit_queries(nq, X.shape[1], 101)
    seeds = torch.from_numpy(rng.integers(0, X.shape[0], (nq, J, V)).astype(np.int32))
    Xg, Gg, Qg = to_gpu(X, G, Qv)
    st = E.init_states(Xg, Qg, seeds, L=L, B=B, D=G.shape[1], metric=metric, team_size=team, policy=policy,
                       stop_eps=eps, kstop=k)
    E.advance(Xg, Gg, Qg, st, B)
    bi, bd = E.branch_topk(st, k)
    ids0, dist0 = E.merge_branches(bi, bd, k)
    ids1, dist1, st1 = E.search(Xg, Gg, Qg, seeds, k=k, L=L, B=B, metric=metric, team_size=team, policy=policy,
                                stop_eps=eps)
    assert torch.equal(ids0, ids1) and torch.equal(dist0, dist1)
    assert torch.equal(st.ids, st1.ids) and torch.equal(st.counters, st1.counters)


def test_active_and_chunked_equal_one_shot():
    """advance over a compacted active list, re-formed between chunks, ends in
    the same states as one advance of the whole budget."""
    X, G = cases.toy(seed=7)
    rng = np.random.default_rng(5)
    nq, J, L, B = 6, 4, 16, 20
    Qv = cases.unit_queries(nq, X.shape[1], 5)
    seeds = torch.from_numpy(rng.integers(0, X.shape[0], (nq, J)).astype(np.int32))
    Xg, Gg, Qg = to_gpu(X, G, Qv)
    kw = dict(L=L, B=B, D=G.shape[1], team_size=16, stop_eps=0.1, kstop=10)
    one = E.init_states(Xg, Qg, seeds, **kw)
    E.advance(Xg, Gg, Qg, one, B)
    two = E.init_states(Xg, Qg, seeds, **kw)
    E.advance_chunked(Xg, Gg, Qg, two, B, 3)
    assert torch.equal(one.ids, two.ids) and torch.equal(one.dist, two.dist)
    assert torch.equal(one.counters[..., :4], two.counters[..., :4])


def test_fp16_corpus_bitwise():
    """fp16 rows: 8-element chunks per lane, widened exactly (vec = 8)."""
    X, G = cases.toy(seed=41)
    Xh = X.astype(np.float16)
    rng = np.random.default_rng(3)
    nq, J, L, B = 4, 3, 16, 16
    Qv = cases.unit_queries(nq, X.shape[1], 3)
    seeds = rng.integers(0, X.shape[0], (nq, J)).astype(np.int32)
    Xg, Gg, Qg = to_gpu(Xh, G, Qv)
    for team in (4, 16, 32):
        st = E.init_states(Xg, Qg, torch.from_numpy(seeds), L=L, B=B, D=G.shape[1], team_size=team)
        E.advance(Xg, Gg, Qg, st, B)
        gi, gd = st.ids.cpu().numpy(), st.dist.cpu().numpy()
        for q in range(nq):
            for j in range(J):
                r = O.branch_run(Xh, G, Qv[q], seeds[q, j], L=L, B=B, team=team, vec=8)
                assert np.array_equal(r["ids"], gi[q, j])
                assert np.array_equal(r["dist"], gd[q, j])
        ref = ref_run(Xg, Gg, Qg, torch.from_numpy(seeds), L, B, 0, team)
        if ref is not None:
            same_state(st, ref)


def test_c1_golden_search():
    """BASELINE config 1 on the reference's own graph and seeds (fixture made by
    running the reference's _refcpu): the GPU's merged top-10 ids equal the
    reference's, and every distance is within one ulp of it (the reference CPU
    path squares with powf, the kernel with one rounded multiply)."""
    g = np.load(f"{cases.__file__.rsplit('/', 1)[0]}/c1.npz")
    X, Q = cases.c1_data()
    G = g["graph"].astype(np.int32)
    L, B, metric, team, k = [int(v) for v in g["knobs"]]
    Xg, Gg, Qg = to_gpu(X, G, Q)
    ids, dist, st = E.search(Xg, Gg, Qg, torch.from_numpy(g["seeds"]), k=k, L=L, B=B, metric=metric,
                             team_size=team, stop_eps=float(g["eps"]))
    assert np.array_equal(ids.cpu().numpy(), g["ids"])
    ulp = np.abs(dist.cpu().numpy().view(np.int32).astype(np.int64) - g["dist"].view(np.int32).astype(np.int64))
    assert ulp.max() <= 1
    oi, od = O.search(X, G, Q, g["seeds"], k=k, L=L, B=B, metric=metric, team=team, stop_eps=float(g["eps"]),
                      kstop=min(k, L))
    assert np.array_equal(ids.cpu().numpy(), oi) and np.array_equal(dist.cpu().numpy(), od)
    assert np.array_equal(st.dist_evals.sum(1).cpu().numpy(), g["evals"])


def _recall(got, truth, k):
    return float(np.mean([len(set(a[:k]) & set(b[:k])) / k for a, b in zip(got, truth)]))


def test_production_mode_matches_reference_statistically():
    """Index.search's mode (shared table + bound + strict claims, no
    per-branch visited tables) on a C1-shaped corpus: the recall of the B200
    kernel is within 0.005 of the reference kernel's (the reference's own
    production flags) on the same graph and seeds, and every returned distance
    equals an exact recomputation within 1e-5 relative."""
    g = np.load(f"{cases.__file__.rsplit('/', 1)[0]}/c1.npz")
    X, _ = cases.c1_data()
    G = g["graph"].astype(np.int32)
    rng = np.random.default_rng(123)
    Q = rng.standard_normal((2000, X.shape[1]), dtype=np.float32)
    Xg, Gg, Qg = to_gpu(X, G, Q)
    from swann_b200 import _select as S
    cat = torch.from_numpy(cases.catalogue(X.shape[0])).to(DEV)
    ent = S.select_nearest(Qg, S.pool_vectors(Xg, cat), 32, metric=1)
    seeds = cat[ent].to(torch.int32)
    kw = dict(k=10, L=12, B=64, metric=1, team_size=16, stop_eps=0.05, shared_cache=True, shared_bound=True,
              exclusive=2, elide_visited=True)
    ids, dist, _ = E.search(Xg, Gg, Qg, seeds, **kw)
    truth = torch.topk(torch.cdist(Qg, Xg), 10, dim=1, largest=False).indices.cpu().numpy()
    mine = _recall(ids.cpu().numpy(), truth, 10)
    # every distance exact
    gi = ids.cpu().numpy()
    ok = gi >= 0
    ex = ((Q[:, None, :].astype(np.float64) - X[np.maximum(gi, 0)].astype(np.float64)) ** 2).sum(-1)
    rel = np.abs(dist.cpu().numpy().astype(np.float64) - ex) / np.maximum(ex, 1e-30)
    assert rel[ok].max() <= 1e-5
    ref = ref_production(Xg, Gg, Qg, seeds, k=10, L=12, B=64, metric=1, team=16, stop_eps=0.05)
    if ref is None:
        pytest.skip("reference kernels not built")
    theirs = _recall(ref[0].cpu().numpy(), truth, 10)
    assert abs(mine - theirs) <= 0.005, (mine, theirs)


@pytest.mark.parametrize("stall,crowd,V,policy", [
    (1, 0.0, 1, 0), (3, 0.0, 1, 0), (2, 0.0, 4, 1),
    (0, 0.3, 1, 0), (0, 0.4, 1, 0), (0, 0.3, 4, 0), (0, 0.5, 4, 1), (2, 0.4, 3, 1),
])
def test_stall_and_crowd_rules_bitwise(stall, crowd, V, policy):
    """The stall rule (stop once the k-th best has not improved for `stall`
    steps) and the crowd rule (retire a lineage after two expansions whose
    neighbours were mostly covered already) of local_search.cu:659-682: queues,
    distances, flags, lineage and every counter -- stalled and crowded included
    -- equal the oracle and the reference's own kernels bit for bit, through
    advance and through the fused kernel."""
    X, G = cases.toy(seed=211)
    rng = np.random.default_rng(stall * 10 + V)
    nq, J, L, B = 8, 3, 16, 40
    Qv = cases.unit_queries(nq, X.shape[1], 5 + V)
    seeds = rng.integers(0, X.shape[0], (nq, J, V)).astype(np.int32)
    Xg, Gg, Qg = to_gpu(X, G, Qv)
    kw = dict(L=L, B=B, D=G.shape[1], team_size=16, policy=policy, stop_eps=-1.0, kstop=10,
              stall_patience=stall, crowd_frac=crowd)
    st = E.init_states(Xg, Qg, torch.from_numpy(seeds), **kw)
    E.advance(Xg, Gg, Qg, st, B)
    st.check()
    if stall:
        assert int(st.stalled.sum()) > 0, "the stall rule never fired: the case tests nothing"
    if crowd:
        assert int(st.crowded.sum()) > 0, "the crowd rule never fired: the case tests nothing"
    gi, gd = st.ids.cpu().numpy(), st.dist.cpu().numpy()
    ge, gl, gc = st.expanded.cpu().numpy(), st.lineage.cpu().numpy(), st.counters.cpu().numpy()
    for q in range(nq):
        for j in range(J):
            r = O.branch_run(X, G, Qv[q], seeds[q, j], L=L, B=B, team=16, policy=policy, stall_patience=stall,
                             crowd_frac=crowd)
            tag = f"q={q} j={j}"
            assert np.array_equal(r["ids"], gi[q, j]), tag
            assert np.array_equal(r["dist"].view(np.int32), gd[q, j].view(np.int32)), tag
            assert np.array_equal(r["expanded"], ge[q, j]), tag
            assert np.array_equal(r["lineage"], gl[q, j]), tag
            for c in (0, 1, 3, 6, 7, 8, 9):
                assert r["counters"][c] == gc[q, j, c], f"{tag} counter {c}"
    ref = ref_run(Xg, Gg, Qg, torch.from_numpy(seeds), L, B, 0, 16, policy=policy, stall=stall, crowd=crowd)
    if ref is not None:
        same_state(st, ref, counters=(0, 1, 2, 3, 6, 7, 8, 9))
    # the fused kernel runs the same walk in one launch
    fi, fd, fst = E.search(Xg, Gg, Qg, torch.from_numpy(seeds), k=10, L=L, B=B, team_size=16, policy=policy,
                           stall_patience=stall, crowd_frac=crowd)
    assert torch.equal(fst.ids, st.ids) and torch.equal(fst.counters, st.counters)
