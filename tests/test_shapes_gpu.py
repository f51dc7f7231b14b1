"""Parity at the production shapes.

The headline configurations score 960-wide fp32 rows (L2) and 1536-wide fp16
rows (inner product), and the north star asks for rows up to 4096 wide.  At
those widths every lane of a team sums many 16-byte chunks (12 at d = 1536
fp16 with team 16), the fused kernel scores two rows per team at once and
keeps an fp16 corpus's query as two planes (eight rows a team in its
small-batch form) -- none of which the toy width (64) exercises.  Here the fused kernel (the one Index.search launches) is held bit
for bit against the C oracle and the reference's own compiled kernels at those
widths and the production knobs, and the production mode's recall on a
C3-shaped corpus is held to the reference kernel's.
"""
import numpy as np
import pytest
import torch

import cases
from oracle import oracle as O
from refcheck import DEV, recall, ref_production, ref_run, same_state, to_gpu
from swann_b200 import _engine as E
from swann_b200 import _select as S

pytestmark = pytest.mark.gpu

SHAPES = [
    # d, fp16 rows, metric, team
    (960, False, E.METRIC_L2, 16),
    (960, False, E.METRIC_L2, 32),
    (1536, True, E.METRIC_IP, 16),
    (1536, True, E.METRIC_IP, 32),
    (4096, True, E.METRIC_IP, 16),
    (4096, False, E.METRIC_L2, 32),
]
_CORPORA = {}


def corpus(d, half, metric):
    """3000 rows, their exact 64-nearest graph; rows stored fp16 when asked."""
    key = (d, half, metric)
    if key not in _CORPORA:
        X, G = cases.toy(n=3000, d=d, deg=64, seed=d + metric, metric=metric)
        if half:
            X = X.astype(np.float16)
        _CORPORA[key] = (X, G)
    return _CORPORA[key]


def queries(nq, d, metric, seed):
    if metric == E.METRIC_IP:
        return cases.unit_queries(nq, d, seed)
    return np.random.default_rng(seed).standard_normal((nq, d), dtype=np.float32)


@pytest.mark.parametrize("form", ["helped", "wide", "narrow"])
@pytest.mark.parametrize("d,half,metric,team", SHAPES)
@pytest.mark.parametrize("L,B,eps", [(12, 64, 0.01), (32, 12, -1.0)])
def test_fused_walk_bitwise_at_production_widths(d, half, metric, team, L, B, eps, form, monkeypatch):
    """Per-branch queues, distances, flags and counters of the fused kernel
    equal the oracle's single-branch walk (swann/_refcpu.py's semantics) and
    the reference kernels' init_states + advance, bit for bit; the merged
    answers equal the oracle's.  Every form of the kernel: the helped one the
    smallest batches get (one branch a CTA, its other warps scoring with it),
    the wide one small batches get (eight rows a team in flight) and the one
    large batches get (two), chosen here through SWB_HELP_CTAS / SWB_WIDE_CTAS."""
    monkeypatch.setenv("SWB_HELP_CTAS", "1000000" if form == "helped" else "0")
    monkeypatch.setenv("SWB_WIDE_CTAS", "1000000" if form == "wide" else "0")
    X, G = corpus(d, half, metric)
    nq, J = 6, 4
    Qv = queries(nq, d, metric, 31 + d)
    seeds = np.random.default_rng(d + L).integers(0, X.shape[0], (nq, J)).astype(np.int32)
    Xg, Gg, Qg = to_gpu(X, G, Qv)
    ids, dist, st = E.search(Xg, Gg, Qg, torch.from_numpy(seeds), k=10, L=L, B=B, metric=metric, team_size=team,
                             stop_eps=eps)
    st.check()
    gi, gd, ge, gc = (t.cpu().numpy() for t in (st.ids, st.dist, st.expanded, st.counters))
    for q in range(nq):
        for j in range(J):
            r = O.branch_run(X, G, Qv[q], seeds[q, j], L=L, B=B, metric=metric, team=team, stop_eps=eps,
                             kstop=10)
            tag = f"d={d} team={team} q={q} j={j}"
            assert np.array_equal(r["ids"], gi[q, j]), tag
            assert np.array_equal(r["dist"].view(np.int32), gd[q, j].view(np.int32)), tag
            assert np.array_equal(r["expanded"], ge[q, j]), tag
            assert r["counters"][0] == gc[q, j, 0] and r["counters"][1] == gc[q, j, 1], tag
    oi, od = O.search(X, G, Qv, seeds, k=10, L=L, B=B, metric=metric, team=team, stop_eps=eps, kstop=10)
    assert np.array_equal(ids.cpu().numpy(), oi)
    assert np.array_equal(dist.cpu().numpy().view(np.int32), od.view(np.int32))
    ref = ref_run(Xg, Gg, Qg, torch.from_numpy(seeds), L, B, metric, team, stop_eps=eps, kstop=10)
    if ref is not None:
        same_state(st, ref)


@pytest.mark.parametrize("d,half,metric,team", [SHAPES[1], SHAPES[2], SHAPES[4]])
def test_shared_table_changes_work_not_results_at_production_widths(d, half, metric, team):
    """The per-query table (no claims, no bound) only saves distance
    evaluations: the answers and queues equal the independent branches'."""
    X, G = corpus(d, half, metric)
    Qv = queries(8, d, metric, 7)
    seeds = torch.from_numpy(np.random.default_rng(3).integers(0, X.shape[0], (8, 16)).astype(np.int32))
    Xg, Gg, Qg = to_gpu(X, G, Qv)
    kw = dict(k=10, L=12, B=64, metric=metric, team_size=team, stop_eps=0.01)
    plain = E.search(Xg, Gg, Qg, seeds, **kw)
    cached = E.search(Xg, Gg, Qg, seeds, shared_cache=True, **kw)
    assert torch.equal(plain[0], cached[0]) and torch.equal(plain[1], cached[1])
    assert torch.equal(plain[2].ids, cached[2].ids)
    assert int(cached[2].cache_hits.sum()) > 0


def _exact_ip_dist(Q, X, ids):
    ok = ids >= 0
    x = X[np.maximum(ids, 0)].astype(np.float64)
    ex = 1.0 - (Q[:, None, :].astype(np.float64) * x).sum(-1)
    return ex, ok


def test_c3_shaped_recall_matches_reference_kernel():
    """BASELINE config 3's model (anisotropic clusters, unit rows stored fp16,
    inner product, d = 1536) at 20k rows: Index.search -- strict claims and a
    per-query table sized from the claims it measured -- reaches a recall@10
    within 0.005 of the reference kernels' production path (exclusive claims,
    the reference's table sizing) on the same graph and seeds, and every
    distance it returns equals an exact recomputation within 1e-5 relative."""
    import swann_b200 as swann
    from swann_b200 import build as Bd
    n, d, nq = 20000, 1536, 4096
    X, Q = cases.aniso_mixture(n, d, clusters=100, seed=5, nq=nq)
    Xh = X.astype(np.float16)
    Xg = torch.from_numpy(Xh).to(DEV)
    Qg = torch.from_numpy(Q).to(DEV)
    G = Bd.build_graph(Xg, metric="ip", degree=64, candidates=128, alpha=1.2)
    cat = torch.from_numpy(cases.catalogue(n)).to(DEV)
    index = swann.Index(Xg, G, metric="ip", catalogue=cat)
    op = dict(k=10, branches=32, queue=12, budget=64, stop_eps=0.01, team=16)
    index.search(Q, **op)                       # first call: the reference's table size
    ids, dist = index.search(Q, **op)           # then: sized from the claims measured
    slots = index.table_slots_for(32, 64, 12, 0.01, G.shape[1])
    assert slots < E.cache_size(32, 64, G.shape[1]), "the table was not sized from measured claims"
    with torch.no_grad():
        truth = torch.topk(Qg @ Xg.float().T, 10, dim=1).indices.cpu().numpy()
    mine = recall(ids, truth, 10)
    ex, ok = _exact_ip_dist(Q, Xh, ids)
    rel = np.abs(dist.astype(np.float64) - ex) / np.maximum(np.abs(ex), 1e-30)
    assert ok.all() and rel.max() <= 1e-5, rel.max()
    assert mine >= 0.9, mine
    ent = S.select_nearest(Qg, S.pool_vectors(Xg, cat).float(), 32, metric=0)
    ref = ref_production(Xg, G, Qg, cat[ent].to(torch.int32), k=10, L=12, B=64, metric=0, team=16, stop_eps=0.01)
    if ref is None:
        pytest.skip("reference kernels not built")
    theirs = recall(ref[0].cpu().numpy(), truth, 10)
    assert abs(mine - theirs) <= 0.005, (mine, theirs)


@pytest.mark.parametrize("half,metric", [(True, "ip"), (False, "l2")])
def test_index_search_at_width_4096(half, metric):
    """Index.search at d = 4096 (the widest row the north star names): the
    query and queues fit on chip, and every answer carries its exact
    distance."""
    import swann_b200 as swann
    m = E.METRIC_IP if metric == "ip" else E.METRIC_L2
    X, G = corpus(4096, half, m)
    Q = queries(64, 4096, m, 99)
    Xg, Gg = torch.from_numpy(X).to(DEV), torch.from_numpy(G).to(DEV)
    index = swann.Index(Xg, Gg, metric=metric, catalogue_size=1024)
    ids, dist = index.search(Q, k=10, branches=16, stop_eps=0.05)
    assert (ids >= 0).all()
    x = X.astype(np.float64)[ids]
    if m == E.METRIC_IP:
        ex = 1.0 - (Q[:, None, :].astype(np.float64) * x).sum(-1)
    else:
        ex = ((Q[:, None, :].astype(np.float64) - x) ** 2).sum(-1)
    assert np.allclose(dist, ex, rtol=1e-5, atol=1e-6)
