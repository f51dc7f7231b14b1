"""The drop-in boundary at the reference's own argument lists.

swann_b200.refext has the three entry points the reference's Python calls
through ext() (swann/csrc/local_search.cu:741-955).  Here both it and the
reference's own compiled kernels (oracle/_ref) are called with identical
arguments -- the same tensors' copies, the same knobs -- and every output is
compared: queues, distances, flags, lineage and counters bit for bit, the
per-query table (cache_id / cache_d) as the set of (node, distance) entries it
holds (which slot a node lands in depends on the order concurrent inserts
arrive in, in both implementations), the visited tables as sets, and the
merge's results.  Finally the reference's own swann/_engine.py is run with its
extension slot filled by this module.
"""
import numpy as np
import pytest
import torch

import cases
from oracle import oracle as O
from refcheck import DEV, to_gpu
from swann_b200 import _engine as E
from swann_b200 import refext

pytestmark = pytest.mark.gpu


def _ref():
    R = O.ref_kernels()
    if R is None:
        pytest.skip("reference kernels not built")
    return R


def _state(Q, J, L, H, Hc, bound):
    st = dict(ids=torch.empty((Q, J, L), dtype=torch.int32, device=DEV),
              dist=torch.empty((Q, J, L), dtype=torch.float32, device=DEV),
              expd=torch.empty((Q, J, L), dtype=torch.uint8, device=DEV),
              lin=torch.empty((Q, J, L), dtype=torch.uint8, device=DEV),
              vis=torch.empty((Q, J, H), dtype=torch.int32, device=DEV),
              ctr=torch.empty((Q, J, 10), dtype=torch.int32, device=DEV))
    st["cid"] = torch.empty((Q, Hc) if Hc else (0, 0), dtype=torch.int32, device=DEV)
    st["cdd"] = torch.empty((Q, Hc) if Hc else (0, 0), dtype=torch.float32, device=DEV)
    st["bnd"] = torch.empty((Q,) if bound else (0,), dtype=torch.float32, device=DEV)
    return st


def _run(mod, Xg, Gg, Qg, seeds, L, B, H, Hc, bound, metric, team, policy, eps, kstop, exclusive, stall, crowd,
         splits):
    Q, J, V = seeds.shape
    st = _state(Q, J, L, H, Hc, bound)
    mod.init_states(Xg, Qg, seeds, st["ids"], st["dist"], st["expd"], st["lin"], st["vis"], st["ctr"], metric, team,
                    st["cid"], st["cdd"], st["bnd"])
    e0 = torch.empty(0, dtype=torch.int32, device=DEV)
    e0f = torch.empty(0, dtype=torch.float32, device=DEV)
    for delta in splits:
        mod.advance(Xg, Gg, Qg, st["ids"], st["dist"], st["expd"], st["lin"], st["vis"], st["ctr"], metric, team,
                    delta, B, policy, V, eps, kstop, st["cid"], st["cdd"], st["bnd"], exclusive, stall, crowd, e0,
                    e0, e0f, e0f, 0.0)
    torch.cuda.synchronize()
    return st


def _entries(cid, cdd):
    """The table as {node: distance bits} per query."""
    out = []
    ci, cd = cid.cpu().numpy(), cdd.cpu().numpy().view(np.int32)
    for q in range(ci.shape[0]):
        m = ci[q] != 0
        out.append(dict(zip((ci[q][m] - 1).tolist(), cd[q][m].tolist())))
    return out


def _visited_sets(vis):
    v = vis.cpu().numpy()
    return [[frozenset(row[row != 0].tolist()) for row in per_q] for per_q in v]


@pytest.mark.parametrize("metric,team,V,policy,eps,stall,crowd,splits", [
    (0, 16, 1, 0, 0.05, 0, 0.0, (24,)),
    (1, 32, 4, 1, 0.1, 0, 0.0, (5, 19)),
    (0, 8, 3, 1, -1.0, 2, 0.4, (24,)),
    (1, 16, 1, 0, -1.0, 0, 0.3, (7, 7, 10)),
])
def test_branch_states_equal_reference_kernels(metric, team, V, policy, eps, stall, crowd, splits):
    """Independent branches (no shared state): every output equal, including
    across resumed advance calls."""
    R = _ref()
    X, G = cases.toy(seed=300 + metric, metric=metric)
    Qv = cases.unit_queries(6, X.shape[1], 9) if metric == 0 else \
        np.random.default_rng(9).standard_normal((6, X.shape[1]), dtype=np.float32)
    seeds = torch.from_numpy(np.random.default_rng(V).integers(0, X.shape[0], (6, 3, V)).astype(np.int32)).to(DEV)
    Xg, Gg, Qg = to_gpu(X, G, Qv)
    B, L, H = 24, 16, E.visited_size(24, G.shape[1])
    args = (Xg, Gg, Qg, seeds, L, B, H, 0, False, metric, team, policy, eps, 10, 0, stall, crowd, splits)
    mine, theirs = _run(refext, *args), _run(R, *args)
    for key in ("ids", "expd", "lin", "ctr"):
        assert torch.equal(mine[key], theirs[key]), key
    assert torch.equal(mine["dist"].view(torch.int32), theirs["dist"].view(torch.int32))
    assert _visited_sets(mine["vis"]) == _visited_sets(theirs["vis"])


@pytest.mark.parametrize("fp16", [False, True])
def test_shared_table_round_trips_through_the_reference_layout(fp16):
    """A per-query table shared by 6 branches, no claims and no bound (so the
    walk is deterministic): queues bit for bit, the table holds the same
    (node, distance) entries as the reference kernels' cache_id / cache_d --
    also when carried between advance calls -- and each branch's evaluations
    plus table hits match."""
    R = _ref()
    X, G = cases.toy(seed=77)
    Xs = X.astype(np.float16) if fp16 else X
    Qv = cases.unit_queries(5, X.shape[1], 4)
    seeds = torch.from_numpy(np.random.default_rng(5).integers(0, X.shape[0], (5, 6, 1)).astype(np.int32)).to(DEV)
    Xg, Gg, Qg = to_gpu(Xs, G, Qv)
    B, L = 16, 16
    Hc = E.cache_size(6, B, G.shape[1])
    args = (Xg, Gg, Qg, seeds, L, B, E.visited_size(B, G.shape[1]), Hc, False, 0, 16, 0, -1.0, 10, 0, 0, 0.0,
            (6, 10))
    mine, theirs = _run(refext, *args), _run(R, *args)
    for key in ("ids", "expd", "lin"):
        assert torch.equal(mine[key], theirs[key]), key
    assert torch.equal(mine["dist"].view(torch.int32), theirs["dist"].view(torch.int32))
    for c in (0, 3, 8, 9):
        assert torch.equal(mine["ctr"][..., c], theirs["ctr"][..., c]), c
    # which branch scores a node first is a race in both implementations, so
    # evaluations and hits split differently between branches; every fresh
    # neighbour is one or the other, so their sum per branch is fixed
    both = lambda st: st["ctr"][..., 1] + st["ctr"][..., 4]  # noqa: E731
    assert torch.equal(both(mine), both(theirs))
    assert _entries(mine["cid"], mine["cdd"]) == _entries(theirs["cid"], theirs["cdd"])
    # every slot the reference leaves empty reads (0, FLT_MAX) here too
    empty = mine["cid"] == 0
    assert bool((mine["cdd"][empty] == torch.finfo(torch.float32).max).all())


def test_merge_equals_reference():
    R = _ref()
    ids, dist = cases.merge_inputs(Q=33, J=7, kk=10, seed=12)
    a = refext.merge_branches(torch.from_numpy(ids).to(DEV), torch.from_numpy(dist).to(DEV), 10)
    b = R.merge_branches(torch.from_numpy(ids).to(DEV), torch.from_numpy(dist).to(DEV), 10)
    assert isinstance(a, list) and len(a) == 2
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_argument_errors_are_runtime_errors():
    """The reference's TORCH_CHECKs surface as RuntimeError; so do these."""
    X, G = cases.toy(n=200, d=16, deg=8, seed=1)
    Xg, Gg, Qg = to_gpu(X, G, cases.unit_queries(2, 16, 1))
    st = _state(2, 1, 8, 3, 0, False)      # H = 3: not a power of two
    seeds = torch.zeros((2, 1, 1), dtype=torch.int32, device=DEV)
    with pytest.raises(RuntimeError, match="power of two"):
        refext.init_states(Xg, Qg, seeds, st["ids"], st["dist"], st["expd"], st["lin"], st["vis"], st["ctr"], 0, 16,
                           st["cid"], st["cdd"], st["bnd"])
    st = _state(2, 1, 8, 4, 0, False)
    with pytest.raises(RuntimeError, match="team"):
        refext.init_states(Xg, Qg, seeds, st["ids"], st["dist"], st["expd"], st["lin"], st["vis"], st["ctr"], 0, 12,
                           st["cid"], st["cdd"], st["bnd"])


def test_reference_engine_runs_on_this_module():
    """The reference's own swann/_engine.py (installed under baseline/_ref),
    unmodified, with its extension slot filled by this module: its search()
    returns what it returns on its own kernels (independent branches)."""
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent / "baseline" / "_ref"
    if not (root / "swann" / "_engine.py").exists():
        pytest.skip("reference package not installed under baseline/_ref")
    R = _ref()
    sys.path.insert(0, str(root))
    try:
        import swann._engine as RE
    finally:
        sys.path.remove(str(root))
    X, G = cases.toy(seed=19)
    Qv = cases.unit_queries(7, X.shape[1], 19)
    seeds = torch.from_numpy(np.random.default_rng(2).integers(0, X.shape[0], (7, 4)).astype(np.int32))
    Xg, Gg, Qg = to_gpu(X, G, Qv)
    saved = RE._EXT
    try:
        RE._EXT = refext
        a_ids, a_dist, a_st = RE.search(Xg, Gg, Qg, seeds, k=10, L=16, B=20, stop_eps=0.05)
        RE._EXT = R
        b_ids, b_dist, b_st = RE.search(Xg, Gg, Qg, seeds, k=10, L=16, B=20, stop_eps=0.05)
    finally:
        RE._EXT = saved
    assert torch.equal(a_ids, b_ids) and torch.equal(a_dist, b_dist)
    assert torch.equal(a_st.ids, b_st.ids) and torch.equal(a_st.counters, b_st.counters)
