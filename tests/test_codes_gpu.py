"""The sign-code prefilter in advance (swann/csrc/local_search.cu:205-243,
560-572; swann/_engine.py:281-337): a neighbour whose 1-bit estimate lies past
the expansion limit by more than the margin is never read.

The reference's code writer is missing, so the codes here come from
swann_b200.corpus.build_codes.  What is checked: an infinite margin changes
nothing, bit for bit; a finite one skips rows, keeps every distance exact and
keeps the answers close; and, given the same code files, the advance equals
the reference's own kernels (oracle/_ref) branch for branch -- up to the last
bit of the query's two sums, which the reference adds with float atomics in
whatever order they land, so a skip decision within a rounding of its
threshold may go either way."""
import numpy as np
import pytest
import torch

import cases
from oracle import oracle as O
from swann_b200 import _engine as E
from swann_b200 import corpus as C

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _setup(seed=5, n=3000, d=96, deg=32, nq=40, J=4):
    X, G = cases.toy(n=n, d=d, deg=deg, seed=seed, metric=0)
    rng = np.random.default_rng(seed)
    Q = rng.standard_normal((nq, d)).astype(np.float32)
    Q /= np.linalg.norm(Q, axis=1, keepdims=True)
    seeds = rng.integers(0, n, (nq, J)).astype(np.int32)
    Xg, Gg, Qg = (torch.from_numpy(np.ascontiguousarray(a)).to(DEV) for a in (X, G, Q))
    return X, Q, Xg, Gg, Qg, torch.from_numpy(seeds).to(DEV), C.build_codes(Xg)


def _run(Xg, Gg, Qg, seeds, codes=None, metric=0):
    st = E.init_states(Xg, Qg, seeds, L=16, B=40, D=Gg.shape[1], metric=metric, team_size=16, stop_eps=0.05,
                       kstop=10)
    E.advance(Xg, Gg, Qg, st, 40, codes=codes)
    torch.cuda.synchronize()
    return st


def _top10(st):
    ids, dist = E.merge_branches(*E.branch_topk(st, 10), 10)
    return ids.cpu().numpy()


def test_infinite_margin_changes_nothing():
    X, Q, Xg, Gg, Qg, seeds, (cd, al, mu) = _setup()
    base = _run(Xg, Gg, Qg, seeds)
    coded = _run(Xg, Gg, Qg, seeds, codes=(cd, al, mu, float("inf")))
    for name in ("ids", "dist", "expanded", "lineage", "counters"):
        assert torch.equal(getattr(base, name), getattr(coded, name)), name


def test_margin_skips_rows_and_keeps_distances_exact():
    X, Q, Xg, Gg, Qg, seeds, (cd, al, mu) = _setup()
    base = _run(Xg, Gg, Qg, seeds)
    tight = _run(Xg, Gg, Qg, seeds, codes=(cd, al, mu, 0.05))
    scored_base = int(base.counters[..., 1].sum())
    scored_tight = int(tight.counters[..., 1].sum())
    assert 0 < scored_tight < scored_base
    ids, dist = tight.ids.cpu().numpy(), tight.dist.cpu().numpy()
    ok = ids >= 0
    exact = 1.0 - np.einsum("qjld,qd->qjl", X[np.where(ok, ids, 0)].astype(np.float64), Q.astype(np.float64))
    assert np.allclose(dist[ok], exact[ok], atol=1e-5)
    truth = np.argsort(-(Q @ X.T), axis=1)[:, :10]
    rec = lambda got: np.mean([len(set(a) & set(b)) / 10 for a, b in zip(got, truth)])
    assert rec(_top10(tight)) >= rec(_top10(base)) - 0.05


def test_codes_are_inner_product_only():
    X, Q, Xg, Gg, Qg, seeds, (cd, al, mu) = _setup()
    with pytest.raises(NotImplementedError):
        _run(Xg, Gg, Qg, seeds, codes=(cd, al, mu, 0.1), metric=1)


def test_codes_of_the_wrong_shape_are_refused():
    X, Q, Xg, Gg, Qg, seeds, (cd, al, mu) = _setup()
    with pytest.raises(ValueError):
        _run(Xg, Gg, Qg, seeds, codes=(cd[:, :1], al, mu, 0.1))


@pytest.mark.parametrize("margin,eps", [(0.05, 0.05), (0.15, 0.1), (0.0, 0.0)])
def test_skips_match_the_reference_kernels(margin, eps):
    """Same corpus, graph, seeds and code files through this advance and the
    reference's (local_search.cu:205-243,560-585): queues, distances, flags,
    lineage and counters equal branch for branch, except counter 3, where the
    reference also counts skips (which advance_chunked would read as
    'exhausted'); a branch may differ only where a skip decision sat within
    the rounding of the reference's atomically summed query terms."""
    R = O.ref_kernels()
    if R is None:
        pytest.skip("reference kernels not built")
    X, Q, Xg, Gg, Qg, seeds, (cd, al, mu) = _setup(seed=9, nq=64)
    L, B = 16, 40
    st = E.init_states(Xg, Qg, seeds, L=L, B=B, D=Gg.shape[1], metric=0, team_size=16, stop_eps=eps, kstop=10)
    E.advance(Xg, Gg, Qg, st, B, codes=(cd, al, mu, margin))
    s3 = seeds.unsqueeze(-1).contiguous()
    Qn, J = seeds.shape
    H = E.visited_size(B, Gg.shape[1])
    ids = torch.empty((Qn, J, L), dtype=torch.int32, device=DEV)
    dist = torch.empty((Qn, J, L), dtype=torch.float32, device=DEV)
    expd = torch.empty((Qn, J, L), dtype=torch.uint8, device=DEV)
    lin = torch.empty((Qn, J, L), dtype=torch.uint8, device=DEV)
    vis = torch.empty((Qn, J, H), dtype=torch.int32, device=DEV)
    ctr = torch.empty((Qn, J, 10), dtype=torch.int32, device=DEV)
    ei = torch.empty((0, 0), dtype=torch.int32, device=DEV)
    ef = torch.empty((0, 0), dtype=torch.float32, device=DEV)
    eb = torch.empty((0,), dtype=torch.float32, device=DEV)
    R.init_states(Xg, Qg, s3, ids, dist, expd, lin, vis, ctr, 0, 16, ei, ef, eb)
    e0 = torch.empty(0, dtype=torch.int32, device=DEV)
    R.advance(Xg, Gg, Qg, ids, dist, expd, lin, vis, ctr, 0, 16, B, B, 0, 1, float(eps), 10, ei, ef, eb, 0, 0, 0.0,
              e0, cd, al, mu, float(margin))
    torch.cuda.synchronize()
    plain = _run_plain(Xg, Gg, Qg, seeds, L, B, eps)
    evals = (int(plain.dist_evals.sum()), int(st.dist_evals.sum()), int(ctr[..., 1].sum()))
    assert evals[1] < evals[0] and evals[2] < evals[0], f"no row was skipped: the case tests nothing {evals}"
    keep = [c for c in range(10) if c != 3]
    same = ((st.ids == ids).all(-1) & (st.dist.view(torch.int32) == dist.view(torch.int32)).all(-1)
            & (st.expanded == expd).all(-1) & (st.lineage == lin).all(-1)
            & (st.counters[..., keep] == ctr[..., keep]).all(-1))
    bad = int((~same).sum())
    detail = {"evals plain/mine/ref": evals, "ids": int((st.ids != ids).any(-1).sum()),
              "dist": int((st.dist.view(torch.int32) != dist.view(torch.int32)).any(-1).sum()),
              "counters": [int((st.counters[..., c] != ctr[..., c]).sum()) for c in range(10)]}
    assert bad <= max(1, same.numel() // 50), f"{bad} of {same.numel()} branches differ: {detail}"


def _run_plain(Xg, Gg, Qg, seeds, L, B, eps):
    st = E.init_states(Xg, Qg, seeds, L=L, B=B, D=Gg.shape[1], metric=0, team_size=16, stop_eps=eps, kstop=10)
    E.advance(Xg, Gg, Qg, st, B)
    torch.cuda.synchronize()
    return st
