"""The sign-code prefilter in advance (swann/csrc/local_search.cu:205-243,
560-572; swann/_engine.py:281-337): a neighbour whose 1-bit estimate lies past
the expansion limit by more than the margin is never read.

The reference's code writer is missing, so the codes here come from
swann_b200.corpus.build_codes; parity with the reference's skip decisions is
not pinned (its query sums are float atomics).  What is checked: an infinite
margin changes nothing, bit for bit; a finite one skips rows, keeps every
distance exact and keeps the answers close."""
import numpy as np
import pytest
import torch

import cases
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
