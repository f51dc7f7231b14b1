"""Entry selection (select_nearest -> swb_select_topk) against the reference's
own procedure on the same scores: the catalogue scored slice by slice and
torch.topk(largest=False) folded over the slices (swann/_select.py:93-130),
run on the CPU from the GPU's score matrix."""
import numpy as np
import pytest
import torch

from swann_b200 import _engine as E
from swann_b200 import _select as S

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _reference(Qg, Vp, Ek, metric, slice_P):
    """swann/_select.py:select_nearest, evaluated on the CPU from the same
    slice scores the GPU path computes; also returns those scores [n, P]."""
    n, P = Qg.shape[0], Vp.shape[0]
    bi = torch.empty(n, 0, dtype=torch.long)
    bv = torch.empty(n, 0)
    allc = []
    qn = (Qg * Qg).sum(1).view(-1, 1).cpu() if metric != E.METRIC_IP else None
    for s in range(0, P, slice_P):
        V = Vp[s:s + slice_P]
        with S.reduced_precision(True):
            sc = (Qg @ V.T).cpu()
        c = (1.0 - sc) if metric == E.METRIC_IP else ((V * V).sum(1).view(1, -1).cpu() - 2.0 * sc + qn)
        allc.append(c)
        v, i = torch.topk(c, min(Ek, c.shape[1]), dim=1, largest=False)
        bv = torch.cat([bv, v], 1)
        bi = torch.cat([bi, i + s], 1)
        if bv.shape[1] > Ek:
            v, j = torch.topk(bv, Ek, dim=1, largest=False)
            bv, bi = v, torch.gather(bi, 1, j)
    return bi, bv, torch.cat(allc, 1)


def _check(got, want_i, want_v, c):
    """Same entries per query and the same distance at every position: the
    order of exactly equal distances is the one thing torch.topk leaves open
    (this path takes the lower index first)."""
    assert got.shape == want_i.shape
    assert torch.equal(torch.gather(c, 1, got), want_v)
    assert torch.equal(got.sort(1).values, want_i.sort(1).values)
    ties = (got != want_i).any(1)
    assert int(ties.sum()) <= max(2, got.shape[0] // 100)


@pytest.mark.parametrize("metric", [E.METRIC_IP, E.METRIC_L2])
@pytest.mark.parametrize("Ek,P,slice_P", [(32, 4096, 8192), (32, 4096, 1000), (48, 3000, 8192), (128, 2500, 700),
                                          (40, 24, 8192), (5, 999, 8192)])
def test_select_matches_reference_topk(metric, Ek, P, slice_P):
    g = torch.Generator(device="cpu").manual_seed(7 + Ek + P)
    n, d = 777, 96
    Q = torch.randn((n, d), generator=g)
    V = torch.randn((P, d), generator=g)
    if metric == E.METRIC_IP:
        Q = Q / Q.norm(dim=1, keepdim=True)
        V = V / V.norm(dim=1, keepdim=True)
    Qg, Vg = Q.to(DEV), V.to(DEV)
    got = S.select_nearest(Qg, Vg, Ek, metric=metric, slice_P=slice_P)
    want_i, want_v, c = _reference(Qg, Vg, Ek, metric, slice_P)
    _check(got.cpu(), want_i, want_v, c)


def test_select_matches_on_index_catalogue():
    """The production call: queries against an Index's catalogue rows."""
    import cases
    X, G = cases.toy(n=6000, d=64, deg=32, seed=3, metric=0)
    import swann_b200 as swann
    idx = swann.Index(torch.from_numpy(X).to(DEV), torch.from_numpy(G).to(DEV), metric="ip", catalogue_size=2048)
    rng = np.random.default_rng(1)
    Q = rng.standard_normal((300, 64)).astype(np.float32)
    Q /= np.linalg.norm(Q, axis=1, keepdims=True)
    Qg = torch.from_numpy(Q).to(DEV)
    got = S.select_nearest(Qg, idx._cat, 32, metric=0).cpu()
    want_i, want_v, c = _reference(Qg, idx._cat, 32, 0, 8192)
    _check(got, want_i, want_v, c)
