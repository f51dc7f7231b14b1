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


def _topk_direct(sc, Ek, metric, vn=None, qn=None, slices=1):
    """swb_select_topk over the score matrix `sc` [n, P] in `slices` column
    slices (the later ones resuming the running list)."""
    from swann_b200 import _lib as N
    n, P = sc.shape
    bd = torch.empty((n, Ek), dtype=torch.float32, device=DEV)
    bi = torch.empty((n, Ek), dtype=torch.int64, device=DEV)
    bounds = np.linspace(0, P, slices + 1).astype(int)
    for k, (a, b) in enumerate(zip(bounds[:-1], bounds[1:])):
        part = sc[:, a:b].contiguous()
        v = vn[a:b].contiguous() if vn is not None else None
        rc = N.lib().swb_select_topk(N.ptr(part), n, b - a, part.stride(0), N.ptr(v), N.ptr(qn), int(metric), Ek,
                                     int(a), N.ptr(bd), N.ptr(bi), int(k > 0), N.stream_of(part))
        N.check(rc, "swb_select_topk")
    torch.cuda.synchronize()
    return bd.cpu(), bi.cpu()


def _exact(sc, Ek, metric, vn=None, qn=None):
    """The Ek smallest (distance, column) keys per row, computed on the CPU in
    float32 with the same expressions; equal distances go to the lower column."""
    sc = sc.cpu()
    if metric == E.METRIC_IP:
        d = 1.0 - sc
    else:
        d = (vn.cpu().view(1, -1) - 2.0 * sc) + qn.cpu().view(-1, 1)
    cols = torch.arange(sc.shape[1]).expand_as(d)
    # a stable sort by distance keeps equal distances in column order
    order = torch.sort(d, dim=1, stable=True).indices
    k = min(Ek, sc.shape[1])
    return torch.gather(d, 1, order[:, :k]), torch.gather(cols, 1, order[:, :k])


def _layout(kind, n, P, g):
    """Score matrices built to stress the selection: `lane` puts every row's
    best scores in the columns one lane of the warp reads (4 of every 128),
    `trend` makes each row's scores rise (distances fall) along the row, `ties`
    draws from a handful of values, `random` is plain Gaussian."""
    if kind == "random":
        return torch.randn((n, P), generator=g)
    if kind == "trend":
        return torch.linspace(-1, 1, P).view(1, -1) + 1e-3 * torch.randn((n, P), generator=g)
    if kind == "ties":
        return torch.randint(0, 6, (n, P), generator=g).float() / 8
    sc = torch.randn((n, P), generator=g) - 4.0
    cols = torch.arange(P)
    owner = (cols % 128) // 4                     # the lane that reads each column
    lane = torch.randint(0, 32, (n, 1), generator=g)
    return torch.where(owner.view(1, -1) == lane, sc + 8.0, sc)


@pytest.mark.parametrize("kind", ["lane", "trend", "ties", "random"])
@pytest.mark.parametrize("metric", [E.METRIC_IP, E.METRIC_L2])
@pytest.mark.parametrize("Ek,P,slices", [(32, 4096, 1), (32, 4096, 3), (5, 1000, 1), (64, 2500, 2), (128, 4096, 1),
                                          (48, 37, 1), (128, 300, 2)])
def test_select_topk_exact_on_stressed_scores(kind, metric, Ek, P, slices):
    """swb_select_topk equals the exact (distance, column) order bit for bit on
    rows built against its filter-and-merge: best entries all in one lane's
    columns, distances falling along the row (nearly every column survives the
    filter, so the list is merged once per 32 columns), and heavy ties (the
    lower column first), over one slice or several resumed ones."""
    g = torch.Generator(device="cpu").manual_seed(11 + Ek + P + slices)
    n = 300
    sc = _layout(kind, n, P, g)
    vn = qn = None
    if metric == E.METRIC_L2:
        vn = torch.rand((P,), generator=g) * 4
        qn = torch.rand((n,), generator=g) * 4
        vn, qn = vn.to(DEV), qn.to(DEV)
    bd, bi = _topk_direct(sc.to(DEV), Ek, metric, vn, qn, slices)
    want_d, want_i = _exact(sc, Ek, metric, vn, qn)
    k = want_i.shape[1]
    assert torch.equal(bi[:, :k], want_i)
    assert torch.equal(bd[:, :k], want_d)
    if k < Ek:
        assert bool((bi[:, k:] == -1).all())
