"""Entry (seed) selection: the E catalogue entries nearest each query.

Drop-in for swann/_select.py (geniussyn/SWANN:54-128): `pool_vectors`,
`catalog_scores`, `select_nearest` and `reduced_precision`, same arithmetic --
a TF32 matmul of the queries against the catalogue rows in slices of 8192,
turned into the corpus metric, with a running top-E (swb_select_topk).  The
matmul is a plain library GEMM (cuBLAS through torch); its output only chooses
starting points, and the search re-scores everything exactly.
"""
from __future__ import annotations

import torch

from ._engine import METRIC_IP, METRIC_L2  # noqa: F401


class reduced_precision:
    """Scope in which fp32 matmuls may use TF32 (allow_tf32 is process-global)."""

    def __init__(self, on=True):
        self.on = bool(on)

    def __enter__(self):
        self.prev = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = self.on
        return self

    def __exit__(self, *exc):
        torch.backends.cuda.matmul.allow_tf32 = self.prev
        return False


def pool_vectors(Xg, pool_t):
    """The catalogue's rows as their own matrix, held for the life of the index."""
    return Xg[pool_t.long()].contiguous()


def catalog_scores(Qg, Xg, pool_t, metric=METRIC_IP, Vp=None, precision="tf32"):
    """Distance from every query to every pool entry, in the corpus's metric."""
    V = Vp if Vp is not None else Xg[pool_t.long()]
    if precision == "fp16":
        s = (Qg.half() @ V.half().T).float()
    else:
        with reduced_precision(precision == "tf32"):
            s = Qg @ V.T
    if metric == METRIC_IP:
        return 1.0 - s
    return (V * V).sum(1).view(1, -1) - 2.0 * s + (Qg * Qg).sum(1).view(-1, 1)


def select_nearest(Qg, Vp, E, metric=METRIC_IP, precision="tf32", slice_P=8192):
    """Indices (into the catalogue) of the E nearest entries per query, sorted
    nearest first: the catalogue is scored a slice at a time (a library GEMM,
    the reference's precision choices) and each slice folded into a running
    best by swb_select_topk, which reads the scores once and keeps the list in
    shared memory (the reference runs two torch.topk per slice).  Same entries
    as the reference, up to the order of exactly equal distances."""
    from . import _lib as N
    n, P = Qg.shape[0], Vp.shape[0]
    Ee = min(int(E), P)
    bd = torch.empty((n, Ee), dtype=torch.float32, device=Qg.device)
    bi = torch.empty((n, Ee), dtype=torch.int64, device=Qg.device)
    if n == 0 or Ee == 0:
        return bi
    qn = (Qg * Qg).sum(1).contiguous() if metric != METRIC_IP else None
    stream = N.stream_of(Qg)
    for s in range(0, P, slice_P):
        V = Vp[s:s + slice_P]
        if precision == "fp16":
            sc = (Qg.half() @ V.half().T).float()
        else:
            with reduced_precision(precision == "tf32"):
                sc = Qg @ V.T
        sc = sc.contiguous()
        vn = (V * V).sum(1).contiguous() if metric != METRIC_IP else None
        rc = N.lib().swb_select_topk(N.ptr(sc), n, V.shape[0], sc.stride(0), N.ptr(vn), N.ptr(qn), int(metric), Ee,
                                     s, N.ptr(bd), N.ptr(bi), int(s > 0), stream)
        N.check(rc, "swb_select_topk")
    return bi
