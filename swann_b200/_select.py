"""Entry (seed) selection: the E catalogue entries nearest each query.

Drop-in for swann/_select.py (geniussyn/SWANN:54-128): `pool_vectors`,
`catalog_scores`, `select_nearest` and `reduced_precision`, same arithmetic --
a TF32 matmul of the queries against the catalogue rows in slices of 8192,
turned into the corpus metric, with a running top-E.  The matmul is a plain
library GEMM (cuBLAS through torch); its output only chooses starting points,
and the search re-scores everything exactly.
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
    """Indices (into the catalogue) of the E nearest entries per query,
    scored a slice of the catalogue at a time and folded into a running best."""
    n, P = Qg.shape[0], Vp.shape[0]
    bi = torch.empty(n, 0, dtype=torch.long, device=Qg.device)
    bv = torch.empty(n, 0, dtype=Qg.dtype, device=Qg.device)
    qn = (Qg * Qg).sum(1).view(-1, 1) if metric != METRIC_IP else None
    for s in range(0, P, slice_P):
        V = Vp[s:s + slice_P]
        if precision == "fp16":
            sc = (Qg.half() @ V.half().T).float()
        else:
            with reduced_precision(precision == "tf32"):
                sc = Qg @ V.T
        c = (1.0 - sc) if metric == METRIC_IP else ((V * V).sum(1).view(1, -1) - 2.0 * sc + qn)
        v, i = torch.topk(c, min(E, c.shape[1]), dim=1, largest=False)
        bv = torch.cat([bv, v], 1)
        bi = torch.cat([bi, i + s], 1)
        if bv.shape[1] > E:
            v, j = torch.topk(bv, E, dim=1, largest=False)
            bv, bi = v, torch.gather(bi, 1, j)
    return bi
