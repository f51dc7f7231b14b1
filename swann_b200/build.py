"""Graph construction: exact candidates, a detour-pruning pass, reverse edges.

Drop-in for swann/build.py (geniussyn/SWANN): `pairwise`, `knn_candidates`,
`robust_prune`, `add_reverse`, `build_graph`, same arguments and results.

  knn_candidates  exact top-C by the metric, self excluded.  A chunk of rows
                  is scored against the whole corpus and each row's C nearest
                  are selected by swb_topc_block (native); the dot products of
                  the chunk come from a tensor-core GEMM.
  robust_prune    swb_prune_tc (inner product): one block per node, the
                  candidates' Gram matrix on the tensor cores, the reference's
                  sequential keep rule; swb_prune (l2): the same on CUDA cores.
  add_reverse     swb_reverse_tc: stable radix sort of the edges by target, row
                  merge + scoring, then the same prune.

The prune and reverse passes decide every detour test as a dimension-ordered
fmaf dot product would (the tensor-core pass recomputes with that chain every
pair its own values cannot decide for certain), so their output is
reproducible bit for bit from the same input.
"""
from __future__ import annotations

import os

import torch

from . import _lib as N
from ._engine import METRIC_IP, METRIC_L2

_METRIC = {"ip": METRIC_IP, "l2": METRIC_L2}


def _m(metric) -> int:
    if isinstance(metric, str):
        if metric not in _METRIC:
            raise ValueError(f"metric must be one of {sorted(_METRIC)}")
        return _METRIC[metric]
    return int(metric)


def pairwise(A, B, metric, bn=None):
    """Distances from every row of A to every row of B, in the corpus's metric
    (swann/build.py:14-25).  Library GEMM; kept for API parity."""
    if _m(metric) == METRIC_IP:
        return 1.0 - (A @ B.T)
    if bn is None:
        bn = (B * B).sum(1)
    return (bn.view(1, -1) - 2.0 * (A @ B.T) + (A * A).sum(1).view(-1, 1)).clamp(min=0)


def row_norms(Xg):
    out = torch.empty(Xg.shape[0], dtype=torch.float32, device=Xg.device)
    with torch.cuda.device(Xg.device):
        N.check(N.lib().swb_row_norms(N.ptr(Xg), N.dtype_code(Xg), Xg.shape[0], Xg.shape[1], N.ptr(out),
                                      N.stream_of(Xg)), "row_norms")
    return out


def _dots(A, B, exact_half):
    """A @ B.T in fp32.  fp16-valued rows multiply exactly in TF32 (11-bit
    significands), so their products are exact and only the accumulation
    order differs from a plain fp32 GEMM."""
    if exact_half:
        try:
            return torch.mm(A.half(), B.half().T, out_dtype=torch.float32)
        except (RuntimeError, TypeError):
            pass
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = bool(exact_half)
    try:
        return A @ B.T
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


class TcOperands:
    """A corpus's rows as the tensor cores read them, prepared once and shared
    by the sweep, the prune and the reverse pass: fp16 rows (fp16-valued
    corpora, padded to a multiple of 64 columns) or tf32 high and low parts
    (padded to a multiple of 32), the fp32 rows, and their squared norms in
    the fmaf-chain order the prune's pair distances use."""

    def __init__(self, Xg, half_exact=None):
        Xg = Xg.contiguous()
        if half_exact is None:
            small = Xg.shape[0] * Xg.shape[1] <= (1 << 26)
            half_exact = bool(Xg.dtype == torch.float16 or (small and torch.equal(Xg.float(), Xg.half().float())))
        self.half = half_exact
        self.X = Xg.float().contiguous()
        self.norms = row_norms(self.X)
        self.dim = self.X.shape[1]
        if half_exact:
            self.A, self.A_lo, self.code = _pad_cols(Xg.half().contiguous(), 64), None, N.F16
        else:
            Xp = _pad_cols(self.X, 32)
            self.A, self.A_lo = torch.empty_like(Xp), torch.empty_like(Xp)
            with torch.cuda.device(Xg.device):
                N.check(N.lib().swb_split_tf32(N.ptr(Xp), Xp.numel(), N.ptr(self.A), N.ptr(self.A_lo),
                                               N.stream_of(Xg)), "split")
            self.code = N.F32
        self.adim = self.A.shape[1]
        self.recomputed = torch.zeros(1, dtype=torch.int64, device=Xg.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=Xg.device)

    def check(self):
        if int(self.status[0]) != 0:
            raise N.SwannError(int(self.status[0]), "a device-side wait timed out in the tensor-core prune")


def _prune_method(method, metric):
    """"tc" or "simt".  By default the tensor cores for inner product and the
    CUDA cores for l2: the l2 pair distance (|x|^2 - 2<x, y>) + |y|^2 cancels
    (|x|^2 + |y|^2 far above the distance on unnormalised rows), so the
    tensor-core Gram's error bound, which scales with |x||y|, sends a large
    share of the pairs to the exact recompute (C5: 2.7 s against 1.6 s on CUDA
    cores, measured).  Both give the same graph."""
    method = method or os.environ.get("SWB_PRUNE") or ("tc" if _m(metric) == METRIC_IP else "simt")
    if method not in ("tc", "simt"):
        raise ValueError("prune method must be 'tc' or 'simt'")
    return method


def _pad_cols(X, mult):
    d = X.shape[1]
    if d % mult == 0:
        return X
    P = torch.zeros((X.shape[0], d + (-d) % mult), dtype=X.dtype, device=X.device)
    P[:, :d] = X
    return P


@torch.no_grad()
def knn_candidates(Xg, C, chunk=4096, metric="ip", col_chunk=1 << 20, half_exact=None, rows=None,
                   method=None, row_block=1 << 18, ops=None):
    """Exact top-C neighbours by the corpus's metric, self excluded
    (swann/build.py:30-43).  Returns (idx int32 [m, C], dst f32 [m, C]) for
    rows=(r0, r1) (default: every row), m = r1 - r0.

    method="mma" (default): swb_sweep_topc, the tcgen05 sweep with the top-C
    fused (fp16-valued rows exactly in kind::f16, others in 3xTF32).
    method="gemm": a library GEMM per row chunk and swb_topc_block.
    The default is "mma" unless SWB_SWEEP names the other."""
    if method is None:
        method = os.environ.get("SWB_SWEEP", "mma")
    if method == "mma":
        return _knn_mma(Xg, C, metric, half_exact, rows, row_block, ops)
    m = _m(metric)
    if not Xg.is_cuda:
        raise ValueError("vectors must be on the GPU")
    Xg = Xg.contiguous()
    n = Xg.shape[0]
    if half_exact is None:
        small = n * Xg.shape[1] <= (1 << 26)
        half_exact = bool(Xg.dtype == torch.float16 or (small and torch.equal(Xg, Xg.half().float())))
    Xf = Xg.float().contiguous()
    norms = row_norms(Xf) if m == METRIC_L2 else None
    R0, R1 = (0, n) if rows is None else rows
    idx = torch.empty((R1 - R0, C), dtype=torch.int32, device=Xg.device)
    dst = torch.empty((R1 - R0, C), dtype=torch.float32, device=Xg.device)
    lib = N.lib()
    with torch.cuda.device(Xg.device):
        s = N.stream_of(Xg)
        for r0 in range(R0, R1, chunk):
            r1 = min(r0 + chunk, R1)
            for c0 in range(0, n, col_chunk):
                c1 = min(c0 + col_chunk, n)
                D = _dots(Xf[r0:r1], Xf[c0:c1], half_exact).contiguous()
                rc = lib.swb_topc_block(N.ptr(D), r1 - r0, D.shape[1], c1 - c0, r0, c0, N.ptr(norms), m, C,
                                        N.ptr(idx[r0 - R0:r1 - R0]), N.ptr(dst[r0 - R0:r1 - R0]), int(c0 > 0), s)
                N.check(rc, "knn_candidates")
                del D
    return idx, dst


def _knn_mma(Xg, C, metric, half_exact, rows, row_block, ops=None):
    m = _m(metric)
    if not Xg.is_cuda:
        raise ValueError("vectors must be on the GPU")
    n = Xg.shape[0]
    if ops is None:
        ops = TcOperands(Xg, half_exact)
    norms = ops.norms if m == METRIC_L2 else None
    hi, lo, code = ops.A, ops.A_lo, ops.code
    R0, R1 = (0, n) if rows is None else rows
    idx = torch.empty((R1 - R0, C), dtype=torch.int32, device=Xg.device)
    dst = torch.empty((R1 - R0, C), dtype=torch.float32, device=Xg.device)
    status = torch.zeros(1, dtype=torch.int32, device=Xg.device)
    lib = N.lib()
    with torch.cuda.device(Xg.device):
        s = N.stream_of(Xg)
        for r0 in range(R0, R1, row_block):
            r1 = min(R1, r0 + row_block)
            ws_bytes = int(lib.swb_sweep_workspace(n, r1 - r0, C, code))
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device=Xg.device)
            rc = lib.swb_sweep_topc(N.ptr(hi), N.ptr(lo), code, n, hi.shape[1], N.ptr(norms), r0, r1 - r0, C, m,
                                    N.ptr(idx[r0 - R0:r1 - R0]), N.ptr(dst[r0 - R0:r1 - R0]), N.ptr(ws), ws_bytes,
                                    N.ptr(status), s)
            N.check(rc, "knn_candidates")
    if int(status[0]) != 0:
        code = int(status[0])
        why = ("the sweep's shared memory was not 1024-byte aligned" if code == N.ERR_SMEM
               else "a device-side wait timed out in the sweep")
        raise N.SwannError(code, why)
    return idx, dst


@torch.no_grad()
def robust_prune(Xg, cand, cdist, deg, alpha=1.2, chunk=4096, deg_per_node=None, metric="ip", protect=None,
                 method=None, ops=None):
    """Keep a candidate only when no nearer kept neighbour detours to it
    (swann/build.py:48-91).  Returns int32 [n, width], -1 padded: width = deg,
    or the largest of `deg_per_node` (per-node caps, int [n]) when given.
    `protect` (bool [n, C], e.g. mutual_rank's) exempts a candidate from the
    detour test.  method "tc" (default; SWB_PRUNE overrides): pair distances
    on the tensor cores, `ops` (TcOperands) prepared once per corpus; "simt":
    on CUDA cores.  Both give the same graph, bit for bit; the default is
    "tc" for inner product and "simt" for l2 (see _prune_method)."""
    method = _prune_method(method, metric)
    Xf = ops.X if (method == "tc" and ops is not None) else Xg.float().contiguous()
    cand = cand.to(torch.int32).contiguous()
    cdist = cdist.float().contiguous()
    n, C = cand.shape
    width = int(deg)
    dpn = None
    if deg_per_node is not None:
        dpn = deg_per_node.to(device=Xg.device, dtype=torch.int32).contiguous()
        if dpn.shape != (n,):
            raise ValueError("deg_per_node must have one entry per node")
        width = int(dpn.max())
    prot = None
    if protect is not None:
        prot = protect.to(device=Xg.device, dtype=torch.uint8).contiguous()
        if prot.shape != (n, C):
            raise ValueError("protect must have the candidate matrix's shape")
    out = torch.empty((n, width), dtype=torch.int32, device=Xg.device)
    with torch.cuda.device(Xg.device):
        if method == "tc":
            ops = ops or TcOperands(Xg)
            rc = N.lib().swb_prune_tc(N.ptr(ops.X), N.ptr(ops.A), N.ptr(ops.A_lo), ops.code, ops.adim,
                                      N.ptr(ops.norms), Xf.shape[0], Xf.shape[1], N.ptr(cand), N.ptr(cdist), n, C,
                                      width, float(alpha), _m(metric), N.ptr(dpn), N.ptr(prot), N.ptr(out),
                                      N.ptr(ops.recomputed), N.ptr(ops.status), N.stream_of(Xg))
        else:
            rc = N.lib().swb_prune(N.ptr(Xf), Xf.shape[0], Xf.shape[1], N.ptr(cand), N.ptr(cdist), n, C, width,
                                   float(alpha), _m(metric), N.ptr(dpn), N.ptr(prot), N.ptr(out), N.stream_of(Xg))
    N.check(rc, "robust_prune")
    if method == "tc":
        ops.check()
    return out


@torch.no_grad()
def add_reverse(Xg, G, deg, chunk=2048, alpha=1.2, max_in=64, deg_per_node=None, metric="ip", rows=None,
                method=None, ops=None):
    """Offer every edge back to its target, then re-prune the union per node
    (swann/build.py:96-150).  rows=(r0, r1) re-prunes only those rows (a
    rank's block of a sharded build); G is always the whole graph.  With
    `deg_per_node` (int [n]) the caps are per node and the width is their
    largest, as robust_prune writes it.  `method` / `ops` as robust_prune."""
    method = _prune_method(method, metric)
    if method == "tc":
        ops = ops or TcOperands(Xg)
    Xf = ops.X if method == "tc" else Xg.float().contiguous()
    G = G.to(torch.int32).contiguous()
    n = G.shape[0]
    r0, r1 = (0, n) if rows is None else rows
    dpn = None
    width = int(deg)
    if deg_per_node is not None:
        dpn = deg_per_node.to(device=Xg.device, dtype=torch.int32).contiguous()
        width = int(dpn.max())
    if G.shape[1] != width:
        raise ValueError("add_reverse: the graph's width must equal deg (the largest per-node degree)")
    deg = width
    out = torch.empty((r1 - r0, deg), dtype=torch.int32, device=Xg.device)
    lib = N.lib()
    ws_bytes = int(lib.swb_reverse_workspace(n, r1 - r0, G.shape[1], max_in))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=Xg.device)
    with torch.cuda.device(Xg.device):
        if method == "tc":
            rc = lib.swb_reverse_tc(N.ptr(Xf), N.ptr(ops.A), N.ptr(ops.A_lo), ops.code, ops.adim, N.ptr(ops.norms),
                                    n, Xf.shape[1], N.ptr(G), int(deg), float(alpha), int(max_in), _m(metric),
                                    N.ptr(dpn), r0, r1 - r0, N.ptr(out), N.ptr(ws), ws_bytes,
                                    N.ptr(ops.recomputed), N.ptr(ops.status), N.stream_of(Xg))
        else:
            rc = lib.swb_reverse(N.ptr(Xf), n, Xf.shape[1], N.ptr(G), int(deg), float(alpha), int(max_in),
                                 _m(metric), N.ptr(dpn), r0, r1 - r0, N.ptr(out), N.ptr(ws), ws_bytes,
                                 N.stream_of(Xg))
    N.check(rc, "add_reverse")
    if method == "tc":
        ops.check()
    return out


@torch.no_grad()
def build_graph(X, metric: str = "ip", degree: int = 96, candidates: int = 128, alpha: float = 1.2):
    """Return an (n, degree) int32 neighbour table on the GPU (build.py:156-171)."""
    if X.device.type != "cuda":
        X = X.cuda()
    Xg = X.contiguous()
    ops = TcOperands(Xg)
    cand, cdist = knn_candidates(Xg, candidates, metric=metric, ops=ops)
    G = robust_prune(Xg, cand, cdist, degree, alpha=alpha, metric=metric, ops=ops)
    del cand, cdist
    G = add_reverse(Xg, G, degree, alpha=alpha, metric=metric, ops=ops)
    return G.to(torch.int32).contiguous()
