"""The reference's extension interface, over libswann_b200.so.

geniussyn/SWANN reaches its kernels through one function, `ext()` in
swann/_engine.py:42-63, which JIT-builds swann/csrc/local_search.cu and returns
a pybind module with three entry points (local_search.cu:741-955):

    init_states(X, Qv, seeds, ids, dist, expd, lin, visited, counters,
                metric, team_size, cache_id, cache_d, bound)
    advance(X, G, Qv, ids, dist, expd, lin, visited, counters, metric,
            team_size, delta, max_expansions, policy, V, stop_eps, kstop,
            cache_id, cache_d, bound, exclusive, stall_patience, crowd_frac,
            active, codes, alpha, cmu, code_margin)
    merge_branches(bids, bdist, k) -> [ids, dist]

This module has exactly those three functions, with the same argument lists,
meanings, in-place writes and exception type (RuntimeError), so the reference's
own Python keeps running unchanged when its `ext()` returns this module:

    import swann._engine, swann_b200.refext
    swann._engine._EXT = swann_b200.refext

The reference keeps the per-query distance table as two arrays, cache_id
(int32, id + 1, 0 = empty) and cache_d (float32, FLT_MAX = not scored yet);
the kernels here keep it as one 64-bit word per slot ((id + 1) << 32 | the
distance's bits, 0 = empty) so that one compare-and-swap claims a node or
returns its distance.  The two forms hold the same information; each call
packs the caller's pair into a word array, runs, and writes the pair back,
so tables carried between calls (advance after advance) stay the caller's.
Empty tensors mean "feature off", as in the reference.
"""
from __future__ import annotations

import torch

from . import _lib as N

FLT_MAX_BITS = 0x7F7FFFFF
N_CTR = 10          # counters per branch (local_search.cu:35-41)
N_METRIC_IP = 0


class _Scratch:
    """The packed table of the last shape used, reused across calls."""

    def __init__(self):
        self.buf = None

    def get(self, shape, device):
        n = shape[0] * shape[1]
        if self.buf is None or self.buf.numel() < n or self.buf.device != device:
            self.buf = torch.empty(max(n, 1), dtype=torch.int64, device=device)
        return self.buf[:n].view(shape)


_TABLE = _Scratch()


def _fail(msg):
    raise RuntimeError(msg)


def _check(rc, what):
    if rc != N.OK:
        raise N.SwannError(rc, f"{what}: {N.lib().swb_last_error().decode(errors='replace')}")


def _check_common(X, Qv, ids, dist, expd, visited, counters):
    """The reference's check_common (local_search.cu:726-739)."""
    if not (X.is_cuda and X.is_contiguous() and X.dtype in (torch.float32, torch.float16)):
        _fail("X: contiguous cuda float32 or float16")
    if not (Qv.is_cuda and Qv.dtype == torch.float32 and Qv.is_contiguous()):
        _fail("Q: contiguous cuda float32")
    if not (ids.dtype == torch.int32 and ids.is_contiguous()):
        _fail("ids: contiguous int32")
    if not (dist.dtype == torch.float32 and dist.is_contiguous()):
        _fail("dist: contiguous float32")
    if not (expd.dtype == torch.uint8 and expd.is_contiguous()):
        _fail("expanded: contiguous uint8")
    if not (visited.dtype == torch.int32 and visited.is_contiguous()):
        _fail("visited: contiguous int32")
    if not (counters.dtype == torch.int32 and counters.is_contiguous()):
        _fail("counters: contiguous int32")


def _table_size(cache_id, cache_d):
    if cache_id.numel() == 0:
        return 0
    if not (cache_id.dtype == torch.int32 and cache_id.is_contiguous() and cache_d.dtype == torch.float32
            and cache_d.is_contiguous() and cache_d.shape == cache_id.shape):
        _fail("cache: contiguous int32 / float32")
    Hc = int(cache_id.shape[1])
    if Hc & (Hc - 1):
        _fail("cache size must be a power of two")
    return Hc


def _pack(cache_id, cache_d):
    """(id + 1, distance) pairs -> 64-bit words; an empty slot (id 0) is 0."""
    words = _TABLE.get(tuple(cache_id.shape), cache_id.device)
    hi = cache_id.to(torch.int64) << 32
    lo = cache_d.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    torch.where(cache_id != 0, hi | lo, torch.zeros((), dtype=torch.int64, device=cache_id.device), out=words)
    return words


def _unpack(words, cache_id, cache_d):
    """64-bit words -> the caller's (id + 1, distance) pair, in place; an empty
    slot reads (0, FLT_MAX) as the reference's init writes it."""
    cache_id.copy_((words >> 32).to(torch.int32))
    lo = (words & 0xFFFFFFFF).to(torch.int32)
    lo = torch.where(words == 0, torch.full_like(lo, FLT_MAX_BITS), lo)
    cache_d.copy_(lo.view(torch.float32))


def _ptr(t):
    return N.ptr(t)


def _stream(t):
    return N.stream_of(t)


def init_states(X, Qv, seeds, ids, dist, expd, lin, visited, counters, metric, team_size, cache_id, cache_d,
                bound):
    """Initialise per-branch search states (local_search.cu:741-776)."""
    _check_common(X, Qv, ids, dist, expd, visited, counters)
    if not (lin.dtype == torch.uint8 and lin.is_contiguous()):
        _fail("lineage: contiguous uint8")
    Q, J, L = ids.shape
    H = int(visited.shape[2])
    V = int(seeds.shape[2]) if seeds.dim() == 3 else 1
    if V > 128:
        _fail("seeds per branch exceed MAXD (the init sort buffer)")
    if L > 512:
        _fail("L exceeds MAXL")
    if H & (H - 1):
        _fail("visited table size must be a power of two")
    if counters.shape[2] != N_CTR:
        _fail("counters last dim must be NCTR")
    if Q > 65535:
        _fail(f"batch of {Q} queries exceeds the 65535 the grid's y dimension allows; split the batch")
    Hc = _table_size(cache_id, cache_d)
    words = _TABLE.get((Q, Hc), X.device) if Hc else None   # cleared by the kernel
    seeds = seeds.contiguous()
    with torch.cuda.device(X.device):
        rc = N.lib().swb_search_init(
            _ptr(X), N.dtype_code(X), X.shape[0], X.shape[1], _ptr(Qv), _ptr(seeds), Q, J, V,
            _ptr(ids), _ptr(dist), _ptr(expd), _ptr(lin), L, _ptr(visited), H, _ptr(counters), int(metric),
            int(team_size), _ptr(words) if Hc else None, Hc, _ptr(bound), _stream(X))
    _check(rc, "init_states")
    if Hc:
        _unpack(words, cache_id, cache_d)


def advance(X, G, Qv, ids, dist, expd, lin, visited, counters, metric, team_size, delta, max_expansions, policy,
            V_in, stop_eps, kstop, cache_id, cache_d, bound, exclusive, stall_patience, crowd_frac, active, codes,
            alpha, cmu, code_margin):
    """Advance each branch by up to `delta` expansions, in place
    (local_search.cu:778-841)."""
    _check_common(X, Qv, ids, dist, expd, visited, counters)
    if not (lin.dtype == torch.uint8 and lin.is_contiguous()):
        _fail("lineage: contiguous uint8")
    if not (G.is_cuda and G.dtype == torch.int32 and G.is_contiguous()):
        _fail("G: contiguous cuda int32")
    Q, J, L = ids.shape
    H = int(visited.shape[2])
    if G.shape[1] > 128:
        _fail("graph degree exceeds MAXD")
    if V_in > 256:
        _fail("lineage count exceeds 256 (lineage is a uint8)")
    if L > 512:
        _fail("L exceeds MAXL")
    if H & (H - 1):
        _fail("visited table size must be a power of two")
    Hc = _table_size(cache_id, cache_d)
    nact = int(active.numel())
    if nact and not (active.dtype == torch.int32 and active.is_contiguous()):
        _fail("active: contiguous int32")
    cw = 0
    if codes.numel():
        if int(metric) != N_METRIC_IP:
            _fail("the sign-code filter is written for the normalised inner-product corpora")
        if not (codes.is_cuda and codes.dtype == torch.int32 and codes.is_contiguous()):
            _fail("codes: contiguous cuda int32")
        if alpha.numel() != codes.shape[0] or cmu.numel() != X.shape[1]:
            _fail("codes, alpha and mu must agree with the corpus")
        cw = int(codes.shape[1])
        if cw * 32 < X.shape[1]:
            _fail("code words do not cover the dimension")
    words = _pack(cache_id, cache_d) if Hc else None
    with torch.cuda.device(X.device):
        rc = N.lib().swb_search_advance(
            _ptr(X), N.dtype_code(X), X.shape[0], X.shape[1], _ptr(G), G.shape[1], _ptr(Qv), _ptr(ids), _ptr(dist),
            _ptr(expd), _ptr(lin), Q, J, L, _ptr(visited), H, _ptr(counters), int(metric), int(team_size),
            int(delta), int(max_expansions), int(policy), int(V_in), float(stop_eps), int(kstop),
            _ptr(words) if Hc else None, Hc, _ptr(bound), int(exclusive), int(stall_patience), float(crowd_frac),
            _ptr(active) if nact else None, nact, _ptr(codes) if cw else None, _ptr(alpha) if cw else None,
            _ptr(cmu) if cw else None, float(code_margin), cw, None, _stream(X))
    _check(rc, "advance")
    if Hc:
        _unpack(words, cache_id, cache_d)


def merge_branches(bids, bdist, k):
    """Dedup by id and take the k nearest, per query (local_search.cu:925-947).
    Returns [ids int32 [Q, k], dist float32 [Q, k]]."""
    if not (bids.is_cuda and bdist.is_cuda):
        _fail("merge inputs must be on the GPU")
    if bids.dim() != 3 or bdist.shape != bids.shape:
        _fail("expected (Q, V, kk) for both ids and distances")
    if bids.dtype != torch.int32:
        _fail("ids must be int32")
    if bdist.dtype != torch.float32:
        _fail("distances must be float32")
    bids, bdist = bids.contiguous(), bdist.contiguous()
    Q, V, kk = bids.shape
    if not (0 < k <= V * kk):
        _fail("k must be in 1..V*kk")
    oi = torch.empty((Q, int(k)), dtype=torch.int32, device=bids.device)
    od = torch.empty((Q, int(k)), dtype=torch.float32, device=bids.device)
    with torch.cuda.device(bids.device):
        rc = N.lib().swb_merge_branches(_ptr(bids), _ptr(bdist), Q, V, kk, int(k), _ptr(oi), _ptr(od),
                                        _stream(bids))
    _check(rc, "merge_branches")
    return [oi, od]

