"""ctypes front-end of the C oracle -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import this module, and only as a checker or as the timed CPU baseline; the
product (``swann_b200``) never does.

Every function mirrors one reference function (paths inside geniussyn/SWANN):

  team_distance     swann/_refcpu.py:21-48
  branch_run        swann/_refcpu.py:146-151 (init_state + advance)
  search            _refcpu.run per branch + merge (tests/test_engine.py:200-208);
                    with shared_* flags, a lockstep emulation of the kernel's
                    shared table / bound / claims (swann/csrc/local_search.cu)
  merge_branches    swann/csrc/local_search.cu:863-919
  knn_candidates    swann/build.py:30-43 (exact, in double)
  robust_prune      swann/build.py:48-91
  add_reverse       swann/build.py:96-150

It also hosts the loader for the reference's own compiled kernels
(``oracle/_ref``), used by the GPU tests as a second checker.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
METRIC_IP, METRIC_L2 = 0, 1
POLICY_BEST, POLICY_ROUND_ROBIN = 0, 1
NCTR = 10

_LIB = None


def lib():
    global _LIB
    if _LIB is None:
        so = HERE / "liboracle.so"
        if not so.exists():
            from .build_oracle import build_oracle  # noqa: WPS433
            build_oracle()
        _LIB = C.CDLL(str(so))
        _declare(_LIB)
    return _LIB


def _p(a):
    return a.ctypes.data_as(C.c_void_p)


def _declare(L):
    vp, i32, i64, f32 = C.c_void_p, C.c_int, C.c_int64, C.c_float
    L.or_team_distance.restype = f32
    L.or_team_distance.argtypes = [vp, vp, i32, i32, i32, i32]
    L.or_branch_run.restype = i32
    L.or_branch_run.argtypes = [vp, i32, vp, i32, vp, vp, i32, i32, i32, i32, i32, i32,
                                i32, f32, i32, i32, f32, i32, vp, vp, vp, vp, vp]
    L.or_merge_branches.restype = None
    L.or_merge_branches.argtypes = [vp, vp, i32, i32, i32, i32, vp, vp]
    L.or_search.restype = i32
    L.or_search.argtypes = [vp, i64, i32, vp, i32, vp, i32, vp, i32, i32, i32, i32, i32,
                            i32, i32, i32, i32, f32, i32, i32, i32, i32, i32, i32, f32, i32, vp, vp, vp]
    L.or_knn_candidates.restype = i32
    L.or_knn_candidates.argtypes = [vp, i64, i32, i32, i32, i64, i64, i32, vp, vp, vp]
    L.or_robust_prune.restype = i32
    L.or_robust_prune.argtypes = [vp, i64, i32, vp, vp, i32, i32, f32, i32, vp, vp, i32, vp]
    L.or_set_square_mode.restype = None
    L.or_set_square_mode.argtypes = [i32]
    L.or_add_reverse.restype = i32
    L.or_add_reverse.argtypes = [vp, i64, i32, vp, i32, f32, i32, i32, vp, i32, vp]


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _i32(a):
    return np.ascontiguousarray(a, dtype=np.int32)


class square_mode:
    """Scope in which L2 terms are squared as _refcpu squares them (libm powf,
    ``"refcpu"``) instead of as the kernel does (one rounded multiply,
    ``"kernel"``, the default)."""

    def __init__(self, mode="refcpu"):
        self.mode = {"kernel": 0, "refcpu": 1}[mode]

    def __enter__(self):
        lib().or_set_square_mode(self.mode)
        return self

    def __exit__(self, *exc):
        lib().or_set_square_mode(0)
        return False


def default_vec(X) -> int:
    """16-byte loads: 4 fp32 or 8 fp16 elements per lane step."""
    return 8 if np.asarray(X).dtype == np.float16 else 4


def team_distance(q, x, metric=METRIC_IP, team=32, vec=4) -> np.float32:
    q, x = _f32(q), _f32(x)
    return np.float32(lib().or_team_distance(_p(q), _p(x), q.shape[0], metric, team, vec))


def branch_run(X, G, q, seeds, L=16, B=16, metric=METRIC_IP, team=32, vec=None,
               policy=POLICY_BEST, stop_eps=-1.0, kstop=10, delta=None, stall_patience=0, crowd_frac=0.0):
    """One branch, init + advance(delta or B).  Returns dict of L-slot arrays.
    stall_patience / crowd_frac: the kernel's stall and crowd rules
    (swann/csrc/local_search.cu:659-682), 0 = off."""
    vec = default_vec(X) if vec is None else vec
    X, G, q = _f32(X), _i32(G), _f32(q)
    seeds = _i32(np.atleast_1d(seeds))
    ids = np.empty(L, np.int32); dist = np.empty(L, np.float32)
    expd = np.empty(L, np.uint8); lin = np.empty(L, np.uint8); ctr = np.empty(NCTR, np.int32)
    lib().or_branch_run(_p(X), X.shape[1], _p(G), G.shape[1], _p(q), _p(seeds), seeds.shape[0],
                        L, B, metric, team, vec, policy, float(stop_eps), kstop, int(stall_patience),
                        float(crowd_frac), B if delta is None else delta, _p(ids), _p(dist), _p(expd), _p(lin),
                        _p(ctr))
    return dict(ids=ids, dist=dist, expanded=expd, lineage=lin, counters=ctr)


def search(X, G, Q, seeds, k=10, L=16, B=16, metric=METRIC_IP, team=32, vec=None,
           policy=POLICY_BEST, stop_eps=-1.0, kstop=None, shared_cache=False,
           shared_bound=False, exclusive=False, elide_visited=False, threads=0,
           counters=False, stall_patience=0, crowd_frac=0.0):
    """seeds [nq, J] or [nq, J, V].  Returns (ids [nq,k], dist [nq,k][, ctr])."""
    vec = default_vec(X) if vec is None else vec
    X, G, Q = _f32(X), _i32(G), _f32(Q)
    seeds = _i32(seeds)
    if seeds.ndim == 2:
        seeds = seeds[:, :, None].copy()
    nq, J, V = seeds.shape
    kstop = k if kstop is None else kstop
    ids = np.empty((nq, k), np.int32); dist = np.empty((nq, k), np.float32)
    ctr = np.zeros((nq, J, NCTR), np.int32)
    lib().or_search(_p(X), X.shape[0], X.shape[1], _p(G), G.shape[1], _p(Q), nq, _p(seeds), J, V,
                    k, L, B, metric, team, vec, policy, float(stop_eps), kstop,
                    int(shared_cache), int(shared_bound), int(exclusive), int(elide_visited),
                    int(stall_patience), float(crowd_frac), int(threads), _p(ids), _p(dist), _p(ctr))
    return (ids, dist, ctr) if counters else (ids, dist)


def merge_branches(ids, dist, k):
    ids, dist = _i32(ids), _f32(dist)
    Q, J, kk = ids.shape
    oi = np.empty((Q, k), np.int32); od = np.empty((Q, k), np.float32)
    lib().or_merge_branches(_p(ids), _p(dist), Q, J, kk, k, _p(oi), _p(od))
    return oi, od


def knn_candidates(X, C, metric=METRIC_IP, rows=None, threads=0, exact64=False):
    """Exact top-C by (distance, id), self excluded.  rows=(r0, r1) for a sample."""
    X = _f32(X)
    n = X.shape[0]
    r0, r1 = (0, n) if rows is None else rows
    idx = np.empty((r1 - r0, C), np.int32); dst = np.empty((r1 - r0, C), np.float32)
    d64 = np.empty((r1 - r0, C), np.float64) if exact64 else None
    lib().or_knn_candidates(_p(X), n, X.shape[1], C, metric, r0, r1, threads, _p(idx), _p(dst),
                            _p(d64) if exact64 else None)
    return (idx, dst, d64) if exact64 else (idx, dst)


def robust_prune(X, cand, cdist, deg, alpha=1.2, metric=METRIC_IP, threads=0, deg_per_node=None, protect=None):
    """deg_per_node: per-node caps (the width is then their largest);
    protect: bool [n, C] candidates exempt from the detour test."""
    X, cand, cdist = _f32(X), _i32(cand), _f32(cdist)
    dpn = None if deg_per_node is None else _i32(deg_per_node)
    width = int(deg) if dpn is None else int(dpn.max())
    prot = None if protect is None else np.ascontiguousarray(protect, dtype=np.uint8)
    out = np.empty((cand.shape[0], width), np.int32)
    lib().or_robust_prune(_p(X), cand.shape[0], X.shape[1], _p(cand), _p(cdist), cand.shape[1],
                          width, float(alpha), metric, _p(dpn) if dpn is not None else None,
                          _p(prot) if prot is not None else None, threads, _p(out))
    return out


def add_reverse(X, G, deg, alpha=1.2, max_in=64, metric=METRIC_IP, threads=0, deg_per_node=None):
    """deg_per_node: per-node caps of the re-prune; G's width is their largest."""
    X, G = _f32(X), _i32(G)
    dpn = None if deg_per_node is None else _i32(deg_per_node)
    out = np.empty((G.shape[0], G.shape[1]), np.int32)
    lib().or_add_reverse(_p(X), X.shape[0], X.shape[1], _p(G), G.shape[1], float(alpha), max_in,
                         metric, _p(dpn) if dpn is not None else None, threads, _p(out))
    return out


def build_graph(X, metric=METRIC_IP, degree=96, candidates=128, alpha=1.2, threads=0):
    """The reference's three stages (swann/build.py:156-171), on the CPU."""
    cand, cd = knn_candidates(X, candidates, metric, threads=threads)
    G = robust_prune(X, cand, cd, degree, alpha, metric, threads=threads)
    return add_reverse(X, G, degree, alpha, metric=metric, threads=threads)


# ---------------------------------------------------------------------------
# the reference's own kernels, compiled for sm_100a (checker on the GPU box)

_REF = None


def ref_kernels():
    """The compiled reference extension (init_states / advance / merge_branches),
    or None when it was not built (no reference tree where the build ran)."""
    global _REF
    if _REF is None:
        so = HERE / "_ref" / "swann_ref_ls.so"
        if not so.exists():
            return None
        import importlib.util
        import torch  # noqa: F401  (the extension links against torch)
        spec = importlib.util.spec_from_file_location("swann_ref_ls", str(so))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        _REF = mod
    return _REF


def cpu_count() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1
