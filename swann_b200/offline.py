"""The offline graph builder's extras (offline/build_graph.py), on this build's
kernels: candidates from an existing graph, mutual-rank protection, per-node
degrees for the entry pool, an in-degree floor and filling empty degree slots
-- the same names, arguments and meaning as the reference's functions, and
`build_graph_offline` for its pipeline (build_graph.py:389-470).

Where the reference's result hangs on an unspecified order (torch.sort /
torch.argsort without stable=True) the order here is fixed: ties by position
when sorting candidates, the lowest source node when several offer an edge to
the same target in enforce_min_in.
"""
from __future__ import annotations

import time

import numpy as np
import torch

from . import _lib as N
from . import build as B

RULES = {"near": 0, "far": 1, "bridge": 2}


def _m(metric):
    return 0 if metric == "ip" else 1


@torch.no_grad()
def candidates_from_graph(Xg, Gc, C, metric="ip", chunk=1024):
    """Candidates from an existing approximate graph with exact distances
    (build_graph.py:73-99): the first min(C, width) neighbours of each node,
    -1 entries and the node itself at 3.4e38, ordered nearest first."""
    Xf = Xg.float().contiguous()
    Gc = Gc.to(device=Xf.device, dtype=torch.int32).contiguous()
    n = Gc.shape[0]
    C = min(int(C), Gc.shape[1])
    idx = torch.empty((n, C), dtype=torch.int32, device=Xf.device)
    dst = torch.empty((n, C), dtype=torch.float32, device=Xf.device)
    with torch.cuda.device(Xf.device):
        rc = N.lib().swb_graph_candidates(N.ptr(Xf), n, Xf.shape[1], N.ptr(Gc), Gc.shape[1], C, _m(metric),
                                          N.ptr(idx), N.ptr(dst), N.stream_of(Xf))
    N.check(rc, "candidates_from_graph")
    return idx, dst


@torch.no_grad()
def mutual_rank(cand, M, chunk=2048):
    """bool [n, C]: cand[u, i] (i < M) lists u among its own first M
    (build_graph.py:102-130); the prune's `protect`."""
    cand = cand.to(torch.int32).contiguous()
    n, C = cand.shape
    out = torch.empty((n, C), dtype=torch.uint8, device=cand.device)
    with torch.cuda.device(cand.device):
        rc = N.lib().swb_mutual_rank(N.ptr(cand), n, C, int(min(M, C)), N.ptr(out), N.stream_of(cand))
    N.check(rc, "mutual_rank")
    return out.bool()


@torch.no_grad()
def fill_degree(G, cand, rule="bridge", chunk=1024, deg_two=None):
    """Spend a node's empty degree slots on candidates the prune refused
    (build_graph.py:133-202): nearest first ("near"), farthest first ("far"),
    or the nearest with no two-hop path back through the kept graph
    ("bridge").  Returns a new graph; rows are processed `chunk` at a time in
    order, each chunk seeing the earlier chunks' fills."""
    if rule not in RULES:
        raise ValueError(f"rule must be one of {sorted(RULES)}")
    out = G.to(torch.int32).contiguous().clone()
    cand = cand.to(device=out.device, dtype=torch.int32).contiguous()
    n, W = out.shape
    C = cand.shape[1]
    tmp = torch.empty((min(chunk, n), W), dtype=torch.int32, device=out.device)
    with torch.cuda.device(out.device):
        rc = N.lib().swb_fill_degree(N.ptr(out), n, W, N.ptr(cand), C, RULES[rule], int(chunk), N.ptr(tmp),
                                     N.stream_of(out))
    N.check(rc, "fill_degree")
    return out


@torch.no_grad()
def enforce_min_in(Xg, G, cand, min_in, metric="ip", rounds=4, verbose=False):
    """Raise every node's in-degree to `min_in` at a fixed edge count
    (build_graph.py:309-386): a node short of in-edges offers itself to its
    candidates in order, and a target takes it in place of its farthest edge
    whose head is above the floor (never its nearest).  Modifies G in place and
    returns it; per-round figures are in `enforce_min_in.last_stats`."""
    if G.dtype != torch.int32 or not G.is_contiguous():
        raise ValueError("G must be a contiguous int32 tensor (it is modified in place)")
    cand = cand.to(device=G.device, dtype=torch.int32).contiguous()
    n, W = G.shape
    lib = N.lib()
    ws_bytes = int(lib.swb_min_in_workspace(n))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=G.device)
    stats = np.zeros((max(int(rounds), 1), 4), dtype=np.int32)
    ran = np.zeros(1, dtype=np.int32)
    with torch.cuda.device(G.device):
        rc = lib.swb_enforce_min_in(N.ptr(G), n, W, N.ptr(cand), cand.shape[1], int(min_in), int(rounds),
                                    N.ptr(ws), ws_bytes, stats.ctypes.data, ran.ctypes.data, N.stream_of(G))
    N.check(rc, "enforce_min_in")
    enforce_min_in.last_stats = [dict(below=int(a), to_place=int(b), placed=int(c), already_linked=int(d))
                                 for a, b, c, d in stats[:int(ran[0])]]
    if verbose:
        for r, s in enumerate(enforce_min_in.last_stats):
            print(f"  min-in {min_in} round {r}: {s['below']:,} below, {s['to_place']:,} edges to place, "
                  f"placed {s['placed']:,}, already linked {s['already_linked']:,}")
    return G


enforce_min_in.last_stats = []


@torch.no_grad()
def build_graph_offline(X, D=64, cand=128, metric="ip", alpha=1.2, fill=None, cand_graph=None, pool=None,
                        pool_boost=0, mutual=0, min_in=0, min_in_rounds=6):
    """The reference's offline pipeline (build_graph.py:389-470) on the GPU:
    candidates (exact sweep, or `cand_graph`'s edges), per-node degrees for the
    entry `pool` (+`pool_boost`, capped at min(cand, 128)), mutual-rank
    protection, prune, reverse, in-degree floor, degree fill.
    Returns (G int32 [n, width] on the GPU, info dict)."""
    Xg = X if isinstance(X, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(X))
    if Xg.device.type != "cuda":
        Xg = Xg.cuda()
    n = Xg.shape[0]
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    if cand_graph is not None:
        Gc = cand_graph if isinstance(cand_graph, torch.Tensor) else torch.from_numpy(np.asarray(cand_graph))
        cd, cdist = candidates_from_graph(Xg, Gc.to(Xg.device), cand, metric=metric)
    else:
        cd, cdist = B.knn_candidates(Xg, cand, metric=metric)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    dpn = None
    if pool_boost and pool is not None:
        dpn = torch.full((n,), D, dtype=torch.int32, device=Xg.device)
        pi = torch.as_tensor(np.asarray(pool), dtype=torch.int64, device=Xg.device)
        dpn[pi] = min(D + pool_boost, min(cand, 128))
    prot = mutual_rank(cd, mutual) if mutual else None
    G = B.robust_prune(Xg, cd, cdist, D, alpha=alpha, deg_per_node=dpn, metric=metric, protect=prot)
    torch.cuda.synchronize()
    t2 = time.perf_counter()
    G = B.add_reverse(Xg, G, D, alpha=alpha, deg_per_node=dpn, metric=metric).contiguous()
    if min_in:
        G = enforce_min_in(Xg, G, cd, min_in, metric=metric, rounds=min_in_rounds)
    if fill:
        G = fill_degree(G, cd, rule=fill)
    torch.cuda.synchronize()
    t3 = time.perf_counter()
    info = dict(deg=D, cand=cand, candidates="graph" if cand_graph is not None else "exact", alpha=alpha,
                metric=metric, pool_boost=pool_boost, min_in=min_in, mutual=mutual, fill=fill,
                seconds=round(t3 - t0, 3),
                stage_seconds=dict(candidates=round(t1 - t0, 3), prune=round(t2 - t1, 3), reverse=round(t3 - t2, 3)),
                min_in_rounds=list(enforce_min_in.last_stats) if min_in else [])
    return G, info
