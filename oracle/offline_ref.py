"""CPU restatement of the offline builder's extras (offline/build_graph.py) --
test infrastructure only: the checker for swann_b200.offline, never part of
the product path.  Pinned against outputs of the reference's own functions
(tests/golden/offline.npz, written by tests/golden/make_offline_golden.py).

Plain numpy loops over nodes, for small inputs.  Where the reference leaves
an order unspecified (torch.sort / torch.argsort without stable=True), this
fixes it the way the kernels do: ties by position, the lowest source node per
target.
"""
from __future__ import annotations

import numpy as np

FAR = np.float32(3.4e38)


def graph_candidates(X, Gc, C, metric):
    """candidates_from_graph (build_graph.py:73-99): first C entries of each
    row, exact distances (float64 here), -1 and self at 3.4e38, sorted by
    (distance, position)."""
    X = np.asarray(X, np.float64)
    n = Gc.shape[0]
    C = min(C, Gc.shape[1])
    idx = np.empty((n, C), np.int32)
    dst = np.empty((n, C), np.float32)
    for u in range(n):
        ids = Gc[u, :C]
        d = np.full(C, FAR, np.float64)
        ok = (ids >= 0) & (ids != u)
        if metric == 0:
            d[ok] = 1.0 - X[ids[ok]] @ X[u]
        else:
            d[ok] = ((X[ids[ok]] - X[u]) ** 2).sum(1)
        o = np.lexsort((np.arange(C), d))
        idx[u], dst[u] = ids[o], d[o].astype(np.float32)
    return idx, dst


def mutual_rank(cand, M):
    """build_graph.py:102-130: cand[u, i] (i < M) lists u among its first M."""
    n, C = cand.shape
    M = min(M, C)
    out = np.zeros((n, C), np.uint8)
    for u in range(n):
        for i in range(M):
            v = cand[u, i]
            if v >= 0 and (cand[v, :M] == u).any():
                out[u, i] = 1
    return out


def fill_degree(G, cand, rule="bridge", chunk=1024):
    """build_graph.py:133-202, row chunks in order; a chunk's rows see the
    graph as the earlier chunks left it, and each other unfilled."""
    out = G.copy()
    n, W = G.shape
    C = cand.shape[1]
    for s in range(0, n, chunk):
        e = min(s + chunk, n)
        before = out.copy()
        for u in range(s, e):
            kept = before[u]
            two = set()
            if rule == "bridge":
                for w in kept:
                    if w >= 0:
                        two.update(int(x) for x in before[w] if x >= 0)
            free = []
            for i in range(C):
                v = int(cand[u, i])
                taken = v < 0 or v == u or (kept == v).any()
                if not taken and not (rule == "bridge" and v in two):
                    free.append(i)
            if rule == "far":
                free = free[::-1]
            empty = [k for k in range(W) if kept[k] < 0]
            for t in range(min(len(free), len(empty))):
                out[u, empty[t]] = cand[u, free[t]]
    return out


def enforce_min_in(G, cand, min_in, rounds=4):
    """build_graph.py:309-386.  Returns (G, per-round [below, to_place, placed,
    already_linked])."""
    G = G.copy()
    n, W = G.shape
    C = cand.shape[1]
    stats = []
    for _ in range(rounds):
        indeg = np.bincount(G[G >= 0], minlength=n).astype(np.int64)
        weak = np.nonzero(indeg < min_in)[0]
        if weak.size == 0:
            break
        remaining = np.zeros(n, np.int64)
        remaining[weak] = np.minimum(min_in - indeg[weak], C)
        row_stats = [int(weak.size), int(remaining.sum()), 0, 0]
        for i in range(C):
            sel = np.nonzero(remaining > 0)[0]
            if sel.size == 0:
                break
            winner = {}
            for s in sel:                       # ascending: the lowest source wins
                t = int(cand[s, i])
                if t < 0 or t == s:
                    continue
                if (G[t] == s).any():
                    row_stats[3] += 1
                    continue
                winner.setdefault(t, int(s))
            moves = []
            for t, s in winner.items():
                rich = [k for k in range(W) if G[t, k] >= 0 and indeg[G[t, k]] > min_in]
                if rich and rich[-1] >= 1:
                    moves.append((t, s, rich[-1]))
            if not moves:
                continue
            before = indeg.copy()
            for t, s, k in moves:               # a victim loses one in-edge, however often taken
                indeg[G[t, k]] = before[G[t, k]] - 1
            for t, s, k in moves:
                indeg[s] += 1
                G[t, k] = s
                remaining[s] -= 1
                row_stats[2] += 1
        stats.append(row_stats)
    return G, stats
