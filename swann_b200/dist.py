"""One process per GPU: query-sharded search and row-block-sharded build.

Search.  Queries are independent, so a batch is cut into contiguous shards,
one per rank, each searched against that rank's full replica of the corpus,
graph and catalogue.  Nothing is exchanged while searching; the results are
gathered afterwards in rank order (which is query order).

Build.  Rank r owns rows [r*n/W, (r+1)*n/W).  The corpus tiles are
all-gathered once (each rank then holds every row, as the sweep needs), each
rank sweeps and prunes its own rows, the pruned rows are all-gathered so every
rank can see every edge for the reverse pass, each rank merges and re-prunes
its own rows, and a final all-gather assembles the graph.  With NCCL these are
NVLink all-gathers; the same code runs over gloo on CPU for testing.

The per-rank compute is passed in as callables, so the same driver runs the
B200 kernels (swann_b200.build) or, in tests, the CPU oracle.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_bounds(n: int, world: int):
    """Contiguous [start, end) of each of `world` shards of n items."""
    return [(n * r // world, n * (r + 1) // world) for r in range(world)]


def _gather_rows(local: torch.Tensor, n_total: int, world: int, group=None) -> torch.Tensor:
    """All-gather row blocks of possibly unequal length into [n_total, ...]."""
    bounds = shard_bounds(n_total, world)
    width = max(b - a for a, b in bounds)
    pad = torch.zeros((width,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[:local.shape[0]] = local
    out = torch.empty((world * width,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, pad, group=group)
    parts = [out[r * width: r * width + (b - a)] for r, (a, b) in enumerate(bounds)]
    return torch.cat(parts, 0)


def search_sharded(search_fn, Q: torch.Tensor, k: int, group=None):
    """Every rank passes the same full batch Q; rank r searches its shard with
    search_fn(Q_shard) -> (ids [m, k] int32, dist [m, k] float32) on its own
    device, and every rank returns the whole batch's results in query order."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    a, b = shard_bounds(Q.shape[0], world)[rank]
    ids, dd = search_fn(Q[a:b])
    ids = _gather_rows(ids.to(torch.int32), Q.shape[0], world, group)
    dd = _gather_rows(dd.float(), Q.shape[0], world, group)
    return ids, dd


def build_sharded(X_local: torch.Tensor, n: int, sweep_fn, prune_fn, reverse_fn, group=None):
    """Row-block build.  X_local holds this rank's rows of the corpus.

      sweep_fn(X, r0, r1)          -> (cand [r1-r0, C] int32, cdist float32)
      prune_fn(X, cand, cdist)     -> [r1-r0, deg] int32
      reverse_fn(X, G, r0, r1)     -> [r1-r0, deg] int32 (rows r0..r1 of the
                                      reverse pass over the full graph G)
    Returns (X, G): the full corpus and the full graph on every rank."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    r0, r1 = shard_bounds(n, world)[rank]
    X = _gather_rows(X_local, n, world, group)
    cand, cdist = sweep_fn(X, r0, r1)
    G1_local = prune_fn(X, cand, cdist)
    G1 = _gather_rows(G1_local, n, world, group)
    G2_local = reverse_fn(X, G1, r0, r1)
    G = _gather_rows(G2_local, n, world, group)
    return X, G
