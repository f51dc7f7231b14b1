"""The public interface: build an index over vectors, then search it.

Drop-in for swann/index.py (geniussyn/SWANN):

    import swann_b200 as swann
    index = swann.Index.build(X, metric="ip")      # X: (n, d) float32 / float16
    ids, dist = index.search(Q, k=10)

Same constructor, `build`, `search(queries, k, config, **overrides)`, `save`,
`load`, `SearchConfig` defaults and errors.  One addition: `devices=[...]`
replicates the corpus, graph and catalogue on several GPUs and splits each
query batch across them -- queries are independent, so the shards need no
communication and the results come back in input order.  A device-resident
batch is split by locality (`Index.route`: each shard one stretch of the
catalogue's tour); a host batch in contiguous slices.
"""
from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

from . import _engine as E
from . import _select as S

METRICS = {"ip": E.METRIC_IP, "l2": E.METRIC_L2}
MAX_BATCH = 65535
# Bytes of per-query distance tables one launch may use; larger batches are
# searched in consecutive chunks on the same stream.
TABLE_BUDGET = 24 << 30
# host batches larger than this are copied in chunks that overlap the seed selection
COPY_CHUNK = 8192
# blocks of at least this many queries are searched in locality order (below)
LOCALITY_MIN = 1024
# ... and have their shared tables cleared on a side stream during the seed selection
PREPARE_AHEAD_MIN = 1024


@dataclass
class SearchConfig:
    """Knobs, with the reference's defaults (swann/index.py:26-45).

    branches  trajectories one query is split into (warps of the GPU).
    queue     width of each branch's candidate queue.
    budget    cap on expansions per branch; `stop_eps` usually binds first.
    stop_eps  stop a branch once its best candidate is worse than the query's
              current k-th answer by this fraction; negative disables it.
    team      lanes cooperating on one distance (fixes the summation order).
    """
    branches: int = 32
    queue: int = 12
    budget: int = 64
    stop_eps: float = 0.05
    team: int = 16
    k: int = 10


class _Replica:
    """What one GPU holds: the corpus, the graph, the catalogue and its rows."""

    def __init__(self, X, G, catalogue, dev):
        self.dev = dev
        self.X = X if X.device == dev else X.to(dev)
        self.G = G if G.device == dev else G.to(dev)
        self.catalogue = catalogue if catalogue.device == dev else catalogue.to(dev)
        # gather the P catalogue rows first, then widen them: no fp32 copy of
        # the whole corpus (the values are the same either way)
        self.cat_rows = S.pool_vectors(self.X, self.catalogue).float()


class Index:
    """A proximity graph plus the vectors it indexes, resident on one or more GPUs."""

    def __init__(self, vectors: torch.Tensor, graph: torch.Tensor, metric: str = "ip",
                 catalogue: torch.Tensor | None = None, catalogue_size: int = 4096, seed: int = 0,
                 devices=None, table_slots: int | None = None, locality: bool = True):
        if vectors.device.type != "cuda":
            raise ValueError("vectors must already be on the GPU")
        if vectors.dtype not in (torch.float32, torch.float16):
            raise ValueError("vectors must be float32 or float16")
        if metric not in METRICS:
            raise ValueError(f"metric must be one of {sorted(METRICS)}")
        vec = 8 if vectors.dtype == torch.float16 else 4
        if vectors.shape[1] % vec:
            raise ValueError(f"the dimension must be a multiple of {vec} for {vectors.dtype} vectors "
                             "(the kernels read 16-byte row chunks); pad the vectors with zeros")
        self.X = vectors.contiguous()
        self.G = graph.to(device=self.X.device, dtype=torch.int32).contiguous()
        self.metric = metric
        self._m = METRICS[metric]
        # Search a large block of queries in the order of their nearest catalogue
        # entry, so the queries running side by side walk the same part of the
        # graph and share its rows in L2; the answers go back in input order.
        # Queries are independent, so this changes when a query runs, not what
        # it computes.
        self.locality = bool(locality)
        if catalogue is None:
            n = self.X.shape[0]
            rng = np.random.default_rng(seed)
            pick = np.sort(rng.permutation(n)[:min(catalogue_size, n)])
            catalogue = torch.from_numpy(pick.astype(np.int64)).to(self.X.device)
        self.catalogue = catalogue.to(self.X.device)
        if devices is None:
            devs = [self.X.device]
        else:
            devs = [torch.device("cuda", d) if isinstance(d, int) else torch.device(d) for d in devices]
        self._replicas = [_Replica(self.X, self.G, self.catalogue, d) for d in devs]
        self._cat = self._replicas[0].cat_rows
        self._tour = _catalogue_tour(self._cat, self._m) if self.locality else None
        lm = _landmarks(self._cat, self._tour) if self._tour is not None else None
        for r in self._replicas:
            r.tour = None if self._tour is None else self._tour.to(r.dev)
            r.landmarks = None if lm is None else tuple(t.to(r.dev) for t in lm)
        # Slots of each query's distance table.  A power of two fixes it.
        # None (the default) sizes it from what the queries claim: the first
        # search of a configuration uses the reference's sizing
        # (swann/_engine.py:186-198, 131072 slots at 32 branches), and every
        # search records the most slots any of its queries claimed; later
        # searches of that configuration use TABLE_HEADROOM times that, a
        # power of two.  The table only ever holds the nodes a query's
        # branches score (a few thousand), and a probe run that finds no free
        # slot scores the row uncached, so the size moves the work and the
        # clearing cost, never what a result may be.
        if table_slots is not None and (table_slots < 2 or table_slots & (table_slots - 1)):
            raise ValueError("table_slots must be a power of two")
        self.table_slots = table_slots
        self._claims = {}        # (branches, budget, queue, stop_eps, degree) -> most claims per query
        self._pending = []       # claim counts still on their way to the host (overflow guard off)

    @property
    def devices(self):
        return [r.dev for r in self._replicas]

    # -- sharding by locality -------------------------------------------------
    def route(self, queries: torch.Tensor):
        """An order of a device-resident batch along the catalogue's locality
        tour (int64, on the queries' device), or None without a tour: equal
        contiguous slices of it are query shards whose members sit in one
        stretch of the tour.  Each query goes to its nearest of LANDMARKS
        catalogue entries spread evenly along the tour (a TF32 GEMM against
        them, the arithmetic select_nearest uses); ties keep input order.  A
        GPU searching such a shard walks a fraction of the graph with as many
        queries per region as one GPU searching the whole batch, so queries
        running side by side share rows in L2.  The order depends only on the
        batch and the index, so every process computing it gets the same one."""
        if self._tour is None or queries.shape[0] == 0:
            return None
        r = next((x for x in self._replicas if x.dev == queries.device), self._replicas[0])
        lm_rows, lm_keys, lm_norms = r.landmarks
        Q = queries.to(r.dev).float()
        with S.reduced_precision(True):
            sc = Q @ lm_rows.T
        near = torch.argmax(sc, dim=1) if self._m == METRICS["ip"] else torch.argmin(lm_norms[None, :] - 2.0 * sc, 1)
        order = torch.argsort(lm_keys[near], stable=True)
        return order.to(queries.device)

    # -- per-query table size ------------------------------------------------
    def table_slots_for(self, branches, budget, queue, stop_eps, degree) -> int:
        """Slots of the per-query table a search with these knobs runs with."""
        if self.table_slots is not None:
            return self.table_slots
        self._fold_pending()
        ref = E.cache_size(branches, budget, degree)
        seen = self._claims.get(_claims_key(branches, budget, queue, stop_eps, degree))
        if seen is None:
            return ref
        return min(ref, max(TABLE_MIN, E.next_pow2(int(TABLE_HEADROOM * seen))))

    def _note_claims(self, key, claims, host_value=None):
        """Record the most slots a query of one launch claimed: `host_value`
        when the caller already read it, else read later without a stall."""
        if host_value is not None:
            self._claims[key] = max(self._claims.get(key, 0), int(host_value))
            return
        buf = torch.empty((1,), dtype=torch.int64, pin_memory=True)
        buf.copy_(claims.reshape(1), non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(claims.device))
        self._pending.append((key, buf, ev))

    def _fold_pending(self):
        keep = []
        for key, buf, ev in self._pending:
            if ev.query():
                self._claims[key] = max(self._claims.get(key, 0), int(buf[0]))
            else:
                keep.append((key, buf, ev))
        self._pending = keep

    # -- construction ----------------------------------------------------
    @classmethod
    def build(cls, vectors, metric: str = "ip", degree: int = 96, candidates: int = 128,
              alpha: float = 1.2, **kw) -> "Index":
        """Build a graph over `vectors` on the GPU (exact sweep, prune, reverse)."""
        from .build import build_graph
        X = _as_cuda(vectors)
        G = build_graph(X, metric=metric, degree=degree, candidates=candidates, alpha=alpha)
        return cls(X, G, metric=metric, **kw)

    # -- search ----------------------------------------------------------
    def search(self, queries, k: int = 10, config: SearchConfig | None = None, **overrides):
        """Return (ids, distances), each (nq, k), as numpy arrays."""
        ids, dist = self.search_tensors(queries, k=k, config=config, **overrides)
        return ids.cpu().numpy(), dist.cpu().numpy()

    def search_tensors(self, queries, k: int = 10, config: SearchConfig | None = None, **overrides):
        """Like `search`, but returns torch tensors on the first device."""
        cfg = config or SearchConfig(k=k)
        for key, value in overrides.items():
            if not hasattr(cfg, key):
                raise TypeError(f"unknown search option {key!r}")
            setattr(cfg, key, value)
        nq = int(queries.shape[0])
        if nq > MAX_BATCH:
            raise ValueError(f"batch of {nq} exceeds the 65535 the kernel's grid allows; split it")
        reps = self._replicas
        bounds = np.linspace(0, nq, len(reps) + 1).astype(np.int64)
        host = queries if not isinstance(queries, torch.Tensor) or queries.device.type == "cpu" else None
        if host is not None and isinstance(host, np.ndarray):
            host = torch.from_numpy(np.ascontiguousarray(host))
        # Several GPUs and a device-resident batch: shards by locality (route);
        # host batches keep contiguous shards, each copied over its own GPU's link.
        order = self.route(queries) if (len(reps) > 1 and host is None) else None
        outs, checks = [], []
        landed = []   # host batches: an event after each replica's copies
        for r, (a, b) in zip(reps, zip(bounds[:-1], bounds[1:])):
            if b <= a:
                continue
            with torch.cuda.device(r.dev):
                Hc = self.table_slots_for(cfg.branches, cfg.budget, cfg.queue, cfg.stop_eps, r.G.shape[1])
                if host is not None and b - a > COPY_CHUNK:
                    # Host queries: copied chunk by chunk on a side stream; each
                    # chunk's seeds are selected as it lands (the copies overlap
                    # the selection when the host memory is pinned), then the
                    # block is searched as one, so its locality order spans the
                    # whole block.
                    comp = torch.cuda.current_stream(r.dev)
                    # the shared tables are cleared while the queries cross the link
                    prep = self._prepare_ahead(r, b - a, cfg, Hc)
                    side = self._copy_stream(r.dev)
                    buf = torch.empty((b - a, host.shape[1]), dtype=host.dtype, device=r.dev)
                    side.wait_stream(comp)   # buf's memory is ready on the search stream
                    ready = []
                    with torch.cuda.stream(side):
                        for c0 in range(0, b - a, COPY_CHUNK):
                            c1 = min(b - a, c0 + COPY_CHUNK)
                            buf[c0:c1].copy_(host[a + c0:a + c1], non_blocking=True)
                            ev = torch.cuda.Event()
                            ev.record(side)
                            ready.append((c0, c1, ev))
                    landed.append(ready[-1][2])
                    Qd = buf if buf.dtype == torch.float32 else None
                    ents = []
                    for c0, c1, ev in ready:
                        comp.wait_event(ev)
                        ents.append(S.select_nearest(buf[c0:c1].float().contiguous(), r.cat_rows, cfg.branches,
                                                     metric=self._m))
                    if Qd is None:
                        Qd = buf.float().contiguous()
                    self._search_part(r, Qd, k, cfg, Hc, outs, checks, ent=torch.cat(ents), prep=prep)
                else:
                    src = host if host is not None else queries
                    part = src[a:b] if order is None else src[order[a:b]]
                    Qd = part.to(r.dev, non_blocking=True).float().contiguous()
                    if host is not None:
                        ev = torch.cuda.Event()
                        ev.record(torch.cuda.current_stream(r.dev))
                        landed.append(ev)
                    self._search_part(r, Qd, k, cfg, Hc, outs, checks)
        # The caller may reuse its host buffer once this returns: wait for the
        # copies out of it (not for the search).
        for ev in landed:
            ev.synchronize()
        overflow = 0
        # The visited tables are elided whenever a query has more than one
        # branch (the claims table does their job), and then no insert can
        # fail: the overflow check has nothing to read, so it is not waited
        # for, and a caller's next batch can be queued behind this one.
        guard = E._OVERFLOW_GUARD and cfg.branches <= 1
        for r, ctr in checks:
            key = _claims_key(cfg.branches, cfg.budget, cfg.queue, cfg.stop_eps, r.G.shape[1])
            # the most table slots one query claimed (its branches' claims plus
            # their seeds), and the visited-table overflow count
            claims = (ctr[..., 5].to(torch.int64).sum(1) + ctr.shape[1]).max()
            if guard:
                fails, most = torch.stack([ctr[..., 2].to(torch.int64).sum(), claims]).tolist()
                overflow += fails
                self._note_claims(key, claims, host_value=most)
            else:
                self._note_claims(key, claims)
        if overflow:
            raise RuntimeError("visited table overflowed: raise the budget used for sizing")
        dev0 = reps[0].dev
        ids = torch.cat([o[0].to(dev0) for o in outs]) if outs else torch.empty((0, k), dtype=torch.int32)
        dist = torch.cat([o[1].to(dev0) for o in outs]) if outs else torch.empty((0, k))
        if order is not None:   # back to input order
            back = order.to(dev0)
            ids_in, dist_in = torch.empty_like(ids), torch.empty_like(dist)
            ids_in[back], dist_in[back] = ids, dist
            ids, dist = ids_in, dist_in
        return ids, dist

    def _prepare_ahead(self, r, nq, cfg, Hc):
        """When a block of `nq` queries runs as one launch: clear that launch's
        shared tables on a side stream, beside the work queued after this call
        (copies, seed selection), and return the event the launch waits on;
        None otherwise."""
        step = max(1, min(nq, TABLE_BUDGET // (8 * Hc)))
        if nq < PREPARE_AHEAD_MIN or step != nq:
            return None
        side = self._side_stream(r.dev, "prepare")
        side.wait_stream(torch.cuda.current_stream(r.dev))
        E.prepare_lean(nq, cfg.branches, cfg.budget, r.G.shape[1], r.dev, side, table_slots=Hc)
        prep = torch.cuda.Event()
        prep.record(side)
        return prep

    def _search_part(self, r, Qd, k, cfg, Hc, outs, checks, ent=None, prep=False):
        """Seed selection and the fused search of one device-resident block of
        queries, in table-budget sized launches (and locality order, see
        `locality`); appends (ids, dist) in input order to `outs` and each
        launch's (replica, counters) to `checks`.  `ent`: the seeds' catalogue
        indices when already selected; `prep`: the event of a `_prepare_ahead`
        already issued for this block (False: issue it here)."""
        nq = Qd.shape[0]
        step = max(1, min(nq, TABLE_BUDGET // (8 * Hc)))
        if prep is False:
            # the tables are cleared while the seeds are selected and sorted
            prep = self._prepare_ahead(r, nq, cfg, Hc)
        if ent is None:
            ent = S.select_nearest(Qd, r.cat_rows, cfg.branches, metric=self._m)
        seeds = r.catalogue[ent].to(torch.int32)
        order = self.locality_order(ent, r)
        if order is not None:
            Qd, seeds = Qd[order].contiguous(), seeds[order].contiguous()
        part = []
        for c0 in range(0, nq, step):
            c1 = min(nq, c0 + step)
            if prep is not None:
                torch.cuda.current_stream(r.dev).wait_event(prep)
            ids, dist, ctr, _ = _search_device(r, Qd[c0:c1], seeds[c0:c1], k, cfg, self._m, Hc,
                                               prepared=prep is not None)
            part.append((ids, dist))
            checks.append((r, ctr))
        ids = torch.cat([p[0] for p in part]) if len(part) > 1 else part[0][0]
        dist = torch.cat([p[1] for p in part]) if len(part) > 1 else part[0][1]
        if order is not None:
            back = torch.empty_like(order)
            back[order] = torch.arange(order.numel(), device=order.device)
            ids, dist = ids[back], dist[back]
        outs.append((ids, dist))

    def locality_order(self, ent, r=None):
        """The order a block of queries runs in (None: input order), from each
        query's selected catalogue entries `ent` [nq, E]: by the nearest entry's
        position on the catalogue's locality tour."""
        if not self.locality or ent.shape[0] < LOCALITY_MIN or ent.shape[1] == 0:
            return None
        tour = (r or self._replicas[0]).tour
        key = ent[:, 0] if tour is None else tour[ent[:, 0]]
        return torch.argsort(key, stable=True)

    def _copy_stream(self, dev):
        return self._side_stream(dev, "copy")

    def _side_stream(self, dev, role):
        streams = self.__dict__.setdefault("_side_streams", {})
        key = (torch.device(dev).index, role)
        if key not in streams:
            streams[key] = torch.cuda.Stream(device=dev)
        return streams[key]

    # -- persistence -----------------------------------------------------
    def save(self, path) -> None:
        """Write graph.npy, catalogue.npy and index.json (the reference's format)."""
        path = Path(path)
        path.mkdir(parents=True, exist_ok=True)
        np.save(path / "graph.npy", self.G.cpu().numpy())
        np.save(path / "catalogue.npy", self.catalogue.cpu().numpy())
        (path / "index.json").write_text(json.dumps(
            {"metric": self.metric, "n": int(self.X.shape[0]), "d": int(self.X.shape[1]),
             "degree": int(self.G.shape[1])}, indent=2))

    @classmethod
    def load(cls, path, vectors, **kw) -> "Index":
        path = Path(path)
        meta = json.loads((path / "index.json").read_text())
        X = _as_cuda(vectors)
        G = torch.from_numpy(np.load(path / "graph.npy")).to(X.device)
        cat = torch.from_numpy(np.load(path / "catalogue.npy")).to(X.device)
        return cls(X, G, metric=meta["metric"], catalogue=cat, **kw)

    def __repr__(self) -> str:
        n, d = self.X.shape
        return (f"Index(n={n:,}, d={d}, degree={self.G.shape[1]}, metric={self.metric!r}, "
                f"dtype={self.X.dtype}, devices={len(self._replicas)})")


# catalogues up to this size get a greedy walk over every entry (an O(P^2) pass,
# once); larger ones a two-level tour over TOUR_COARSE walked entries
TOUR_MAX = 16384
TOUR_COARSE = 4096
# measured-claims table sizing: slots = TABLE_HEADROOM x the most slots one query
# claimed so far, a power of two, at least TABLE_MIN (load <= 67% for the
# busiest query seen, ~15% for a typical one at C3)
TABLE_HEADROOM = 1.5
TABLE_MIN = 4096


# catalogue entries a batch is routed by when it is sharded over several GPUs
LANDMARKS = 256


def _landmarks(cat_rows, tour, count=LANDMARKS):
    """LANDMARKS catalogue entries spread evenly along the tour: their rows
    (fp32), their tour positions and their squared norms."""
    P = cat_rows.shape[0]
    by_pos = torch.argsort(tour.to(cat_rows.device))
    pick = by_pos[torch.linspace(0, P - 1, min(count, P), device=cat_rows.device).round().long()]
    rows = cat_rows[pick].float().contiguous()
    return rows, tour.to(cat_rows.device)[pick].contiguous(), (rows * rows).sum(1).contiguous()


def _claims_key(branches, budget, queue, stop_eps, degree):
    return (int(branches), int(budget), int(queue), float(stop_eps), int(degree))


def _catalogue_tour(cat_rows, metric):
    """Each catalogue entry's position on a locality tour of the catalogue
    (int64 [P]), or None for fewer than two entries: sorting queries by their
    nearest entry's position keeps queries whose entries are close -- not only
    equal -- side by side.  Up to TOUR_MAX entries the tour is a greedy
    nearest-neighbour walk over the whole catalogue (an O(P^2) pass, once).
    Beyond that, TOUR_COARSE entries spread over the catalogue are walked that
    way, every entry joins its nearest walked entry's cell, and the tour runs
    cell by cell along the coarse walk (entries of one cell in catalogue
    order): queries that share a cell, or start in neighbouring cells, run
    side by side."""
    P = cat_rows.shape[0]
    if P < 2:
        return None
    V = cat_rows.float()
    with torch.no_grad():
        if P <= TOUR_MAX:
            return torch.from_numpy(_greedy_walk(_entry_distances(V, V, metric).cpu().numpy()))
        pick = torch.linspace(0, P - 1, TOUR_COARSE, device=V.device).round().long()
        C = V[pick]
        cpos = torch.from_numpy(_greedy_walk(_entry_distances(C, C, metric).cpu().numpy())).to(V.device)
        cell = torch.empty(P, dtype=torch.int64, device=V.device)
        for s in range(0, P, 8192):
            cell[s:s + 8192] = cpos[_entry_distances(V[s:s + 8192], C, metric).argmin(1)]
        ids = torch.arange(P, device=V.device)
        order = torch.argsort(cell * P + ids)
        pos = torch.empty_like(order)
        pos[order] = ids
    return pos.cpu()


def _entry_distances(A, B, metric):
    """[len(A), len(B)] distances in the corpus metric (fp32 matmul: only an
    ordering heuristic depends on them)."""
    if metric == METRICS["ip"]:
        return 1.0 - A @ B.T
    return (A * A).sum(1)[:, None] - 2.0 * (A @ B.T) + (B * B).sum(1)[None, :]


def _greedy_walk(D):
    """Positions (int64 [P]) along a greedy nearest-neighbour walk from entry 0
    over the distance matrix D [P, P] (numpy)."""
    P = D.shape[0]
    pos = np.empty(P, np.int64)
    seen = np.zeros(P, bool)
    cur = 0
    for i in range(P):
        pos[cur] = i
        seen[cur] = True
        if i + 1 < P:
            row = np.where(seen, np.inf, D[cur])
            cur = int(np.argmin(row))
    return pos


def _search_device(r: _Replica, Qd, seeds, k, cfg, metric, table_slots, prepared=False):
    """The fused search on one replica: shared table, bound and claims on,
    per-branch visited tables elided (swann/index.py:105-109).

    Claims are strict (exclusive=2): a node another branch has claimed is
    skipped even while its distance is still being computed.  The reference
    rescores such a node (local_search.cu:553-556); there the window is one
    team's distance computation, but a warp here claims a whole expansion at
    once and scores it through a pipeline, so the literal rule would let
    branches retread each other's ground far more often than the reference
    does.  Strict claims keep recall within 0.002 of the reference kernel's
    on the same graph and seeds, with fewer expansions."""
    return E.search_fused_lean(
        r.X, r.G, Qd, seeds, k=k, L=cfg.queue, B=cfg.budget, metric=metric, team_size=cfg.team,
        stop_eps=cfg.stop_eps, shared_cache=True, shared_bound=True, exclusive=2, elide_visited=True,
        table_slots=table_slots, prepared=prepared)


def _as_cuda(a) -> torch.Tensor:
    if isinstance(a, np.ndarray):
        a = torch.from_numpy(np.ascontiguousarray(a))
    if a.device.type != "cuda":
        a = a.cuda()
    return a.contiguous()
