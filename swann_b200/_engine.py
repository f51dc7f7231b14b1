"""The search engine's host layer: resumable per-branch state over the sm_100a kernels.

Drop-in for swann/_engine.py (geniussyn/SWANN): the same functions, knobs,
constants and SearchState, with the same semantics --

  queue      best-L over everything evaluated so far, sorted by (distance, id),
             with the `expanded` flag carried along by every merge;
  stop       budget spent, or no retained candidate left unexpanded;
  budget     node expansions per branch (distance evaluations are counted
             separately);
  resume     advance(a) then advance(b) == advance(a + b).

Every computation runs in libswann_b200.so (swann_b200/csrc); this module only
sizes and allocates the caller-owned state tensors and passes their pointers.
`search` runs the fused kernel (init, walk, per-branch top-k and the merge in
one launch) whenever no chunking or active list is asked for.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _lib as N

POLICY_BEST = 0          # expand the nearest unexpanded candidate, always
POLICY_ROUND_ROBIN = 1   # give each seed lineage its turn

METRIC_IP = 0   # distance = 1 - dot. Vectors must be L2-normalised.
METRIC_L2 = 1   # distance = ||q - x||^2
NCTR = 10       # expansions, distance evals, hash failures, exhausted, cache hits,
                # cache slots claimed, stalled, crowded, fan-out sum, fan-out count


def ext():
    """The loaded native library (the reference returns its torch extension)."""
    return N.lib()


def next_pow2(x: int) -> int:
    n = 1
    while n < x:
        n <<= 1
    return n


def visited_size(B: int, D: int) -> int:
    """Per-branch visited table: load factor <= 0.5 even if every expansion
    inserts D new nodes (swann/_engine.py:73-77)."""
    return next_pow2(2 * (1 + B * D))


def cache_size(J, B, D, share=4.0, cap=1 << 20):
    """Slots of the per-query distance table, sized for what J branches of B
    expansions touch together given an overlap factor `share`
    (swann/_engine.py:186-198).  A bounded probe that finds no room only costs
    a recomputation."""
    want = 2 * (1 + J * (1 + B * D) / share)
    return min(next_pow2(int(want)), cap)


@dataclass
class SearchState:
    """Everything a branch needs to be stopped and resumed, and nothing else."""
    ids: torch.Tensor        # int32  [Q, J, L]  -1 = empty slot
    dist: torch.Tensor       # float32[Q, J, L]
    expanded: torch.Tensor   # uint8  [Q, J, L]
    lineage: torch.Tensor    # uint8  [Q, J, L]
    visited: torch.Tensor    # int32  [Q, J, H]  H == 1: switched off
    counters: torch.Tensor   # int32  [Q, J, NCTR]
    B: int
    metric: int
    team_size: int
    V: int = 1
    policy: int = POLICY_BEST
    stop_eps: float = -1.0
    stall_patience: int = 0
    crowd_frac: float = 0.0
    kstop: int = 10
    # Per-query distance table [Q, Hc] as int64 words: (id + 1) << 32 | float
    # bits of the distance.  Empty = off.  Shared by a query's branches.
    cache: torch.Tensor = None
    # Per-query k-th-best bound [Q]; empty = off.
    bound: torch.Tensor = None
    # 1: skip nodes another branch has scored (the reference's rule); 2: also
    # skip nodes another branch has claimed but not yet scored; 0: off
    exclusive: int = 0
    # int32 [1] device status word: a device wait that gave up writes
    # SWB_ERR_TIMEOUT here
    status: torch.Tensor = None

    @property
    def shape(self):
        return tuple(self.ids.shape)

    @property
    def cache_id(self) -> torch.Tensor:
        """id + 1 of each table slot (0 = empty), as the reference stores it."""
        if self.cache is None or self.cache.numel() == 0:
            return torch.empty((0, 0), dtype=torch.int32, device=self.ids.device)
        return (self.cache >> 32).to(torch.int32)

    @property
    def cache_d(self) -> torch.Tensor:
        """Distance held by each table slot (FLT_MAX = claimed, not yet scored)."""
        if self.cache is None or self.cache.numel() == 0:
            return torch.empty((0, 0), dtype=torch.float32, device=self.ids.device)
        return (self.cache & 0xFFFFFFFF).to(torch.int32).view(torch.float32)

    @property
    def expansions(self):
        return self.counters[..., 0]

    @property
    def dist_evals(self):
        return self.counters[..., 1]

    @property
    def hash_failures(self):
        return self.counters[..., 2]

    @property
    def exhausted(self):
        return self.counters[..., 3]

    @property
    def cache_hits(self):
        return self.counters[..., 4]

    @property
    def slots_claimed(self):
        return self.counters[..., 5]

    @property
    def stalled(self):
        return self.counters[..., 6]

    @property
    def crowded(self):
        return self.counters[..., 7]

    @property
    def fanout(self):
        return self.counters[..., 8], self.counters[..., 9]

    def check(self):
        """Raise if the visited table overflowed (nodes were dropped) or a
        device-side wait gave up.  Synchronises (reads a count back)."""
        nf = int(self.hash_failures.sum())
        if nf:
            raise RuntimeError(
                f"visited table overflowed on {int((self.hash_failures > 0).sum())} branches "
                f"({nf} failed inserts): raise max_expansions used for sizing, or the table size")
        if self.status is not None and int(self.status[0]) != 0:
            raise N.SwannError(int(self.status[0]), "a device-side wait timed out during the search")

    def overflow(self) -> torch.Tensor:
        """The overflow count, left on the device (no synchronisation)."""
        return self.hash_failures.sum()

    def clone(self) -> "SearchState":
        def c(t):
            return None if t is None else t.clone()
        return SearchState(ids=c(self.ids), dist=c(self.dist), expanded=c(self.expanded),
                           lineage=c(self.lineage), visited=c(self.visited), counters=c(self.counters),
                           B=self.B, metric=self.metric, team_size=self.team_size, V=self.V,
                           policy=self.policy, stop_eps=self.stop_eps, stall_patience=self.stall_patience,
                           crowd_frac=self.crowd_frac, kstop=self.kstop, cache=c(self.cache),
                           bound=c(self.bound), exclusive=self.exclusive, status=c(self.status))


_OVERFLOW_GUARD = True


def overflow_guard(on: bool) -> bool:
    """Turn the per-search overflow check (a host synchronisation) on or off.
    Returns the old setting (swann/_engine.py:203-216)."""
    global _OVERFLOW_GUARD
    was, _OVERFLOW_GUARD = _OVERFLOW_GUARD, bool(on)
    return was


def _check_inputs(X, Qv):
    if not (X.is_cuda and X.dtype in (torch.float32, torch.float16) and X.is_contiguous()):
        raise ValueError("X: contiguous cuda float32 or float16")
    if not (Qv.is_cuda and Qv.dtype == torch.float32 and Qv.is_contiguous()):
        raise ValueError("Q: contiguous cuda float32")


def _empty(dtype, dev, shape=(0,)):
    return torch.empty(shape, dtype=dtype, device=dev)


def _alloc_state(X, Q, J, L, V, B, D, metric, team_size, policy, stop_eps, kstop, shared_cache,
                 shared_bound, exclusive, stall_patience, crowd_frac, elide_visited):
    elide = bool(elide_visited and exclusive and shared_cache and J > 1 and V == 1)
    H = 1 if elide else visited_size(B, D)
    dev = X.device
    st = SearchState(
        ids=torch.empty((Q, J, L), dtype=torch.int32, device=dev),
        dist=torch.empty((Q, J, L), dtype=torch.float32, device=dev),
        expanded=torch.empty((Q, J, L), dtype=torch.uint8, device=dev),
        lineage=torch.empty((Q, J, L), dtype=torch.uint8, device=dev),
        visited=torch.empty((Q, J, H), dtype=torch.int32, device=dev),
        counters=torch.empty((Q, J, NCTR), dtype=torch.int32, device=dev),
        B=B, metric=metric, team_size=team_size, V=V, policy=policy, stop_eps=float(stop_eps),
        kstop=int(kstop), stall_patience=int(stall_patience), crowd_frac=float(crowd_frac),
    )
    if shared_cache and J > 1:
        st.cache = torch.empty((Q, cache_size(J, B, D)), dtype=torch.int64, device=dev)
    else:
        st.cache = _empty(torch.int64, dev, (0, 0))
    st.exclusive = int(exclusive) if (shared_cache and J > 1) else 0
    st.bound = (torch.empty((Q,), dtype=torch.float32, device=dev) if (shared_bound and J > 1)
                else _empty(torch.float32, dev))
    st.status = torch.zeros((1,), dtype=torch.int32, device=dev)
    return st


def _seeds3(seeds, dev):
    seeds = seeds.to(device=dev, dtype=torch.int32).contiguous()
    if seeds.dim() == 2:
        seeds = seeds.unsqueeze(-1).contiguous()
    return seeds


def init_states(X, Qv, seeds, L=16, B=16, D=None, metric=METRIC_IP, team_size=32, policy=POLICY_BEST,
                stop_eps=-1.0, kstop=10, shared_cache=False, shared_bound=False, exclusive=False,
                stall_patience=0, crowd_frac=0.0, elide_visited=False) -> SearchState:
    """One state per (query, branch); `seeds` is int32 [Q, J] (one entry per
    branch) or [Q, J, V] (V entries sharing one branch), -1 = empty."""
    _check_inputs(X, Qv)
    if D is None:
        raise ValueError("D (the graph out-degree) is required: it sizes the visited table")
    seeds = _seeds3(seeds, X.device)
    Q, J, V = seeds.shape
    st = _alloc_state(X, Q, J, L, V, B, D, metric, team_size, policy, stop_eps, kstop, shared_cache,
                      shared_bound, exclusive, stall_patience, crowd_frac, elide_visited)
    H = st.visited.shape[2]
    Hc = st.cache.shape[1] if st.cache.numel() else 0
    with torch.cuda.device(X.device):
        rc = N.lib().swb_search_init(
            N.ptr(X), N.dtype_code(X), X.shape[0], X.shape[1], N.ptr(Qv), N.ptr(seeds), Q, J, V,
            N.ptr(st.ids), N.ptr(st.dist), N.ptr(st.expanded), N.ptr(st.lineage), L,
            N.ptr(st.visited), H, N.ptr(st.counters), int(metric), int(team_size),
            N.ptr(st.cache), Hc, N.ptr(st.bound), N.stream_of(X))
    N.check(rc, "init_states")
    return st


def advance(X, G, Qv, state: SearchState, delta_expansions: int, active=None, codes=None) -> SearchState:
    """Advance every branch (or the flattened q*J+j indices in `active`) by up
    to `delta_expansions` more expansions, in place."""
    _check_inputs(X, Qv)
    if not (G.is_cuda and G.dtype == torch.int32 and G.is_contiguous()):
        raise ValueError("G: contiguous cuda int32")
    code_args = (None, None, None, 0.0, 0)
    if codes is not None:
        code_args = _code_args(codes, X, state)
    Q, J, L = state.ids.shape
    H = state.visited.shape[2]
    Hc = state.cache.shape[1] if state.cache is not None and state.cache.numel() else 0
    n_active = 0
    if active is not None:
        active = active.to(device=X.device, dtype=torch.int32).contiguous()
        n_active = active.numel()
        if n_active == 0:
            return state
    with torch.cuda.device(X.device):
        rc = N.lib().swb_search_advance(
            N.ptr(X), N.dtype_code(X), X.shape[0], X.shape[1], N.ptr(G), G.shape[1], N.ptr(Qv),
            N.ptr(state.ids), N.ptr(state.dist), N.ptr(state.expanded), N.ptr(state.lineage), Q, J, L,
            N.ptr(state.visited), H, N.ptr(state.counters), int(state.metric), int(state.team_size),
            int(delta_expansions), int(state.B), int(state.policy), int(state.V), float(state.stop_eps),
            int(state.kstop), N.ptr(state.cache), Hc, N.ptr(state.bound), int(state.exclusive),
            int(state.stall_patience), float(state.crowd_frac), N.ptr(active), n_active,
            *code_args, N.ptr(state.status), N.stream_of(X))
    N.check(rc, "advance")
    return state


def _code_args(codes, X, state):
    """(codes, alpha, mu, margin) as load_codes returns them -> the ABI's five
    code arguments, checked (swann/csrc/local_search.cu:778-841 takes them as
    codes, alpha, cmu, margin)."""
    if state.metric != METRIC_IP:
        raise NotImplementedError("the sign-code prefilter is inner product only (local_search.cu:222-243)")
    cd, al, mu, margin = codes
    n, d = X.shape
    words = (d + 31) // 32
    cd = cd.to(device=X.device, dtype=torch.int32).contiguous()
    al = al.to(device=X.device, dtype=torch.float32).contiguous()
    mu = mu.to(device=X.device, dtype=torch.float32).contiguous()
    if tuple(cd.shape) != (n, words) or tuple(al.shape) != (n,) or tuple(mu.shape) != (d,):
        raise ValueError(f"codes must be [n, {words}] int32 with alpha [n] and mu [d]")
    return (N.ptr(cd), N.ptr(al), N.ptr(mu), float(margin), words)


def load_codes(data, name=None, margin=0.20, device="cuda"):
    """The sign code, its per-node scale and the corpus mean, as `advance` wants
    (swann/_engine.py:320-337): codes_<name>.npy, alpha_<name>.npy and
    mu_<name>.npy in a corpus directory, `name` from its manifest when not
    given.  `margin` is in the corpus's distance units and is set per corpus.
    `swann_b200.corpus.write_codes` writes these files."""
    import json
    from pathlib import Path
    d = Path(data)
    if name is None:
        man = json.loads((d / "manifest.json").read_text())
        name = "1bit" if man["metric"].startswith("ip") else "int8"
    cd = torch.from_numpy(np.load(d / f"codes_{name}.npy")).to(device)
    al = torch.from_numpy(np.load(d / f"alpha_{name}.npy")).to(device)
    cm = torch.from_numpy(np.load(d / f"mu_{name}.npy")).to(device)
    return cd.contiguous(), al.contiguous(), cm.contiguous(), margin


def branch_topk(state: SearchState, k: int):
    """Per-branch best-min(k, L), straight off the (sorted) queue."""
    kk = min(k, state.ids.shape[-1])
    return state.ids[..., :kk].clone(), state.dist[..., :kk].clone()


def merge_branches(ids: torch.Tensor, dist: torch.Tensor, k: int, fused: bool = True):
    """Branch results [Q, J, kk] -> one top-k per query, duplicates removed by
    id, padding (-1, +inf).  The kernel handles any shape whose sort fits in
    shared memory; the tensor definition serves the rest."""
    if fused and ids.is_cuda and ids.dim() == 3:
        ids = ids.contiguous().to(torch.int32)
        dist = dist.contiguous().float()
        Q, J, kk = ids.shape
        oi = torch.empty((Q, k), dtype=torch.int32, device=ids.device)
        od = torch.empty((Q, k), dtype=torch.float32, device=ids.device)
        with torch.cuda.device(ids.device):
            rc = N.lib().swb_merge_branches(N.ptr(ids), N.ptr(dist), Q, J, kk, k, N.ptr(oi), N.ptr(od),
                                            N.stream_of(ids))
        if rc == N.OK:
            return oi, od
        if rc != N.ERR_SMEM:
            N.check(rc, "merge_branches")
    return _merge_branches_tensor(ids, dist, k)


def _merge_branches_tensor(ids: torch.Tensor, dist: torch.Tensor, k: int):
    """The merge as tensor operations: sort by (distance, id), keep the first
    copy of each id, take k (the definition the kernels are checked against)."""
    Q = ids.shape[0]
    fi = ids.reshape(Q, -1).to(torch.int64)
    fd = dist.reshape(Q, -1).clone().float()
    fd[fi < 0] = float("inf")
    fi = torch.where(fi < 0, torch.full_like(fi, 2 ** 31 - 1), fi)
    o1 = torch.argsort(fi, dim=1, stable=True)
    fd, fi = torch.gather(fd, 1, o1), torch.gather(fi, 1, o1)
    o2 = torch.argsort(fd, dim=1, stable=True)
    fd, fi = torch.gather(fd, 1, o2), torch.gather(fi, 1, o2)
    dup = torch.zeros_like(fi, dtype=torch.bool)
    dup[:, 1:] = fi[:, 1:] == fi[:, :-1]
    keep = (~dup) & (fi != 2 ** 31 - 1)
    oi = torch.full((Q, k), -1, dtype=torch.int32, device=ids.device)
    od = torch.full((Q, k), float("inf"), dtype=torch.float32, device=ids.device)
    rank = torch.cumsum(keep.to(torch.int64), 1) - 1
    sel = keep & (rank < k)
    r, c = sel.nonzero(as_tuple=True)
    oi[r, rank[r, c]] = fi[r, c].to(torch.int32)
    od[r, rank[r, c]] = fd[r, c]
    return oi, od


def advance_chunked(X, G, Qv, state: SearchState, total: int, chunk: int, codes=None) -> int:
    """Advance in chunks, re-forming the grid over the branches still running.
    Returns the number of launches."""
    launches, spent = 0, 0
    while spent < total:
        alive = ((state.exhausted == 0) & (state.stalled == 0) &
                 (state.expansions < state.B)).reshape(-1).nonzero().squeeze(1)
        if alive.numel() == 0:
            break
        step = min(chunk, total - spent)
        advance(X, G, Qv, state, step, active=alive.to(torch.int32).contiguous(), codes=codes)
        spent += step
        launches += 1
    return launches


class Workspace:
    """Per-device scratch of the fused search, grown on demand and reused."""

    def __init__(self):
        self.bufs = {}

    def get(self, name, numel, dtype, device):
        key = (name, str(device))
        t = self.bufs.get(key)
        if t is None or t.numel() < numel or t.dtype != dtype:
            t = torch.empty(max(numel, 1), dtype=dtype, device=device)
            self.bufs[key] = t
        return t[:numel]


_WS = Workspace()


def prepare_lean(Q, J, B, D, dev, stream, table_slots=None, shared_cache=True, shared_bound=True):
    """Clears what a query's branches share -- the per-query tables, bounds and
    completion counters of the lean workspace -- for a following
    search_fused_lean(..., prepared=True) of Q queries and J branches, on
    `stream`, so the clear can run beside other work (the seed selection).  The
    caller orders that search after this stream's work (an event)."""
    Hc = table_slots or cache_size(J, B, D)
    shared = J > 1
    cache = (_WS.get("cache", Q * Hc, torch.int64, dev).view(Q, -1)
             if (shared_cache and shared) else _empty(torch.int64, dev, (0, 0)))
    bound = _WS.get("bound", Q, torch.float32, dev) if (shared_bound and shared) else _empty(torch.float32, dev)
    qdone = _WS.get("qdone", Q, torch.int32, dev)
    Hc = cache.shape[1] if cache.numel() else 0
    with torch.cuda.device(dev):
        N.check(N.lib().swb_search_prepare(Q, N.ptr(cache), Hc, N.ptr(bound), N.ptr(qdone), stream.cuda_stream),
                "search")


def _fused(X, G, Qv, seeds, k, L, B, metric, team_size, policy, stop_eps, shared_cache, shared_bound,
           exclusive, stall_patience, crowd_frac, elide_visited, kstop, keep_state, table_slots=None,
           prepared=False):
    _check_inputs(X, Qv)
    if not (G.is_cuda and G.dtype == torch.int32 and G.is_contiguous()):
        raise ValueError("G: contiguous cuda int32")
    seeds = _seeds3(seeds, X.device)
    Q, J, V = seeds.shape
    dev = X.device
    kstop = k if kstop is None else kstop
    kk = min(k, L)
    D = G.shape[1]
    elide = bool(elide_visited and exclusive and shared_cache and J > 1 and V == 1)
    H = 1 if elide else visited_size(B, D)
    if keep_state:
        st = _alloc_state(X, Q, J, L, V, B, D, metric, team_size, policy, stop_eps, kstop, shared_cache,
                          shared_bound, exclusive, stall_patience, crowd_frac, elide_visited)
        visited, cache, bound, status, ctr = st.visited, st.cache, st.bound, st.status, st.counters
    else:
        st = None
        visited = _WS.get("visited", Q * J * H, torch.int32, dev) if H > 1 else _empty(torch.int32, dev)
        Hc = table_slots or cache_size(J, B, D)
        cache = (_WS.get("cache", Q * Hc, torch.int64, dev).view(Q, -1)
                 if (shared_cache and J > 1) else _empty(torch.int64, dev, (0, 0)))
        bound = _WS.get("bound", Q, torch.float32, dev) if (shared_bound and J > 1) else _empty(torch.float32, dev)
        status = torch.zeros((1,), dtype=torch.int32, device=dev)
        ctr = torch.empty((Q, J, NCTR), dtype=torch.int32, device=dev)
    excl = int(exclusive) if (shared_cache and J > 1) else 0
    Hc = cache.shape[1] if cache.numel() else 0
    bi = _WS.get("branch_ids", Q * J * kk, torch.int32, dev)
    bd = _WS.get("branch_dist", Q * J * kk, torch.float32, dev)
    qdone = _WS.get("qdone", Q, torch.int32, dev)
    oi = torch.empty((Q, k), dtype=torch.int32, device=dev)
    od = torch.empty((Q, k), dtype=torch.float32, device=dev)
    lib = N.lib()
    with torch.cuda.device(dev):
        s = N.stream_of(X)
        if not prepared:
            N.check(lib.swb_search_prepare(Q, N.ptr(cache), Hc, N.ptr(bound), N.ptr(qdone), s), "search")
        rc = lib.swb_search_fused(
            N.ptr(X), N.dtype_code(X), X.shape[0], X.shape[1], N.ptr(G), D, N.ptr(Qv), N.ptr(seeds),
            Q, J, V, k, L, B, int(metric), int(team_size), int(policy), float(stop_eps), int(kstop),
            N.ptr(visited), H, N.ptr(cache), Hc, N.ptr(bound), int(excl), int(stall_patience),
            float(crowd_frac), N.ptr(bi), N.ptr(bd), N.ptr(qdone), N.ptr(oi), N.ptr(od),
            N.ptr(st.ids) if st else None, N.ptr(st.dist) if st else None,
            N.ptr(st.expanded) if st else None, N.ptr(st.lineage) if st else None,
            N.ptr(ctr), N.ptr(status), s)
    N.check(rc, "search")
    return oi, od, st, ctr, status


def search_fused(X, G, Qv, seeds, k=10, L=16, B=16, metric=METRIC_IP, team_size=32, policy=POLICY_BEST,
                 stop_eps=-1.0, shared_cache=False, shared_bound=False, exclusive=False, stall_patience=0,
                 crowd_frac=0.0, elide_visited=False, kstop=None):
    """init -> advance(B) -> branch_topk -> merge as one kernel launch (plus one
    clearing launch for what a query's branches share).  Returns
    (ids, dist, state) with the final per-branch state."""
    oi, od, st, _, _ = _fused(X, G, Qv, seeds, k, L, B, metric, team_size, policy, stop_eps, shared_cache,
                              shared_bound, exclusive, stall_patience, crowd_frac, elide_visited, kstop, True)
    return oi, od, st


def search_fused_lean(X, G, Qv, seeds, k=10, L=16, B=16, metric=METRIC_IP, team_size=32, policy=POLICY_BEST,
                      stop_eps=-1.0, shared_cache=False, shared_bound=False, exclusive=False, stall_patience=0,
                      crowd_frac=0.0, elide_visited=False, kstop=None, table_slots=None, prepared=False):
    """The fused search writing only results, counters [Q, J, NCTR] and the
    status word (the path Index.search runs).  `table_slots` overrides the
    per-query table size (a power of two); `prepared`: the shared state was
    already cleared by prepare_lean (same Q, J, B, D, table_slots), ordered
    before this call.  Returns (ids, dist, ctr, status)."""
    oi, od, _, ctr, status = _fused(X, G, Qv, seeds, k, L, B, metric, team_size, policy, stop_eps, shared_cache,
                                    shared_bound, exclusive, stall_patience, crowd_frac, elide_visited, kstop,
                                    False, table_slots, prepared)
    return oi, od, ctr, status


def search(X, G, Qv, seeds, k=10, L=16, B=16, metric=METRIC_IP, team_size=32, policy=POLICY_BEST,
           stop_eps=-1.0, shared_cache=False, shared_bound=False, exclusive=False, stall_patience=0,
           crowd_frac=0.0, elide_visited=False, chunk=0, codes=None):
    """init -> advance(budget) -> per-branch best-k -> merged top-k.  One shot."""
    if chunk or codes is not None:
        st = init_states(X, Qv, seeds, L=L, B=B, D=G.shape[1], metric=metric, team_size=team_size,
                         policy=policy, stop_eps=stop_eps, kstop=k, shared_cache=shared_cache,
                         shared_bound=shared_bound, exclusive=exclusive, stall_patience=stall_patience,
                         crowd_frac=crowd_frac, elide_visited=elide_visited)
        if chunk:
            advance_chunked(X, G, Qv, st, B, chunk, codes=codes)
        else:
            advance(X, G, Qv, st, B, codes=codes)
        if _OVERFLOW_GUARD:
            st.check()
        bi, bd = branch_topk(st, k)
        ids, dist = merge_branches(bi, bd, k)
        return ids, dist, st
    ids, dist, st = search_fused(X, G, Qv, seeds, k=k, L=L, B=B, metric=metric, team_size=team_size,
                                 policy=policy, stop_eps=stop_eps, shared_cache=shared_cache,
                                 shared_bound=shared_bound, exclusive=exclusive,
                                 stall_patience=stall_patience, crowd_frac=crowd_frac,
                                 elide_visited=elide_visited)
    if _OVERFLOW_GUARD:
        st.check()
    return ids, dist, st
