"""Shared helpers of the GPU parity tests: inputs to the device, and the
reference's own compiled kernels (oracle/_ref, swann/csrc/local_search.cu of
geniussyn/SWANN built unmodified for sm_100a) driven the way the reference's
swann/_engine.py drives them (init_states, then one advance of the budget)."""
import numpy as np
import torch

from oracle import oracle as O
from swann_b200 import _engine as E

DEV = "cuda"


def to_gpu(X, G, Qv):
    return (torch.from_numpy(np.ascontiguousarray(X)).to(DEV), torch.from_numpy(np.ascontiguousarray(G)).to(DEV),
            torch.from_numpy(np.ascontiguousarray(Qv)).to(DEV))


def ref_run(Xg, Gg, Qg, seeds, L, B, metric, team, policy=0, stop_eps=-1.0, kstop=10, V=None, stall=0,
            crowd=0.0):
    """The reference's own init_states + advance, deterministic mode (the
    stall and crowd rules as given)."""
    R = O.ref_kernels()
    if R is None:
        return None
    seeds = seeds.to(DEV, torch.int32).contiguous()
    if seeds.dim() == 2:
        seeds = seeds.unsqueeze(-1).contiguous()
    Q, J, V = seeds.shape
    H = E.visited_size(B, Gg.shape[1])
    ids = torch.empty((Q, J, L), dtype=torch.int32, device=DEV)
    dist = torch.empty((Q, J, L), dtype=torch.float32, device=DEV)
    expd = torch.empty((Q, J, L), dtype=torch.uint8, device=DEV)
    lin = torch.empty((Q, J, L), dtype=torch.uint8, device=DEV)
    vis = torch.empty((Q, J, H), dtype=torch.int32, device=DEV)
    ctr = torch.empty((Q, J, 10), dtype=torch.int32, device=DEV)
    ei = torch.empty((0, 0), dtype=torch.int32, device=DEV)
    ef = torch.empty((0, 0), dtype=torch.float32, device=DEV)
    eb = torch.empty((0,), dtype=torch.float32, device=DEV)
    R.init_states(Xg, Qg, seeds, ids, dist, expd, lin, vis, ctr, metric, team, ei, ef, eb)
    e0i = torch.empty(0, dtype=torch.int32, device=DEV)
    e0f = torch.empty(0, dtype=torch.float32, device=DEV)
    R.advance(Xg, Gg, Qg, ids, dist, expd, lin, vis, ctr, metric, team, B, B, policy, V, float(stop_eps), kstop,
              ei, ef, eb, 0, int(stall), float(crowd), e0i, e0i, e0f, e0f, 0.0)
    torch.cuda.synchronize()
    return ids, dist, expd, lin, ctr


def same_state(st, ref, counters=(0, 1, 2, 3, 8, 9)):
    ids, dist, expd, lin, ctr = ref
    assert torch.equal(st.ids, ids)
    assert torch.equal(st.dist.view(torch.int32), dist.view(torch.int32))
    assert torch.equal(st.expanded, expd)
    assert torch.equal(st.lineage, lin)
    for c in counters:
        assert torch.equal(st.counters[..., c], ctr[..., c]), f"counter {c}"


def ref_production(Xg, Gg, Qg, seeds, k=10, L=12, B=64, metric=0, team=16, stop_eps=0.05):
    """The reference's production search (swann/index.py:105-109 through
    swann/_engine.py:428-447): shared table at the reference's sizing
    (cache_size), shared bound, exclusive claims, per-branch visited tables
    elided, then branch_topk and the merge -- on the reference's own kernels.
    Returns (ids [Q, k], dist [Q, k]) on the device, or None without them."""
    R = O.ref_kernels()
    if R is None:
        return None
    seeds = seeds.to(DEV, torch.int32).contiguous()
    Qn, J = seeds.shape
    Hc = E.cache_size(J, B, Gg.shape[1])
    ids = torch.empty((Qn, J, L), dtype=torch.int32, device=DEV)
    dist = torch.empty((Qn, J, L), dtype=torch.float32, device=DEV)
    expd = torch.empty((Qn, J, L), dtype=torch.uint8, device=DEV)
    lin = torch.empty((Qn, J, L), dtype=torch.uint8, device=DEV)
    vis = torch.empty((Qn, J, 1), dtype=torch.int32, device=DEV)
    ctr = torch.empty((Qn, J, 10), dtype=torch.int32, device=DEV)
    cid = torch.empty((Qn, Hc), dtype=torch.int32, device=DEV)
    cdd = torch.empty((Qn, Hc), dtype=torch.float32, device=DEV)
    bnd = torch.empty((Qn,), dtype=torch.float32, device=DEV)
    s3 = seeds.unsqueeze(-1).contiguous()
    R.init_states(Xg, Qg, s3, ids, dist, expd, lin, vis, ctr, metric, team, cid, cdd, bnd)
    e0 = torch.empty(0, dtype=torch.int32, device=DEV)
    e0f = torch.empty(0, dtype=torch.float32, device=DEV)
    R.advance(Xg, Gg, Qg, ids, dist, expd, lin, vis, ctr, metric, team, B, B, 0, 1, float(stop_eps), k, cid, cdd,
              bnd, 1, 0, 0.0, e0, e0, e0f, e0f, 0.0)
    kk = min(k, L)
    ri, rd = R.merge_branches(ids[..., :kk].contiguous(), dist[..., :kk].contiguous(), k)
    torch.cuda.synchronize()
    return ri, rd


def recall(got, truth, k):
    got, truth = np.asarray(got), np.asarray(truth)
    return float(np.mean([len(set(a[:k].tolist()) & set(b[:k].tolist())) / k for a, b in zip(got, truth)]))
