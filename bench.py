#!/usr/bin/env python
"""SWANN on B200: QPS at recall@10 >= 0.95, HBM roofline, build seconds.

Workload (the north star's headline): n = 1,000,000 rows,
d = 1536, drawn from 1,000 anisotropic Gaussian clusters (per-dimension scales
log-uniform in [0.1, 1]), rows L2-normalised and stored fp16; fp32 queries
normalised from the same mixture; inner product; k = 10; a batch of 65,535
queries per GPU per step; degree-64 graph (candidates 128, alpha 1.2) built by
this package's kernels.  Seeded synthetic data stands in for the corpora the
reference measured on.

A step is one Index.search of the batch.  The operating point (branches,
queue, stop_eps) is the fastest one whose recall@10 against exact fp32 ground
truth is >= 0.95, chosen before timing on a fixed subset of the batch.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
    torchrun --nproc-per-node N bench.py --gpus N ...   (one process per GPU)

Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CONFIGS = {
    # name: (n, d, clusters, dtype, metric, batch)
    "c3": dict(n=1_000_000, d=1536, clusters=1000, half=True, metric="ip", batch=65535, k=10,
               desc="C3: 1M x 1536 fp16 inner-product corpus, 1000 anisotropic clusters"),
    "c2": dict(n=1_000_000, d=960, clusters=100, half=False, metric="l2", batch=10000, k=10,
               desc="C2: 1M x 960 fp32 L2 corpus, 100-component isotropic mixture (sigma 0.3)"),
    "c1": dict(n=10_000, d=128, clusters=0, half=False, metric="l2", batch=100, k=10,
               desc="C1: 10k x 128 fp32 N(0,1) L2 corpus (CPU-runnable case)"),
    "small": dict(n=100_000, d=256, clusters=100, half=True, metric="ip", batch=8192, k=10,
                  desc="small: 100k x 256 fp16 inner-product corpus (smoke-scale)"),
    # wide-dim large corpus, k = 100, queue 16, branches 64
    # 10,000 well-separated clusters make the exact-candidate graph one component per
    # cluster, so every cluster needs catalogue entries: 131072 (the reference's
    # large-catalogue setting, swann/_select.py:93-106) rather than 4096
    "c4": dict(n=10_000_000, d=768, clusters=10000, half=True, metric="ip", batch=50000, k=100,
               ladder=[(64, 16)], catalogue=131072,
               desc="C4: 10M x 768 fp16 inner-product corpus, 10000 anisotropic clusters, k 100"),
    "c4s": dict(n=200_000, d=768, clusters=1000, half=True, metric="ip", batch=4096, k=100, ladder=[(64, 16)],
                desc="C4-shaped small case: 200k x 768 fp16 inner product, k 100"),
    # the graph build benchmark (2M x 1024 fp32, L2)
    "c5": dict(n=2_000_000, d=1024, clusters=1000, half=False, metric="l2", batch=0, k=10,
               desc="C5: 2M x 1024 fp32 L2 corpus, 1000-component mixture (sigma 0.3)"),
    # small build shapes for ncu captures (fp16 IP and fp32 L2)
    "b16s": dict(n=100_000, d=1536, clusters=200, half=True, metric="ip", batch=0, k=10,
                 desc="build profiling case: 100k x 1536 fp16 inner product"),
    "b32s": dict(n=100_000, d=1024, clusters=100, half=False, metric="l2", batch=0, k=10,
                 desc="build profiling case: 100k x 1024 fp32 L2"),
    # C3-shaped profiling case: same row width and mixture model, a corpus
    # (0.6 GB) still larger than L2, small enough for an ncu capture
    "c3s": dict(n=200_000, d=1536, clusters=200, half=True, metric="ip", batch=4096, k=10,
                desc="C3-shaped profiling case: 200k x 1536 fp16 inner product, 200 clusters"),
}
LADDER = [(32, 12), (32, 16), (64, 16), (64, 24), (128, 32)]
EPS = [0.0, 0.01, 0.02, 0.05, 0.08, 0.12, 0.2, 0.3]   # the reference grid (reproduce.sh) plus 0
TARGET = 0.95


# ---------------------------------------------------------------------------
# synthetic data (seeded, generated on the device in chunks)

def gen_mixture(n, d, clusters, seed, dev, half, normalise, aniso=True, chunk=1 << 16, sigma=0.3):
    g = torch.Generator(device=dev)
    g.manual_seed(1234)   # the mixture itself is shared by corpus and queries
    if clusters:
        centres = torch.randn((clusters, d), generator=g, device=dev)
        if aniso:
            lo, hi = np.log(0.1), np.log(1.0)
            scales = torch.exp(lo + (hi - lo) * torch.rand((clusters, d), generator=g, device=dev))
        else:
            scales = torch.full((clusters, d), sigma, device=dev)
    gs = torch.Generator(device=dev)
    gs.manual_seed(seed)
    out = torch.empty((n, d), dtype=torch.float16 if half else torch.float32, device=dev)
    for a in range(0, n, chunk):
        b = min(n, a + chunk)
        z = torch.randn((b - a, d), generator=gs, device=dev)
        if clusters:
            c = torch.randint(0, clusters, (b - a,), generator=gs, device=dev)
            x = centres[c] + scales[c] * z
        else:
            x = z
        if normalise:
            x = x / x.norm(dim=1, keepdim=True)
        out[a:b] = x.to(out.dtype)
    return out


def make_corpus(cfg, dev):
    aniso = cfg["metric"] == "ip"
    norm = cfg["metric"] == "ip"
    X = gen_mixture(cfg["n"], cfg["d"], cfg["clusters"], 1, dev, cfg["half"], norm, aniso=aniso)
    return X


def make_queries(cfg, dev, rank, batch):
    aniso = cfg["metric"] == "ip"
    norm = cfg["metric"] == "ip"
    return gen_mixture(batch, cfg["d"], cfg["clusters"], 1000 + rank, dev, False, norm, aniso=aniso)


@torch.no_grad()
def exact_topk(X, Q, k, metric, rows=1024):
    """Exact fp32 ground truth (fp32 GEMM, no TF32), in blocks of queries whose
    score block stays near 8 GB."""
    rows = max(64, min(rows, (2 << 30) // max(1, X.shape[0])))
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    Xf = X.float()
    xn = (Xf * Xf).sum(1) if metric == "l2" else None
    out = []
    for a in range(0, Q.shape[0], rows):
        s = Q[a:a + rows] @ Xf.T
        if metric == "ip":
            out.append(torch.topk(s, k, dim=1).indices)
        else:
            out.append(torch.topk(xn.view(1, -1) - 2.0 * s, k, dim=1, largest=False).indices)
    torch.backends.cuda.matmul.allow_tf32 = prev
    del Xf
    return torch.cat(out).cpu().numpy()


def recall(ids, truth, k):
    ids = np.asarray(ids)[:, :k]
    hit = [len(set(a.tolist()) & set(b.tolist())) for a, b in zip(ids, truth[:, :k])]
    return float(np.mean(hit)) / k


# ---------------------------------------------------------------------------
# clocks during the timed region

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.path = Path(os.environ.get("SWB_CLOCK_LOG", f"/tmp/swb_clocks_{os.getpid()}.csv"))

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.idx), "-lms", "200"], stdout=self.fh,
                                         stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()
        return False

    def summary(self):
        if self.proc is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        rows = []
        for line in self.path.read_text().splitlines():
            p = [x.strip() for x in line.split(",")]
            if len(p) < 9:
                continue
            try:
                rows.append((float(p[1]), float(p[2]), p[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i in range(4) if r[i].lower().startswith("active")})
        load = [s for s, _, _ in rows]
        return {"sm_mhz": statistics.median(load), "sm_max_mhz": max(m for _, m, _ in rows),
                "samples": len(rows), "reasons": reasons}


# ---------------------------------------------------------------------------

def measured_peak_hbm():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except (KeyError, ValueError):
            pass
    return 6650.0, "fallback"


def profile_traffic(name):
    """Per-launch DRAM bytes of the top kernel from a committed ncu summary."""
    p = ROOT / "profiles" / f"{name}.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except ValueError:
            return None
    return None


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def build_index(cfg, dev, world, rank):
    """The graph by this package's kernels: single GPU, or row blocks over
    the ranks with NCCL all-gathers (swann_b200.dist.build_sharded)."""
    from swann_b200 import build as B
    from swann_b200 import dist as D
    t = {}
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    n = cfg["n"]
    if world == 1:
        X = make_corpus(cfg, dev)
        torch.cuda.synchronize()
        t["generate_s"] = time.perf_counter() - t0
        t1 = time.perf_counter()
        cand, cd = B.knn_candidates(X, 128, metric=cfg["metric"])
        torch.cuda.synchronize()
        t["sweep_s"] = time.perf_counter() - t1
        t1 = time.perf_counter()
        G1 = B.robust_prune(X, cand, cd, 64, alpha=1.2, metric=cfg["metric"])
        torch.cuda.synchronize()
        t["prune_s"] = time.perf_counter() - t1
        del cand, cd
        t1 = time.perf_counter()
        G = B.add_reverse(X, G1, 64, alpha=1.2, metric=cfg["metric"])
        torch.cuda.synchronize()
        t["reverse_s"] = time.perf_counter() - t1
    else:
        Xfull = make_corpus(cfg, dev)   # each rank keeps only its row block as its "input"
        a, b = D.shard_bounds(n, world)[rank]
        Xl = Xfull[a:b].contiguous()
        del Xfull
        torch.cuda.synchronize()
        t["generate_s"] = time.perf_counter() - t0
        stage = {}

        def sweep(Xa, r0, r1):
            s = time.perf_counter()
            c, d = B.knn_candidates(Xa, 128, metric=cfg["metric"], rows=(r0, r1))
            torch.cuda.synchronize()
            stage["sweep_s"] = time.perf_counter() - s
            return c, d

        def prune(Xa, c, d):
            s = time.perf_counter()
            g = B.robust_prune(Xa, c, d, 64, alpha=1.2, metric=cfg["metric"])
            torch.cuda.synchronize()
            stage["prune_s"] = time.perf_counter() - s
            return g

        def reverse(Xa, G1, r0, r1):
            s = time.perf_counter()
            g = B.add_reverse(Xa, G1, 64, alpha=1.2, metric=cfg["metric"], rows=(r0, r1))
            torch.cuda.synchronize()
            stage["reverse_s"] = time.perf_counter() - s
            return g

        X, G = D.build_sharded(Xl, n, sweep, prune, reverse)
        t.update(stage)
    torch.cuda.synchronize()
    t["total_s"] = time.perf_counter() - t0
    return X, G, t


def cpu_baseline(X, G, Q, seeds, cfg, op, budget_s=15.0):
    """The reference's CPU search path (swann/_refcpu.py, restated in C by the
    oracle) on the host cores: independent branches, merged; timed on a
    bounded sample of the batch."""
    from oracle import oracle as O
    Xh = X.float().cpu().numpy() if X.dtype == torch.float16 else X.cpu().numpy()
    Gh = G.cpu().numpy()
    Qh = Q.cpu().numpy()
    Sh = seeds.cpu().numpy()
    cores = O.cpu_count()
    vec = 8 if X.dtype == torch.float16 else 4
    metric = 0 if cfg["metric"] == "ip" else 1
    kw = dict(k=cfg["k"], L=op["queue"], B=64, metric=metric, team=16, vec=vec, stop_eps=op["stop_eps"],
              kstop=min(cfg["k"], op["queue"]), threads=cores)
    m = cores * 2
    t = time.perf_counter()
    O.search(Xh, Gh, Qh[:m], Sh[:m], **kw)
    el = time.perf_counter() - t
    m2 = int(min(Qh.shape[0], max(m, m * budget_s / max(el, 1e-3))))
    t = time.perf_counter()
    O.search(Xh, Gh, Qh[:m2], Sh[:m2], **kw)
    el = time.perf_counter() - t
    return {"value": m2 / el, "unit": "queries/s", "cores": cores, "kind": "port",
            "sample": f"{m2} queries of the timed batch, the reference's CPU search (independent branches, "
                      f"_refcpu semantics) at the chosen branches/queue/stop_eps, C oracle on {cores} threads",
            "seconds": el}


# per-query table slots per claim of the busiest query (then a power of two);
# the clear of the table is a full write of it every step
TABLE_HEADROOM = 1.5


def table_slots_for(claims):
    from swann_b200 import _engine as E
    return max(4096, E.next_pow2(int(TABLE_HEADROOM * claims)))


def calibrate(index, Qs, truth, cfg):
    """Fastest (branches, queue, stop_eps) with recall >= TARGET on Qs."""
    best = None
    tried = []
    for branches, queue in cfg.get("ladder", LADDER):
        found = False
        for eps in EPS:
            ids, _ = index.search_tensors(Qs, k=cfg["k"], branches=branches, queue=queue, stop_eps=eps)
            torch.cuda.synchronize()
            r = recall(ids.cpu().numpy()[:, :10], truth[:, :10], 10)   # the target is recall@10
            if r < TARGET:
                tried.append((branches, queue, eps, r, None))
                continue
            ts = []
            for _ in range(2):
                s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s0.record()
                index.search_tensors(Qs, k=cfg["k"], branches=branches, queue=queue, stop_eps=eps)
                s1.record()
                torch.cuda.synchronize()
                ts.append(s0.elapsed_time(s1))
            tried.append((branches, queue, eps, r, min(ts)))
            if best is None or min(ts) < best[4]:
                best = (branches, queue, eps, r, min(ts))
            found = True
            break   # larger eps only costs more at this (branches, queue)
        if found and best is not None and branches >= 64:
            break
    return best, tried


def run(args):
    world, rank, local = dist_setup()
    dev = torch.device("cuda", local)
    cfg = dict(CONFIGS[args.config])
    if args.batch:
        cfg["batch"] = args.batch
    import swann_b200 as swann
    from swann_b200 import _engine as E
    from swann_b200 import _select as S

    X, G, build_t = build_index(cfg, dev, world, rank)
    torch.cuda.empty_cache()
    index = swann.Index(X, G, metric=cfg["metric"], catalogue_size=cfg.get("catalogue", 4096))
    batch = cfg["batch"]
    Q = make_queries(cfg, dev, rank, batch)
    gt_n = min(batch, args.gt)
    truth = exact_topk(X, Q[:gt_n], cfg["k"], cfg["metric"])

    # operating point: chosen on rank 0, shared (or fixed on the command line)
    if args.fixed:
        b, q, e = args.fixed.split(",")
        op, tried = dict(branches=int(b), queue=int(q), stop_eps=float(e)), []
    elif rank == 0:
        best, tried = calibrate(index, Q[:gt_n], truth, cfg)
        if best is None:
            best = max(tried, key=lambda t: t[3])
        op = dict(branches=best[0], queue=best[1], stop_eps=best[2])
    else:
        op, tried = None, []
    if world > 1 and not args.fixed:
        import torch.distributed as dist
        box = [op]
        dist.broadcast_object_list(box, src=0)
        op = box[0]

    # Size the per-query distance table from what the queries actually claim:
    # TABLE_HEADROOM times the busiest query's claims, a power of two (load
    # <= 67% for that query, ~15% for a typical one).  A probe run that finds
    # no slot scores the row uncached, so a fuller table costs dedup, not results.
    ent = S.select_nearest(Q[:gt_n], index._cat, op["branches"], metric=index._m)
    sd = index.catalogue[ent].to(torch.int32)
    _, _, ctr, _ = E.search_fused_lean(X, G, Q[:gt_n], sd, k=cfg["k"], L=op["queue"], B=64, metric=index._m,
                                       team_size=16, stop_eps=op["stop_eps"], shared_cache=True,
                                       shared_bound=True, exclusive=2, elide_visited=True)
    claims = (ctr[..., 5].to(torch.int64).sum(1) + op["branches"]).max().item()
    ref_slots = E.cache_size(op["branches"], 64, G.shape[1])
    slots = min(ref_slots, table_slots_for(claims))
    index.table_slots = slots
    table = {"slots": slots, "reference_slots": ref_slots, "max_claims_per_query": int(claims),
             "max_load": round(claims / slots, 4)}

    def step():
        return index.search_tensors(Q, k=cfg["k"], **op)

    # recall of the full-batch operating point, on the ground-truth subset
    ids, _ = step()
    torch.cuda.synchronize()
    got = ids[:gt_n].cpu().numpy()
    rec = recall(got[:, :10], truth[:, :10], 10)
    rec_k = recall(got, truth, cfg["k"])

    # -- device-resident timing (value) ----------------------------------
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        barrier(world)
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1), world)
    clocks = clk.summary()
    value = world * batch * args.steps / (ms / 1e3)

    # -- end to end through the public API with host buffers -------------
    Qh = Q.cpu().pin_memory()
    for _ in range(max(1, args.warmup // 2)):
        index.search(Qh, k=cfg["k"], **op)
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        out_ids, out_d = index.search(Qh, k=cfg["k"], **op)
    torch.cuda.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t0, world)
    e2e = {"value": world * batch * args.steps / e2e_s, "unit": "queries/s",
           "h2d_bytes_per_step": int(Qh.numel() * Qh.element_size()),
           "d2h_bytes_per_step": int(out_ids.nbytes + out_d.nbytes)}

    # -- roofline of the dominant kernel (the fused search) ----------------
    ent = S.select_nearest(Q, index._cat, op["branches"], metric=index._m)
    seeds = index.catalogue[ent].to(torch.int32)
    order = index.locality_order(ent)   # the order Index.search runs the batch in
    if order is not None:
        Q, seeds = Q[order].contiguous(), seeds[order].contiguous()
    kw = dict(k=cfg["k"], L=op["queue"], B=64, metric=index._m, team_size=16, stop_eps=op["stop_eps"],
              shared_cache=True, shared_bound=True, exclusive=2, elide_visited=True, table_slots=slots)
    _, _, ctr, _ = E.search_fused_lean(X, G, Q, seeds, **kw)
    torch.cuda.synchronize()
    c = ctr.to(torch.int64)
    nodes = int(c[..., 5].sum()) + int(batch * op["branches"])      # claimed + seeds
    exps = int(c[..., 0].sum())
    esize = X.element_size()
    alg_bytes = nodes * cfg["d"] * esize + exps * G.shape[1] * 4
    lib = E.N.lib()
    kt = []
    for _ in range(max(3, args.steps)):
        # prepare + fused, each bracketed by events on the launching stream
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        Jq = op["branches"]
        Hc = slots
        cache = E._WS.get("cache", batch * Hc, torch.int64, dev).view(batch, -1)
        bound = E._WS.get("bound", batch, torch.float32, dev)
        qdone = E._WS.get("qdone", batch, torch.int32, dev)
        kk = min(cfg["k"], op["queue"])
        bi = E._WS.get("branch_ids", batch * Jq * kk, torch.int32, dev)
        bd = E._WS.get("branch_dist", batch * Jq * kk, torch.float32, dev)
        oi = torch.empty((batch, cfg["k"]), dtype=torch.int32, device=dev)
        od = torch.empty((batch, cfg["k"]), dtype=torch.float32, device=dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        s = stream.cuda_stream
        ev[0].record(stream)
        E.N.check(lib.swb_search_prepare(batch, E.N.ptr(cache), Hc, E.N.ptr(bound), E.N.ptr(qdone), s))
        ev[1].record(stream)
        rc = lib.swb_search_fused(
            E.N.ptr(X), E.N.dtype_code(X), X.shape[0], X.shape[1], E.N.ptr(G), G.shape[1], E.N.ptr(Q),
            E.N.ptr(seeds), batch, Jq, 1, cfg["k"], op["queue"], 64, index._m, 16, 0, float(op["stop_eps"]),
            cfg["k"], None, 1, E.N.ptr(cache), Hc, E.N.ptr(bound), 2, 0, 0.0, E.N.ptr(bi), E.N.ptr(bd),
            E.N.ptr(qdone), E.N.ptr(oi), E.N.ptr(od), None, None, None, None, None, E.N.ptr(status), s)
        E.N.check(rc)
        ev[2].record(stream)
        torch.cuda.synchronize()
        kt.append((ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2])))
    prep_ms = statistics.median(t[0] for t in kt)
    fused_ms = statistics.median(t[1] for t in kt)
    peak, peak_kind = measured_peak_hbm()
    achieved = alg_bytes / (fused_ms / 1e3) / 1e9
    prof = profile_traffic(f"search_fused_{args.config}")
    traffic, traffic_src = None, None
    if prof:
        same = prof.get("batch") == batch and prof.get("op") == [op["branches"], op["queue"], op["stop_eps"]]
        if same:
            traffic, traffic_src = prof["traffic_per_launch"], "ncu, this launch shape: " + prof["source"]
        else:   # same kernel and corpus, another batch or operating point: scale by this run's bytes
            traffic = round(prof["traffic_over_algorithmic"] * alg_bytes)
            traffic_src = "ncu traffic/algorithmic ratio %.3f x this run's algorithmic bytes (%s)" % (
                prof["traffic_over_algorithmic"], prof["source"])
    roofline = {"bound": "hbm", "kernel": "swb::fused_kernel", "achieved": round(achieved, 1), "peak": peak,
                "unit": "GB/s", "frac": round(achieved / peak, 4), "peak_source": f"{peak_kind} hbm_gbs",
                "traffic": traffic, "traffic_source": traffic_src,
                # what DRAM itself moved per second (the measured traffic over this run's kernel time); the
                # algorithmic rate above also counts the rows that L2 serves to queries run side by side
                "dram_gbs": round(traffic / (fused_ms / 1e3) / 1e9, 1) if traffic else None,
                "dram_frac": round(traffic / (fused_ms / 1e3) / 1e9 / peak, 4) if traffic else None,
                "algorithmic_bytes_per_launch": alg_bytes, "kernel_ms": round(fused_ms, 3),
                "prepare_ms": round(prep_ms, 3),
                "per_query": {"distinct_nodes_scored": nodes / batch, "expansions": exps / batch}}

    line = {
        "metric": f"QPS at recall@10>={TARGET} ({cfg['desc']}, batch {batch} per GPU)",
        "value": round(value, 1), "unit": "queries/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded Gaussian mixture generated on the GPU, BASELINE.json config)",
        "config": {"workload": args.config, "n": cfg["n"], "d": cfg["d"], "storage": "f16" if cfg["half"] else "f32",
                   "metric": cfg["metric"], "batch_per_gpu": batch, "k": cfg["k"], **op, "budget": 64, "team": 16,
                   "recall@10": round(rec, 4), **({f"recall@{cfg['k']}": round(rec_k, 4)} if cfg["k"] != 10 else {}),
                   "recall_sample": gt_n, "graph": "degree 64, candidates 128, alpha 1.2",
                   "catalogue": int(index.catalogue.numel()),
                   "claims": "strict (exclusive=2)", "table": table,
                   "query_order": "nearest catalogue entry" if index.locality else "input",
                   "l2": "inputs larger than L2 (corpus %.1f GB; rows gathered at random)" % (
                       X.numel() * X.element_size() / 1e9),
                   "parallelism": f"query shards x{world}, replicas"},
        "e2e": e2e, "roofline": roofline, "clocks": clocks, "gpu_launches": 2 * args.steps,
        "build": {k: round(v, 3) for k, v in build_t.items()},
        "calibration": [{"branches": b, "queue": q, "stop_eps": e, "recall": round(r, 4),
                         "ms": None if t is None else round(t, 3)} for b, q, e, r, t in tried],
    }
    if rank == 0 and world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline(X, G, Q, seeds, cfg, op)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_build(args):
    """Graph build seconds (sweep / prune / reverse) on one GPU, with the sweep
    against the tensor pipe: 2 n^2 d FLOPs over the measured dense bf16 peak
    for fp16 rows (kind::f16), a sixth of it for fp32 rows (3xTF32 issues three
    tf32 MMAs per product at half the bf16 rate).  The sweep runs for seconds
    under the 1 kW power cap, so the denominator is the sustained GEMM figure;
    the fraction of the burst figure is reported beside it."""
    world, rank, local = dist_setup()
    dev = torch.device("cuda", local)
    cfg = dict(CONFIGS[args.config])
    from swann_b200 import build as B
    X = make_corpus(cfg, dev)
    torch.cuda.synchronize()
    n, d = X.shape
    with ClockSampler(local) as clk:
        t0 = time.perf_counter()
        cand, cd = B.knn_candidates(X, 128, metric=cfg["metric"])
        torch.cuda.synchronize()
        t1 = time.perf_counter()
    G1 = B.robust_prune(X, cand, cd, 64, alpha=1.2, metric=cfg["metric"])
    torch.cuda.synchronize()
    t2 = time.perf_counter()
    G = B.add_reverse(X, G1, 64, alpha=1.2, metric=cfg["metric"])
    torch.cuda.synchronize()
    t3 = time.perf_counter()
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    burst = float(peaks.get("bf16_tflops", 1590.0))
    sustained = float(peaks.get("bf16_tflops_sustained", 1400.0))
    flops = 2.0 * n * n * d
    div = 1.0 if cfg["half"] else 6.0
    ceiling = sustained / div
    achieved = flops / (t1 - t0) / 1e12
    line = {"metric": f"graph build seconds ({cfg['desc']}, degree 64, candidates 128, alpha 1.2)",
            "value": round(t3 - t0, 3), "unit": "s", "n_gpus": world, "higher_is_better": False,
            "data": "synthetic (seeded Gaussian mixture generated on the GPU, BASELINE.json config)",
            "config": {"workload": args.config, "n": n, "d": d, "storage": "f16" if cfg["half"] else "f32",
                       "metric": cfg["metric"], "sweep": os.environ.get("SWB_SWEEP", "mma")},
            "stages_s": {"sweep": round(t1 - t0, 3), "prune": round(t2 - t1, 3), "reverse": round(t3 - t2, 3)},
            "roofline": {"bound": "tensor", "kernel": "swb::sweep::sweep_kernel", "achieved": round(achieved, 1),
                         "peak": round(ceiling, 1), "unit": "TFLOP/s", "frac": round(achieved / ceiling, 4),
                         "peak_source": ("measured bf16_tflops_sustained" if cfg["half"] else
                                         "measured bf16_tflops_sustained / 6 (3xTF32)"),
                         "frac_of_burst": round(achieved / (burst / div), 4), "flops": flops},
            "clocks_during_sweep": clk.summary(),
            "mean_out_degree": round(float((G >= 0).sum(1).float().mean()), 2)}
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_reference(args):
    """The reference's own CPU search path (the C restatement of
    swann/_refcpu.py, independent branches merged) on the host cores, on the
    same workload; the index is built on the GPU by this package first
    (setup, untimed: the reference's CPU build would take days at this size)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    cfg = dict(CONFIGS[args.config])
    if args.batch:
        cfg["batch"] = args.batch
    import swann_b200 as swann
    from oracle import oracle as O
    X, G, _ = build_index(cfg, dev, 1, 0)
    index = swann.Index(X, G, metric=cfg["metric"], catalogue_size=cfg.get("catalogue", 4096))
    Q = make_queries(cfg, dev, 0, cfg["batch"])
    # the operating point of the other arm: --fixed, or the same calibration
    # (recall >= TARGET on the ground-truth subset; untimed setup, like the build)
    if args.fixed:
        b, q, e = args.fixed.split(",")
        op = dict(branches=int(b), queue=int(q), stop_eps=float(e))
    else:
        gt_n = min(cfg["batch"], args.gt)
        truth = exact_topk(X, Q[:gt_n], cfg["k"], cfg["metric"])
        best, tried = calibrate(index, Q[:gt_n], truth, cfg)
        if best is None:
            best = max(tried, key=lambda t: t[3])
        op = dict(branches=best[0], queue=best[1], stop_eps=best[2])
    from swann_b200 import _select as S
    ent = S.select_nearest(Q, index._cat, op["branches"], metric=index._m)
    seeds = index.catalogue[ent].to(torch.int32)
    Xh = X.float().cpu().numpy()
    Gh, Qh, Sh = G.cpu().numpy(), Q.cpu().numpy(), seeds.cpu().numpy()
    cores = O.cpu_count()
    metric = 0 if cfg["metric"] == "ip" else 1
    kw = dict(k=cfg["k"], L=op["queue"], B=64, metric=metric, team=16, vec=8 if cfg["half"] else 4,
              stop_eps=op["stop_eps"], kstop=min(cfg["k"], op["queue"]), threads=cores)
    per = cores * 2
    times = []
    for i in range(args.warmup + args.steps):
        a = (i * per) % max(1, Qh.shape[0] - per)
        t = time.perf_counter()
        O.search(Xh, Gh, Qh[a:a + per], Sh[a:a + per], **kw)
        if i >= args.warmup:
            times.append(time.perf_counter() - t)
    el = sum(times)
    value = per * args.steps / el
    line = {"metric": f"QPS at recall@10>={TARGET} ({cfg['desc']}, batch {cfg['batch']} per GPU)",
            "value": round(value, 2), "unit": "queries/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "impl": "reference",
            "data": "synthetic (seeded Gaussian mixture generated on the GPU, BASELINE.json config)",
            "config": {"workload": args.config, "n": cfg["n"], "d": cfg["d"], **op, "budget": 64, "team": 16},
            "cpu_baseline": {"value": round(value, 2), "unit": "queries/s", "cores": cores, "kind": "port",
                             "sample": f"{per} queries per step (C restatement of swann/_refcpu.py, independent "
                                       f"branches, {cores} threads); index built and the operating point "
                                       f"calibrated on the GPU beforehand, untimed"},
            "e2e": {"value": round(value, 2), "unit": "queries/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# C3's batch schedule: branches 128 up to batch 64, 64 at
# 512, 32 from 4096 on
BATCH_SWEEP = [(1, 128), (8, 128), (64, 128), (512, 64), (4096, 32), (65535, 32)]


def run_batch_sweep(args):
    """QPS and per-batch latency across batch sizes on one GPU, one index.
    The operating point per branch count is the smallest stop_eps (queue 12)
    reaching recall@10 >= TARGET on the ground-truth subset (recall does not
    depend on the batch: queries are independent); each batch size is then
    timed over consecutive slices of the query set with CUDA events."""
    dist_setup()
    dev = torch.device("cuda", 0)
    cfg = dict(CONFIGS[args.config])
    import swann_b200 as swann
    X, G, _ = build_index(cfg, dev, 1, 0)
    torch.cuda.empty_cache()
    index = swann.Index(X, G, metric=cfg["metric"], catalogue_size=cfg.get("catalogue", 4096))
    nmax = max(b for b, _ in BATCH_SWEEP)
    Q = make_queries(cfg, dev, 0, nmax)
    gt_n = min(nmax, args.gt)
    truth = exact_topk(X, Q[:gt_n], cfg["k"], cfg["metric"])
    from swann_b200 import _engine as E
    from swann_b200 import _select as S
    ops = {}
    for _, br in BATCH_SWEEP:
        if br in ops:
            continue
        index.table_slots = None
        for eps in EPS:
            ids, _ = index.search_tensors(Q[:gt_n], k=cfg["k"], branches=br, queue=12, stop_eps=eps)
            r = recall(ids.cpu().numpy()[:, :10], truth[:, :10], 10)
            if r >= TARGET:
                break
        # table sized from measured claims, as the main line does
        sd = index.catalogue[S.select_nearest(Q[:gt_n], index._cat, br, metric=index._m)].to(torch.int32)
        _, _, ctr, _ = E.search_fused_lean(X, G, Q[:gt_n], sd, k=cfg["k"], L=12, B=64, metric=index._m,
                                           team_size=16, stop_eps=eps, shared_cache=True, shared_bound=True,
                                           exclusive=2, elide_visited=True)
        claims = (ctr[..., 5].to(torch.int64).sum(1) + br).max().item()
        ops[br] = (eps, r, min(E.cache_size(br, 64, G.shape[1]), table_slots_for(claims)))
    rows = []
    for b, br in BATCH_SWEEP:
        eps, r, slots = ops[br]
        index.table_slots = slots
        kw = dict(k=cfg["k"], branches=br, queue=12, stop_eps=eps)
        reps = max(args.steps, min(200, nmax // b))
        for i in range(args.warmup):
            index.search_tensors(Q[(i * b) % (nmax - b + 1):][:b], **kw)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(reps):
            a = (i * b) % (nmax - b + 1)
            index.search_tensors(Q[a:a + b], **kw)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        rows.append({"batch": b, "branches": br, "queue": 12, "stop_eps": eps, "recall@10": round(r, 4),
                     "table_slots": slots,
                     "ms_per_batch": round(ms, 3), "qps": round(b / (ms / 1e3), 1), "batches_timed": reps})
    line = {"metric": f"QPS and latency by batch size at recall@10>={TARGET} ({cfg['desc']})",
            "unit": "queries/s", "n_gpus": 1, "higher_is_better": True, "dtype": "f32",
            "data": "synthetic (seeded Gaussian mixture generated on the GPU, BASELINE.json config)",
            "config": {"workload": args.config, "n": cfg["n"], "d": cfg["d"], "k": cfg["k"], "budget": 64,
                       "team": 16, "recall_sample": gt_n, "timing": "CUDA events, device-resident queries"},
            "batches": rows}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="swann_b200", choices=["swann_b200", "reference"])
    ap.add_argument("--config", default="c3", choices=sorted(CONFIGS))
    ap.add_argument("--batch", type=int, default=0)
    ap.add_argument("--gt", type=int, default=8192)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--fixed", default="", help="branches,queue,stop_eps: skip the calibration")
    ap.add_argument("--build-only", action="store_true", help="time the graph build instead of the search")
    ap.add_argument("--batch-sweep", action="store_true", help="QPS and latency across the C3 batch sizes")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.build_only:
        run_build(args)
    elif args.batch_sweep:
        run_batch_sweep(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run(args)


if __name__ == "__main__":
    main()
