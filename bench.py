#!/usr/bin/env python
"""SWANN on B200: QPS at recall@10 >= 0.95, HBM roofline, build seconds.

Workload (the north star's headline): n = 1,000,000 rows,
d = 1536, drawn from 1,000 anisotropic Gaussian clusters (per-dimension scales
log-uniform in [0.1, 1]), rows L2-normalised and stored fp16; fp32 queries
normalised from the same mixture; inner product; k = 10; a global batch of
65,535 queries per step, split across the GPUs in contiguous shards (strong
scaling; the per-GPU-fixed weak figure is reported beside it for N > 1);
degree-64 graph (candidates 128, alpha 1.2) built by this package's kernels.
Seeded synthetic data stands in for the corpora the reference measured on.

A step is one Index.search of each GPU's shard.  The operating point
(branches, queue, stop_eps) is the fastest one whose recall@10 against exact
fp32 ground truth is >= 0.95, chosen before timing on a fixed subset of the
batch.

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

def gen_mixture(n, d, clusters, seed, dev, half, normalise, aniso=True, chunk=1 << 16, sigma=0.3, rows=None):
    """Rows [r0, r1) (default all n) of a seeded Gaussian-mixture corpus.  The
    mixture (centres, scales) comes from one fixed seed; each 65536-row chunk
    draws from its own stream (seed, chunk), so a rank can generate exactly its
    own row block and get the same rows a single process would."""
    g = torch.Generator(device=dev)
    g.manual_seed(1234)   # the mixture itself is shared by corpus and queries
    if clusters:
        centres = torch.randn((clusters, d), generator=g, device=dev)
        if aniso:
            lo, hi = np.log(0.1), np.log(1.0)
            scales = torch.exp(lo + (hi - lo) * torch.rand((clusters, d), generator=g, device=dev))
        else:
            scales = torch.full((clusters, d), sigma, device=dev)
    r0, r1 = (0, n) if rows is None else rows
    out = torch.empty((r1 - r0, d), dtype=torch.float16 if half else torch.float32, device=dev)
    gs = torch.Generator(device=dev)
    for c in range(r0 // chunk, (r1 + chunk - 1) // chunk):
        a, b = c * chunk, min(n, (c + 1) * chunk)
        gs.manual_seed(seed * 1_000_003 + c)
        z = torch.randn((b - a, d), generator=gs, device=dev)
        if clusters:
            cl = torch.randint(0, clusters, (b - a,), generator=gs, device=dev)
            x = centres[cl] + scales[cl] * z
        else:
            x = z
        if normalise:
            x = x / x.norm(dim=1, keepdim=True)
        lo, hi = max(a, r0), min(b, r1)
        out[lo - r0:hi - r0] = x[lo - a:hi - a].to(out.dtype)
    return out


def make_corpus(cfg, dev, rows=None):
    aniso = cfg["metric"] == "ip"
    norm = cfg["metric"] == "ip"
    return gen_mixture(cfg["n"], cfg["d"], cfg["clusters"], 1, dev, cfg["half"], norm, aniso=aniso, rows=rows)


def make_queries(cfg, dev, seed, batch):
    aniso = cfg["metric"] == "ip"
    norm = cfg["metric"] == "ip"
    return gen_mixture(batch, cfg["d"], cfg["clusters"], seed, dev, False, norm, aniso=aniso)


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
        # NCCL writes its version banner (and warnings) to stdout unless given a
        # file; rank 0's stdout carries only the JSON line
        os.environ.setdefault("NCCL_DEBUG_FILE", f"/tmp/swb_nccl_{os.getpid()}.log")
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
    the ranks with NCCL all-gathers (swann_b200.dist.build_sharded); under
    torchrun each rank generates only its own row block of the corpus."""
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
        ops = B.TcOperands(X)       # the rows as the tensor cores read them, shared by the three stages
        cand, cd = B.knn_candidates(X, 128, metric=cfg["metric"], ops=ops)
        torch.cuda.synchronize()
        t["sweep_s"] = time.perf_counter() - t1
        t1 = time.perf_counter()
        G1 = B.robust_prune(X, cand, cd, 64, alpha=1.2, metric=cfg["metric"], ops=ops)
        torch.cuda.synchronize()
        t["prune_s"] = time.perf_counter() - t1
        tp = time.perf_counter()
        parity = candidate_parity(X, cand, cd, metric=cfg["metric"])   # a check of the sweep's lists, not timed
        t["parity_s"] = time.perf_counter() - tp
        del cand, cd
        t1 = time.perf_counter()
        G = B.add_reverse(X, G1, 64, alpha=1.2, metric=cfg["metric"], ops=ops)
        torch.cuda.synchronize()
        t["reverse_s"] = time.perf_counter() - t1
        t["exact_recomputed_pairs"] = int(ops.recomputed[0])
        t["candidate_parity"] = parity
        del ops
    else:
        a, b = D.shard_bounds(n, world)[rank]
        Xl = make_corpus(cfg, dev, rows=(a, b))   # this rank's row block is its input
        torch.cuda.synchronize()
        t["generate_s"] = time.perf_counter() - t0
        stage = {}
        shared = {}

        def operands(Xa):
            if "ops" not in shared:
                shared["ops"] = B.TcOperands(Xa)
            return shared["ops"]

        def sweep(Xa, r0, r1):
            s = time.perf_counter()
            c, d = B.knn_candidates(Xa, 128, metric=cfg["metric"], rows=(r0, r1), ops=operands(Xa))
            torch.cuda.synchronize()
            stage["sweep_s"] = time.perf_counter() - s
            return c, d

        def prune(Xa, c, d):
            s = time.perf_counter()
            g = B.robust_prune(Xa, c, d, 64, alpha=1.2, metric=cfg["metric"], ops=operands(Xa))
            torch.cuda.synchronize()
            stage["prune_s"] = time.perf_counter() - s
            return g

        def reverse(Xa, G1, r0, r1):
            s = time.perf_counter()
            g = B.add_reverse(Xa, G1, 64, alpha=1.2, metric=cfg["metric"], rows=(r0, r1), ops=operands(Xa))
            torch.cuda.synchronize()
            stage["reverse_s"] = time.perf_counter() - s
            return g

        X, G = D.build_sharded(Xl, n, sweep, prune, reverse)
        t.update(stage)
        shared.clear()
    torch.cuda.synchronize()
    t["total_s"] = time.perf_counter() - t0 - t.get("parity_s", 0.0)
    return X, G, t


def sweep_roofline(build_t, n, d, half):
    """The candidate sweep against the tensor pipe: 2 n^2 d FLOPs (counted as
    written) over the measured sustained bf16 GEMM rate for fp16 rows
    (kind::f16), or a sixth of it for fp32 rows (3xTF32: three tf32 MMAs per
    product at half the bf16 rate)."""
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    sustained = float(peaks.get("bf16_tflops_sustained", 1400.0))
    kind = "measured" if "bf16_tflops_sustained" in peaks else "fallback"
    div = 1.0 if half else 6.0
    flops = 2.0 * n * n * d
    sec = build_t.get("sweep_s")
    if not sec:
        return None
    achieved = flops / sec / 1e12
    return {"bound": "tensor", "kernel": "swb::sweep::sweep_kernel", "achieved": round(achieved, 1),
            "peak": round(sustained / div, 1), "unit": "TFLOP/s", "frac": round(achieved / (sustained / div), 4),
            "peak_source": f"{kind} bf16_tflops_sustained" + ("" if half else " / 6 (3xTF32)"), "flops": flops}


def sample_rows(total, m):
    """m row indices spread evenly over [0, total): a sample that follows the
    batch's own order (the input order, not the locality order)."""
    m = max(1, min(int(m), total))
    return np.unique(np.linspace(0, total - 1, m).round().astype(np.int64))


def cpu_baseline(X, G, Q, seeds, cfg, op, budget_s=15.0):
    """The reference's CPU search path (swann/_refcpu.py, restated in C by the
    oracle) on the host cores: independent branches, merged; timed on a
    bounded sample of the batch spread evenly over it in input order."""
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
    pick = sample_rows(Qh.shape[0], cores * 2)
    t = time.perf_counter()
    O.search(Xh, Gh, Qh[pick], Sh[pick], **kw)
    el = time.perf_counter() - t
    pick = sample_rows(Qh.shape[0], max(len(pick), len(pick) * budget_s / max(el, 1e-3)))
    t = time.perf_counter()
    O.search(Xh, Gh, Qh[pick], Sh[pick], **kw)
    el = time.perf_counter() - t
    return {"value": round(len(pick) / el, 2), "unit": "queries/s", "cores": cores, "kind": "port",
            "sample": f"{len(pick)} queries spread evenly over the timed batch in input order; the reference's CPU "
                      f"search (independent branches, _refcpu semantics) at the chosen branches/queue/stop_eps, "
                      f"C oracle on {cores} threads",
            "seconds": round(el, 3)}


def exact_distance_error(X, Q, ids, dist, metric):
    """Largest relative gap between the returned distances and an exact
    (float64) recomputation from the stored rows."""
    ids = ids.to(torch.int64)
    ok = ids >= 0
    x = X[ids.clamp(min=0)].double()
    q = Q.double()[:, None, :]
    ex = 1.0 - (q * x).sum(-1) if metric == "ip" else ((q - x) ** 2).sum(-1)
    rel = (dist.double() - ex).abs() / ex.abs().clamp(min=1e-30)
    return float(rel[ok].max()) if bool(ok.any()) else 0.0


def reference_package():
    """The reference package installed under baseline/_ref (baseline/install.sh),
    or None."""
    path = ROOT / "baseline" / "_ref"
    if not (path / "swann" / "__init__.py").exists():
        return None
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))
    import swann
    return swann


def reference_kernels_for(swann_ref):
    """Hands the reference's engine its own kernels.  The reference compiles
    swann/csrc/local_search.cu on first use (swann/_engine.py:42-63) for the
    architecture TORCH_CUDA_ARCH_LIST names, 12.0 unless set; here the same
    source, compiled with the same flags for sm_100a (oracle/_ref), fills the
    engine's extension slot, so its Python path runs unmodified.  Without that
    build the reference compiles itself for this GPU.  Returns a description."""
    from oracle import oracle as O
    K = O.ref_kernels()
    if K is not None:
        swann_ref._engine._EXT = K
        return "swann/csrc/local_search.cu compiled unmodified for sm_100a (oracle/_ref)"
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    swann_ref._engine.ext()
    return "swann/csrc/local_search.cu compiled by the reference's own ext() for sm_100a"


def time_reference_gpu(ref_index, Qd, k, op, reps=3):
    """The reference's Index.search (its seed selection, engine, kernels and
    the copy of the answers to the host) on a device-resident batch; wall
    clock around synchronous calls (it returns numpy arrays)."""
    kw = dict(k=k, branches=op["branches"], queue=op["queue"], stop_eps=op["stop_eps"])
    ref_index.search(Qd, **kw)
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        t = time.perf_counter()
        ref_index.search(Qd, **kw)
        torch.cuda.synchronize()
        ts.append(time.perf_counter() - t)
    return statistics.median(ts)


def reference_gpu_leg(X, G, catalogue, Qall, truth, gt_n, cfg, op):
    """The same-box GPU bar: the reference's own Index.search on this graph,
    catalogue and operating point -- recall@10 on the ground-truth sample and
    QPS on the whole batch."""
    swann_ref = reference_package()
    if swann_ref is None:
        return {"unavailable": "the reference package is not installed under baseline/_ref (baseline/install.sh)"}
    impl = reference_kernels_for(swann_ref)
    ref_index = swann_ref.Index(X, G, metric=cfg["metric"], catalogue=catalogue)
    ids, _ = ref_index.search(Qall[:gt_n], k=cfg["k"], branches=op["branches"], queue=op["queue"],
                              stop_eps=op["stop_eps"])
    rec = recall(ids[:, :10], truth[:, :10], 10)
    sec = time_reference_gpu(ref_index, Qall, cfg["k"], op)
    del ref_index
    torch.cuda.empty_cache()
    return {"qps": round(Qall.shape[0] / sec, 1), "ms_per_batch": round(sec * 1e3, 3), "batch": int(Qall.shape[0]),
            "recall@10": round(rec, 4), "impl": "swann/index.py Index.search (exclusive claims, the reference's "
                                                "table sizing) over " + impl,
            "timing": "wall clock around the synchronous call (device-resident queries, answers to the host), "
                      "median of 3 after one warm-up"}


def calibrate(search, Qs, truth, cfg):
    """Fastest (branches, queue, stop_eps) with recall >= TARGET on Qs;
    search(Qs, k, branches, queue, stop_eps) -> ids (host or device)."""
    best = None
    tried = []
    for branches, queue in cfg.get("ladder", LADDER):
        found = False
        for eps in EPS:
            ids = search(Qs, cfg["k"], branches, queue, eps)
            torch.cuda.synchronize()
            ids = ids.cpu().numpy() if isinstance(ids, torch.Tensor) else np.asarray(ids)
            r = recall(ids[:, :10], truth[:, :10], 10)   # the target is recall@10
            if r < TARGET:
                tried.append((branches, queue, eps, r, None))
                continue
            ts = []
            for _ in range(2):
                torch.cuda.synchronize()
                t = time.perf_counter()
                search(Qs, cfg["k"], branches, queue, eps)
                torch.cuda.synchronize()
                ts.append((time.perf_counter() - t) * 1e3)
            tried.append((branches, queue, eps, r, min(ts)))
            if best is None or min(ts) < best[4]:
                best = (branches, queue, eps, r, min(ts))
            found = True
            break   # larger eps only costs more at this (branches, queue)
        if found and best is not None and branches >= 64:
            break
    return best, tried


def choose_op(args, search, Qs, truth, cfg, rank, world):
    """The operating point: --fixed, or calibrated on rank 0 and shared."""
    if args.fixed:
        b, q, e = args.fixed.split(",")
        return dict(branches=int(b), queue=int(q), stop_eps=float(e)), []
    op, tried = None, []
    if rank == 0:
        best, tried = calibrate(search, Qs, truth, cfg)
        if best is None:
            best = max(tried, key=lambda t: t[3])
        op = dict(branches=best[0], queue=best[1], stop_eps=best[2])
    if world > 1:
        import torch.distributed as dist
        box = [op]
        dist.broadcast_object_list(box, src=0)
        op = box[0]
    return op, tried


def timed_steps(step, steps, warmup, world, local, sample_clocks=True):
    """W untimed steps, then K steps bracketed by a barrier and a device
    synchronisation on both sides, timed with CUDA events on the launching
    stream; the max over ranks."""
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = ClockSampler(local) if sample_clocks else None
    if clk:
        clk.__enter__()
    try:
        torch.cuda.synchronize()
        barrier(world)
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
    finally:
        if clk:
            clk.__exit__(None, None, None)
    ms = max_over_ranks(e0.elapsed_time(e1), world)
    return ms, (clk.summary() if clk else None)


def run(args):
    world, rank, local = dist_setup()
    dev = torch.device("cuda", local)
    cfg = dict(CONFIGS[args.config])
    if args.batch:
        cfg["batch"] = args.batch
    import swann_b200 as swann
    from swann_b200 import _engine as E
    from swann_b200 import _select as S
    from swann_b200 import dist as D

    X, G, build_t = build_index(cfg, dev, world, rank)
    torch.cuda.empty_cache()
    index = swann.Index(X, G, metric=cfg["metric"], catalogue_size=cfg.get("catalogue", 4096))
    batch = cfg["batch"]                                   # the global batch of one step
    Qall = make_queries(cfg, dev, 1000, batch)             # the same on every rank
    a, b = D.shard_bounds(batch, world)[rank]
    Q = Qall[a:b].contiguous()                             # this rank's shard
    gt_n = min(batch, args.gt)
    truth = exact_topk(X, Qall[:gt_n], cfg["k"], cfg["metric"]) if rank == 0 else None

    def my_search(Qs, k, branches, queue, eps):
        return index.search_tensors(Qs, k=k, branches=branches, queue=queue, stop_eps=eps)[0]

    op, tried = choose_op(args, my_search, Qall[:gt_n], truth, cfg, rank, world)

    # recall and exact distances at the operating point, on the ground-truth sample
    checks = {}
    if rank == 0:
        ids_s, dist_s = index.search_tensors(Qall[:gt_n], k=cfg["k"], **op)
        got = ids_s.cpu().numpy()
        checks["recall@10"] = round(recall(got[:, :10], truth[:, :10], 10), 4)
        if cfg["k"] != 10:
            checks[f"recall@{cfg['k']}"] = round(recall(got, truth, cfg["k"]), 4)
        checks["max_rel_dist_err"] = exact_distance_error(X, Qall[:gt_n], ids_s, dist_s, cfg["metric"])

    # With several GPUs, each step shards the global batch by locality: every
    # rank orders the whole batch along the catalogue tour (Index.route, the
    # same order on every rank) and searches its contiguous slice of that order.
    routed = world > 1 and not args.positional and index.route(Qall) is not None
    if routed:
        import torch.distributed as dist
        o = index.route(Qall)
        sig = torch.tensor([float((o[:4096].double() * torch.arange(4096, device=dev)).sum()), float(o.sum())],
                           dtype=torch.float64, device=dev)
        lo, hi = sig.clone(), sig.clone()
        dist.all_reduce(lo, op=dist.ReduceOp.MIN)
        dist.all_reduce(hi, op=dist.ReduceOp.MAX)
        routed = bool(torch.equal(lo, hi))   # every rank sees the same verdict; else contiguous slices
        if routed:
            Q = Qall[o[a:b]].contiguous()   # this rank's routed shard (for the roofline leg)

    def step():
        if routed:
            order = index.route(Qall)
            return index.search_tensors(Qall[order[a:b]], k=cfg["k"], **op)
        return index.search_tensors(Q, k=cfg["k"], **op)

    # -- device-resident timing (value): strong scaling, the global batch split
    ms, clocks = timed_steps(step, args.steps, args.warmup, world, local)
    value = batch * args.steps / (ms / 1e3)

    # -- weak scaling beside it (N > 1): a full batch on every GPU ----------
    weak = None
    if world > 1:
        Qw = make_queries(cfg, dev, 2000 + rank, batch)   # a whole batch per GPU: nothing to route
        ms_w, _ = timed_steps(lambda: index.search_tensors(Qw, k=cfg["k"], **op), args.steps, args.warmup, world,
                              local, sample_clocks=False)
        weak = {"value": round(world * batch * args.steps / (ms_w / 1e3), 1), "unit": "queries/s",
                "batch_per_gpu": batch, "ms_per_step": round(ms_w / args.steps, 3)}
        del Qw

    # -- end to end through the public API with host buffers -------------
    # host batches are sharded by position (routing needs the batch on a GPU)
    Qh = Qall[a:b].cpu().pin_memory()
    for _ in range(max(1, args.warmup // 2)):
        index.search(Qh, k=cfg["k"], **op)
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        out_ids, out_d = index.search(Qh, k=cfg["k"], **op)
    torch.cuda.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t0, world)
    e2e = {"value": round(batch * args.steps / e2e_s, 1), "unit": "queries/s",
           "h2d_bytes_per_step": int(Qh.numel() * Qh.element_size()),
           "d2h_bytes_per_step": int(out_ids.nbytes + out_d.nbytes),
           "timing": "wall clock, host pinned queries to numpy answers, max over ranks",
           "sharding": "contiguous slices of the global batch"}

    # -- roofline of the dominant kernel (the fused search) on this rank's shard
    nq = Q.shape[0]
    ent = S.select_nearest(Q, index._cat, op["branches"], metric=index._m)
    seeds = index.catalogue[ent].to(torch.int32)
    order = index.locality_order(ent)   # the order Index.search runs the block in
    Qo, so = (Q[order].contiguous(), seeds[order].contiguous()) if order is not None else (Q, seeds)
    slots = index.table_slots_for(op["branches"], 64, op["queue"], op["stop_eps"], G.shape[1])
    kw = dict(k=cfg["k"], L=op["queue"], B=64, metric=index._m, team_size=16, stop_eps=op["stop_eps"],
              shared_cache=True, shared_bound=True, exclusive=2, elide_visited=True, table_slots=slots)
    _, _, ctr, _ = E.search_fused_lean(X, G, Qo, so, **kw)
    torch.cuda.synchronize()
    c = ctr.to(torch.int64)
    nodes = int(c[..., 5].sum()) + int(nq * op["branches"])      # claimed + seeds
    exps = int(c[..., 0].sum())
    claims = int((c[..., 5].sum(1) + op["branches"]).max())
    esize = X.element_size()
    alg_bytes = nodes * cfg["d"] * esize + exps * G.shape[1] * 4
    lib = E.N.lib()
    stream = torch.cuda.current_stream()
    Jq, kk = op["branches"], min(cfg["k"], op["queue"])
    cache = E._WS.get("cache", nq * slots, torch.int64, dev).view(nq, -1)
    bound = E._WS.get("bound", nq, torch.float32, dev)
    qdone = E._WS.get("qdone", nq, torch.int32, dev)
    bi = E._WS.get("branch_ids", nq * Jq * kk, torch.int32, dev)
    bd = E._WS.get("branch_dist", nq * Jq * kk, torch.float32, dev)
    oi = torch.empty((nq, cfg["k"]), dtype=torch.int32, device=dev)
    od = torch.empty((nq, cfg["k"]), dtype=torch.float32, device=dev)
    kt = []
    for _ in range(max(3, args.steps)):
        # prepare + fused, each bracketed by events on the launching stream
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        s = stream.cuda_stream
        ev[0].record(stream)
        E.N.check(lib.swb_search_prepare(nq, E.N.ptr(cache), slots, E.N.ptr(bound), E.N.ptr(qdone), s))
        ev[1].record(stream)
        rc = lib.swb_search_fused(
            E.N.ptr(X), E.N.dtype_code(X), X.shape[0], X.shape[1], E.N.ptr(G), G.shape[1], E.N.ptr(Qo),
            E.N.ptr(so), nq, Jq, 1, cfg["k"], op["queue"], 64, index._m, 16, 0, float(op["stop_eps"]),
            cfg["k"], None, 1, E.N.ptr(cache), slots, E.N.ptr(bound), 2, 0, 0.0, E.N.ptr(bi), E.N.ptr(bd),
            E.N.ptr(qdone), E.N.ptr(oi), E.N.ptr(od), None, None, None, None, None, None, s)
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
        same = prof.get("batch") == nq and prof.get("op") == [op["branches"], op["queue"], op["stop_eps"]]
        if same:
            traffic, traffic_src = prof["traffic_per_launch"], "ncu, this launch shape: " + prof["source"]
        else:   # same kernel and corpus, another batch or operating point: scale by this run's bytes
            traffic = round(prof["traffic_over_algorithmic"] * alg_bytes)
            traffic_src = "ncu traffic/algorithmic ratio %.3f (batch %s) x this run's algorithmic bytes (%s)" % (
                prof["traffic_over_algorithmic"], prof.get("batch"), prof["source"])
    roofline = {"bound": "hbm", "kernel": "swb::fused_kernel", "achieved": round(achieved, 1), "peak": peak,
                "unit": "GB/s", "frac": round(achieved / peak, 4), "peak_source": f"{peak_kind} hbm_gbs",
                "traffic": traffic, "traffic_source": traffic_src,
                # what DRAM itself moved per second (the measured traffic over this run's kernel time); the
                # algorithmic rate above also counts the rows that L2 serves to queries run side by side
                "dram_gbs": round(traffic / (fused_ms / 1e3) / 1e9, 1) if traffic else None,
                "dram_frac": round(traffic / (fused_ms / 1e3) / 1e9 / peak, 4) if traffic else None,
                "algorithmic_bytes_per_launch": alg_bytes, "kernel_ms": round(fused_ms, 3),
                "prepare_ms": round(prep_ms, 3), "launch_batch": nq,
                "per_query": {"distinct_nodes_scored": nodes / nq, "expansions": exps / nq}}
    table = {"slots": slots, "reference_slots": E.cache_size(op["branches"], 64, G.shape[1]),
             "max_claims_per_query": claims, "max_load": round(claims / slots, 4),
             "sizing": "Index default: measured claims x 1.5, a power of two (first call: the reference's size)"}

    line = {
        "metric": f"QPS at recall@10>={TARGET} ({cfg['desc']}, global batch {batch})",
        "value": round(value, 1), "unit": "queries/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded Gaussian mixture generated on the GPU, BASELINE.json config)",
        "config": {"workload": args.config, "n": cfg["n"], "d": cfg["d"], "storage": "f16" if cfg["half"] else "f32",
                   "metric": cfg["metric"], "global_batch": batch, "batch_per_gpu": b - a, "k": cfg["k"], **op,
                   "budget": 64, "team": 16, **checks, "recall_sample": gt_n,
                   "graph": "degree 64, candidates 128, alpha 1.2",
                   "catalogue": int(index.catalogue.numel()), "claims": "strict (exclusive=2)", "table": table,
                   "query_order": "nearest catalogue entry" if index.locality else "input",
                   "l2": "inputs larger than L2 (corpus %.1f GB; rows gathered at random)" % (
                       X.numel() * X.element_size() / 1e9),
                   "parallelism": f"query shards x{world}, replicas",
                   "sharding": ("by locality: each step orders the global batch along the catalogue tour "
                                "(Index.route, timed) and each rank searches its slice" if routed else
                                "contiguous slices of the global batch")},
        "e2e": e2e, "roofline": roofline, "clocks": clocks, "gpu_launches": 3 * args.steps,
        "gpu_launches_per_step": "sel::topk_kernel (seed top-E), swb::prepare_kernel (table clear), "
                                 "swb::fused_kernel (search); plus library GEMM/sort/gather launches",
        "build": {**{k: (round(v, 3) if isinstance(v, float) else v) for k, v in build_t.items()},
                  "roofline": sweep_roofline(build_t, cfg["n"], cfg["d"], cfg["half"]) if world == 1 else None},
        "calibration": [{"branches": b_, "queue": q, "stop_eps": e, "recall": round(r, 4),
                         "ms": None if t is None else round(t, 3)} for b_, q, e, r, t in tried],
    }
    if weak:
        line["weak"] = weak
    if rank == 0 and world == 1 and not args.no_cpu:
        # a sample spread over the batch in input order, with the seeds Index.search selects
        pick = torch.from_numpy(sample_rows(batch, 4096)).to(dev)
        Qs = Qall[pick].contiguous()
        sd = index.catalogue[S.select_nearest(Qs, index._cat, op["branches"], metric=index._m)].to(torch.int32)
        line["cpu_baseline"] = cpu_baseline(X, G, Qs, sd, cfg, op)
    if rank == 0 and world == 1 and not args.no_ref:
        del cache, bound, qdone, bi, bd
        E._WS.bufs.clear()
        torch.cuda.empty_cache()
        refk = reference_gpu_leg(X, G, index.catalogue, Qall, truth, gt_n, cfg, op)
        line["reference_kernel"] = refk
        if "qps" in refk:
            line["vs_reference_kernel"] = {"value_ratio": round(value / refk["qps"], 3),
                                           "e2e_ratio": round(e2e["value"] / refk["qps"], 3),
                                           "recall_delta": round(checks["recall@10"] - refk["recall@10"], 4)}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def tensor_peaks(seconds=3.0, n=8192):
    """Measured dense fp32 GEMM rates (the build's 3xTF32 sweep has no entry
    in MEASURED_PEAKS.json): torch.matmul fp32 with TF32 allowed, and without,
    best of 5 (burst) and back to back for `seconds` (sustained)."""
    a = torch.randn((n, n), device="cuda")
    b = torch.randn((n, n), device="cuda")
    out = {}
    prev = torch.backends.cuda.matmul.allow_tf32
    try:
        for name, tf32 in (("tf32", True), ("fp32", False)):
            torch.backends.cuda.matmul.allow_tf32 = tf32
            for _ in range(2):
                a @ b
            torch.cuda.synchronize()
            best = 1e9
            for _ in range(5):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                a @ b
                e1.record()
                torch.cuda.synchronize()
                best = min(best, e0.elapsed_time(e1))
            flops = 2.0 * n ** 3
            reps = max(1, int(seconds * 1e3 / best))
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                a @ b
            e1.record()
            torch.cuda.synchronize()
            out[f"{name}_tflops"] = round(flops / (best / 1e3) / 1e12, 1)
            out[f"{name}_tflops_sustained"] = round(flops * reps / (e0.elapsed_time(e1) / 1e3) / 1e12, 1)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    del a, b
    torch.cuda.empty_cache()
    return out


def candidate_parity(X, cand, cdist, rows=256, rel=1e-6, metric="l2", chunk=1 << 20):
    """Build parity at full size, for a sample of rows spread over the corpus:
    the sweep's candidate lists against the exact ones (every column, float64,
    the reference's expressions), and -- as the baseline the 1e-6 rule is held
    to -- the lists the reference's own arithmetic gives (swann/build.py:14-43:
    an fp32 GEMM without TF32, the same expressions in fp32, torch.topk).  A
    position where a list differs from the exact one counts as a tie when the
    two ids' exact distances differ by at most `rel` relative; every other
    difference is a mismatch.  Also: the same count against the reference's
    lists directly, and the largest relative gap between a list's own fp32
    distance and the exact one.  Columns are streamed in chunks with a running
    top list, so nothing of the corpus's size is held in float64."""
    n, C = cand.shape
    dev = X.device
    pick = torch.from_numpy(sample_rows(n, rows)).to(dev)
    m = len(pick)
    A64 = X[pick].double()
    an64 = (A64 * A64).sum(1)
    Af = X[pick].float()
    an32 = (Af * Af).sum(1)
    ar = torch.arange(m, device=dev)
    best = [None, None]    # exact: distances, ids (running, (C + 8) per row)
    refb = [None, None]    # the reference's fp32 arithmetic
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for c0 in range(0, n, chunk):
            c1 = min(n, c0 + chunk)
            Xc = X[c0:c1]
            X64 = Xc.double()
            dots = A64 @ X64.T
            D = 1.0 - dots if metric == "ip" else (((X64 * X64).sum(1))[None, :] - 2.0 * dots + an64[:, None]).clamp(min=0)
            Xf = Xc.float()
            s32 = Af @ Xf.T
            R = 1.0 - s32 if metric == "ip" else ((Xf * Xf).sum(1)[None, :] - 2.0 * s32 + an32[:, None]).clamp(min=0)
            inside = (pick >= c0) & (pick < c1)
            D[ar[inside], pick[inside] - c0] = 3.4e38
            R[ar[inside], pick[inside] - c0] = 3.4e38
            for acc, M, kk in ((best, D, C + 8), (refb, R, C)):
                v, i = torch.topk(M, min(kk, c1 - c0), dim=1, largest=False)
                i = i + c0
                if acc[0] is not None:
                    v, j = torch.topk(torch.cat([acc[0], v], 1), kk, dim=1, largest=False)
                    i = torch.gather(torch.cat([acc[1], i], 1), 1, j)
                acc[0], acc[1] = v, i
            del dots, D, R, X64, Xf, s32
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    ed, ei = best
    order = torch.from_numpy(np.lexsort((ei.cpu().numpy(), ed.cpu().numpy()), axis=1)).to(dev)
    ei = torch.gather(ei, 1, order)[:, :C]
    rd, ri = refb

    def exact(ids):
        """exact distances of the rows' listed ids (float64)"""
        V = X[ids.reshape(-1)].double().view(m, C, -1)
        if metric == "ip":
            return 1.0 - (V * A64[:, None, :]).sum(-1)
        return ((V - A64[:, None, :]) ** 2).sum(-1)

    d_ex, d_ref = exact(ei), exact(ri)
    mine = cand[pick].long()
    d_mine = exact(mine)

    def compare(got, dg, want, dw):
        diff = got != want
        tie = (dg - dw).abs() <= rel * dw.abs()
        return int((diff & ~tie).sum()), int((diff & tie).sum())

    m_ex, t_ex = compare(mine, d_mine, ei, d_ex)
    r_ex, rt_ex = compare(ri, d_ref, ei, d_ex)
    m_ref, t_ref = compare(mine, d_mine, ri, d_ref)
    gap_mine = float(((cdist[pick].double() - d_mine).abs() / d_mine.abs().clamp(min=1e-30)).max())
    gap_ref = float(((rd.double() - d_ref).abs() / d_ref.abs().clamp(min=1e-30)).max())
    return {"rows_checked": int(m), "positions": int(m * C), "tie_rule": f"exact distances within {rel:g} relative",
            "vs_exact": {"non_tie_mismatches": m_ex, "tie_swaps": t_ex},
            "reference_fp32_vs_exact": {"non_tie_mismatches": r_ex, "tie_swaps": rt_ex},
            "vs_reference_fp32": {"non_tie_mismatches": m_ref, "tie_swaps": t_ref},
            "max_rel_dist_gap": {"sweep": gap_mine, "reference_fp32": gap_ref},
            "exact": "float64 on the GPU, every column", "reference_fp32": "fp32 GEMM (no TF32) + the reference's "
                                                                           "expressions + torch.topk"}


def run_build(args):
    """Graph build seconds (sweep / prune / reverse) on one GPU, the sweep
    against the tensor pipe (measured sustained bf16 for fp16 rows; for fp32
    rows both a sixth of it and a third of the measured sustained TF32 GEMM
    rate), and the candidate lists of a row sample against the exact ones."""
    world, rank, local = dist_setup()
    dev = torch.device("cuda", local)
    cfg = dict(CONFIGS[args.config])
    from swann_b200 import build as B
    peaks_fp32 = tensor_peaks() if not cfg["half"] else None
    X = make_corpus(cfg, dev)
    torch.cuda.synchronize()
    n, d = X.shape
    with ClockSampler(local) as clk:
        t0 = time.perf_counter()
        ops = B.TcOperands(X)
        cand, cd = B.knn_candidates(X, 128, metric=cfg["metric"], ops=ops)
        torch.cuda.synchronize()
        t1 = time.perf_counter()
    G1 = B.robust_prune(X, cand, cd, 64, alpha=1.2, metric=cfg["metric"], ops=ops)
    torch.cuda.synchronize()
    t2 = time.perf_counter()
    G = B.add_reverse(X, G1, 64, alpha=1.2, metric=cfg["metric"], ops=ops)
    torch.cuda.synchronize()
    t3 = time.perf_counter()
    recomputed = int(ops.recomputed[0])
    del ops
    roof = sweep_roofline({"sweep_s": t1 - t0}, n, d, cfg["half"])
    if peaks_fp32:
        roof["measured_fp32_gemm"] = peaks_fp32
        roof["frac_of_tf32_sustained_over_3"] = round(roof["achieved"] / (peaks_fp32["tf32_tflops_sustained"] / 3), 4)
    prune_flops = 2.0 * n * 128 * 128 * d
    line = {"metric": f"graph build seconds ({cfg['desc']}, degree 64, candidates 128, alpha 1.2)",
            "value": round(t3 - t0, 3), "unit": "s", "n_gpus": world, "higher_is_better": False,
            "data": "synthetic (seeded Gaussian mixture generated on the GPU, BASELINE.json config)",
            "config": {"workload": args.config, "n": n, "d": d, "storage": "f16" if cfg["half"] else "f32",
                       "metric": cfg["metric"], "sweep": os.environ.get("SWB_SWEEP", "mma")},
            "stages_s": {"sweep": round(t1 - t0, 3), "prune": round(t2 - t1, 3), "reverse": round(t3 - t2, 3)},
            "roofline": roof,
            "prune_tflops": round(prune_flops / (t2 - t1) / 1e12, 1),
            "prune": B._prune_method(None, cfg["metric"]), "exact_recomputed_pairs": recomputed,
            "clocks_during_sweep": clk.summary(),
            "mean_out_degree": round(float((G >= 0).sum(1).float().mean()), 2)}
    line["candidate_parity"] = candidate_parity(X, cand, cd, metric=cfg["metric"])
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_reference(args):
    """The reference arm: the reference package, unmodified, from baseline/_ref.
    Its own build (swann/build.py build_graph, torch on the GPU) makes the
    graph, its own Index selects the seeds and -- on its own kernels --
    chooses the operating point (the fastest reaching recall@10 >= 0.95), and
    the timed number is its CPU search path (swann/_refcpu.py, restated in C
    by the oracle) on the host cores, on samples spread over the batch in
    input order.  This package's library is never loaded here."""
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
    swann_ref = reference_package()
    if swann_ref is None:
        print(json.dumps({"impl": "reference", "unavailable": "the reference package is not installed under "
                                                              "baseline/_ref (baseline/install.sh)"}), flush=True)
        return
    from swann import _select as RS
    from swann import build as RB
    from oracle import oracle as O
    impl = reference_kernels_for(swann_ref)
    X = make_corpus(cfg, dev)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    G = RB.build_graph(X, metric=cfg["metric"], degree=64, candidates=128, alpha=1.2)
    torch.cuda.synchronize()
    build_s = time.perf_counter() - t0
    index = swann_ref.Index(X, G, metric=cfg["metric"], catalogue_size=cfg.get("catalogue", 4096))
    Qall = make_queries(cfg, dev, 1000, cfg["batch"])
    gt_n = min(cfg["batch"], args.gt)
    truth = exact_topk(X, Qall[:gt_n], cfg["k"], cfg["metric"])

    def ref_search(Qs, k, branches, queue, eps):
        return index.search(Qs, k=k, branches=branches, queue=queue, stop_eps=eps)[0]

    op, tried = choose_op(args, ref_search, Qall[:gt_n], truth, cfg, 0, 1)
    ids, _ = index.search(Qall[:gt_n], k=cfg["k"], **op)
    rec = recall(ids[:, :10], truth[:, :10], 10)
    gpu_s = time_reference_gpu(index, Qall, cfg["k"], op)
    ent = RS.select_nearest(Qall, index._cat, op["branches"], metric=index._m)
    seeds = index.catalogue[ent].to(torch.int32)
    Xh = X.float().cpu().numpy()
    Gh, Qh, Sh = G.cpu().numpy(), Qall.cpu().numpy(), seeds.cpu().numpy()
    cores = O.cpu_count()
    metric = 0 if cfg["metric"] == "ip" else 1
    kw = dict(k=cfg["k"], L=op["queue"], B=64, metric=metric, team=16, vec=8 if cfg["half"] else 4,
              stop_eps=op["stop_eps"], kstop=min(cfg["k"], op["queue"]), threads=cores)
    per = cores * 16                                       # ~0.3 s of host work a step
    steps = args.warmup + args.steps
    order = sample_rows(Qh.shape[0], per * steps)          # spread over the batch, input order
    times = []
    for i in range(steps):
        pick = order[i::steps][:per]
        t = time.perf_counter()
        O.search(Xh, Gh, Qh[pick], Sh[pick], **kw)
        if i >= args.warmup:
            times.append((time.perf_counter() - t, len(pick)))
    el = sum(t for t, _ in times)
    value = sum(m for _, m in times) / el
    line = {"metric": f"QPS at recall@10>={TARGET} ({cfg['desc']}, global batch {cfg['batch']})",
            "value": round(value, 2), "unit": "queries/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "impl": "reference",
            "data": "synthetic (seeded Gaussian mixture generated on the GPU, BASELINE.json config)",
            "config": {"workload": args.config, "n": cfg["n"], "d": cfg["d"], **op, "budget": 64, "team": 16,
                       "recall@10": round(rec, 4), "recall_sample": gt_n},
            "cpu_baseline": {"value": round(value, 2), "unit": "queries/s", "cores": cores, "kind": "port",
                             "sample": f"{per} queries per step spread over the batch in input order (C restatement "
                                       f"of swann/_refcpu.py, independent branches, {cores} threads); graph by the "
                                       f"reference's build_graph, seeds by its select_nearest, operating point "
                                       f"calibrated on its own GPU kernels beforehand, untimed"},
            "e2e": {"value": round(value, 2), "unit": "queries/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "reference_gpu": {"qps": round(Qall.shape[0] / gpu_s, 1), "ms_per_batch": round(gpu_s * 1e3, 3),
                              "impl": "swann/index.py Index.search over " + impl},
            "build_s": round(build_s, 3),
            "calibration": [{"branches": b_, "queue": q, "stop_eps": e, "recall": round(r, 4),
                             "ms": None if t is None else round(t, 3)} for b_, q, e, r, t in tried]}
    print(json.dumps(line), flush=True)


# C3's batch schedule: branches 128 up to batch 64, 64 at
# 512, 32 from 4096 on
BATCH_SWEEP = [(1, 128), (8, 128), (64, 128), (512, 64), (4096, 32), (65535, 32)]


def wall_per_batch(call, b, nmax, reps):
    """Median wall-clock seconds of one synchronous call(a) over consecutive
    slices [a, a + b) of an nmax-query set, after one untimed call."""
    call(0)
    torch.cuda.synchronize()
    ts = []
    for i in range(reps):
        a = ((i + 1) * b) % (nmax - b + 1)
        t = time.perf_counter()
        call(a)
        torch.cuda.synchronize()
        ts.append(time.perf_counter() - t)
    return statistics.median(ts)


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
    Q = make_queries(cfg, dev, 1000, nmax)
    gt_n = min(nmax, args.gt)
    truth = exact_topk(X, Q[:gt_n], cfg["k"], cfg["metric"])
    ops = {}
    for _, br in BATCH_SWEEP:
        if br in ops:
            continue
        for eps in EPS:
            ids, _ = index.search_tensors(Q[:gt_n], k=cfg["k"], branches=br, queue=12, stop_eps=eps)
            r = recall(ids.cpu().numpy()[:, :10], truth[:, :10], 10)
            if r >= TARGET:
                break
        ops[br] = (eps, r)   # the index now sizes this configuration's table from the claims it measured
    rows = []
    for b, br in BATCH_SWEEP:
        eps, r = ops[br]
        slots = index.table_slots_for(br, 64, 12, eps, G.shape[1])
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
        wall = wall_per_batch(lambda a: index.search(Q[a:a + b], **kw), b, nmax, min(reps, 50))
        rows.append({"batch": b, "branches": br, "queue": 12, "stop_eps": eps, "recall@10": round(r, 4),
                     "table_slots": slots,
                     "ms_per_batch": round(ms, 3), "qps": round(b / (ms / 1e3), 1), "batches_timed": reps,
                     "wall_ms_per_batch": round(wall * 1e3, 3)})
    swann_ref = None if args.no_ref else reference_package()
    if swann_ref is not None:
        # the reference's own Index.search on the same graph, catalogue and
        # operating points, timed like `wall_ms_per_batch` above
        impl = reference_kernels_for(swann_ref)
        ref_index = swann_ref.Index(X, G, metric=cfg["metric"], catalogue=index.catalogue)
        ref_recall = {}
        for row in rows:
            kw = dict(k=cfg["k"], branches=row["branches"], queue=12, stop_eps=row["stop_eps"])
            key = (row["branches"], row["stop_eps"])
            if key not in ref_recall:
                ids, _ = ref_index.search(Q[:gt_n], **kw)
                ref_recall[key] = recall(ids[:, :10], truth[:, :10], 10)
            b = row["batch"]
            sec = wall_per_batch(lambda a: ref_index.search(Q[a:a + b], **kw), b, nmax,
                                 max(3, min(50, nmax // b)))
            row["reference"] = {"wall_ms_per_batch": round(sec * 1e3, 3), "qps": round(b / sec, 1),
                                "recall@10": round(ref_recall[key], 4)}
        del ref_index
        torch.cuda.empty_cache()
    else:
        impl = None
    line = {"metric": f"QPS and latency by batch size at recall@10>={TARGET} ({cfg['desc']})",
            "unit": "queries/s", "n_gpus": 1, "higher_is_better": True, "dtype": "f32",
            "data": "synthetic (seeded Gaussian mixture generated on the GPU, BASELINE.json config)",
            "config": {"workload": args.config, "n": cfg["n"], "d": cfg["d"], "k": cfg["k"], "budget": 64,
                       "team": 16, "recall_sample": gt_n,
                       "timing": "ms_per_batch: CUDA events over back-to-back calls, device-resident queries; "
                                 "wall_ms_per_batch: median wall clock of one synchronous Index.search call "
                                 "(device-resident queries, numpy answers), the reference timed the same way"},
            "reference": impl or "not run (--no-ref, or the reference package is not installed)",
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
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline (and build parity) legs")
    ap.add_argument("--no-ref", action="store_true", help="skip the reference-kernel leg")
    ap.add_argument("--positional", action="store_true", help="N > 1: shard the batch by position, not locality")
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
