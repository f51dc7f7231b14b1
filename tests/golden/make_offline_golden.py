"""Golden vectors for the offline builder's extras, by running the REFERENCE's
own offline/build_graph.py (read-only import) on small CPU tensors:
candidates_from_graph, mutual_rank, robust_prune with per-node degrees and
protected pairs, add_reverse with per-node degrees, fill_degree (all three
rules, 64-row chunks so the chunk order matters) and enforce_min_in.

    python tests/golden/make_offline_golden.py [--ref REFERENCE_ROOT]

Writes tests/golden/offline.npz.  Runs only where the reference is mounted.
"""
from __future__ import annotations

import argparse
import os
import contextlib
import io
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import cases  # noqa: E402

N, D, C, M, DEG, BOOST, MIN_IN, CHUNK = 600, 32, 48, 12, 16, 8, 8, 64


def test_graph(cand, seed):
    """An approximate graph to take candidates from: the candidate lists with
    holes (-1) and a node's own id in some rows."""
    rng = np.random.default_rng(seed)
    Gc = cand[:, :40].copy()
    Gc[rng.random(Gc.shape) < 0.1] = -1
    rows = rng.choice(N, 40, replace=False)
    Gc[rows, 3] = rows
    return Gc


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("SWANN_REFERENCE"),
                    help="root of the reference project (default: $SWANN_REFERENCE)")
    a = ap.parse_args()
    if not a.ref:
        ap.error("name the reference project's root with --ref or $SWANN_REFERENCE")
    sys.path.insert(0, a.ref)
    import torch
    from offline import build_graph as R   # the reference's module, unmodified

    out = {}
    pool = np.arange(0, N, 12)
    for metric, name in ((0, "ip"), (1, "l2")):
        X = cases.build_corpus(N, D, seed=21 + metric, metric=metric)
        Xg = torch.from_numpy(X)
        cand, cdist = R.knn_candidates(Xg, C, chunk=256, metric=name)
        Gc = test_graph(cand.numpy(), 5 + metric)
        gi, gd = R.candidates_from_graph(Xg, torch.from_numpy(Gc), 32, metric=name, chunk=128)
        mut = R.mutual_rank(cand, M, chunk=256)
        dpn = torch.full((N,), DEG, dtype=torch.int32)
        dpn[torch.from_numpy(pool)] = min(DEG + BOOST, min(C, 128))
        Gp = R.robust_prune(Xg, cand, cdist, DEG, alpha=1.2, chunk=256, deg_per_node=dpn, metric=name,
                            protect=mut)
        Gr = R.add_reverse(Xg, Gp, DEG, chunk=256, alpha=1.2, deg_per_node=dpn, metric=name)
        fills = {rule: R.fill_degree(Gr, cand, rule=rule, chunk=CHUNK) for rule in ("near", "far", "bridge")}
        with contextlib.redirect_stdout(io.StringIO()):
            Gm = R.enforce_min_in(Xg, Gr.clone(), cand, MIN_IN, metric=name, rounds=4)
        out.update({
            f"{name}_cand": cand.numpy().astype(np.int32), f"{name}_cdist": cdist.numpy().astype(np.float32),
            f"{name}_gc": Gc.astype(np.int32), f"{name}_gc_idx": gi.numpy().astype(np.int32),
            f"{name}_gc_dst": gd.numpy().astype(np.float32), f"{name}_mutual": mut.numpy().astype(np.uint8),
            f"{name}_dpn": dpn.numpy(), f"{name}_prune": Gp.numpy().astype(np.int32),
            f"{name}_reverse": Gr.numpy().astype(np.int32), f"{name}_min_in": Gm.numpy().astype(np.int32),
            f"{name}_x_digest": np.array([cases.digest(X)]),
        })
        for rule, G in fills.items():
            out[f"{name}_fill_{rule}"] = G.numpy().astype(np.int32)
    out["pool"] = pool
    out["params"] = np.array([N, D, C, M, DEG, BOOST, MIN_IN, CHUNK])
    np.savez_compressed(HERE / "offline.npz", **out)
    print("wrote", HERE / "offline.npz", sorted(out))


if __name__ == "__main__":
    main()
