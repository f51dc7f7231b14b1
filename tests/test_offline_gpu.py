"""The offline builder's extras on the GPU (swann_b200.offline, csrc/offline.cu,
the prune's per-node degrees and protection) against the oracle, on the inputs
of tests/golden/offline.npz (the reference's own outputs pin the oracle in
test_offline_golden.py)."""
from pathlib import Path

import numpy as np
import pytest
import torch

import cases
from oracle import offline_ref as R
from oracle import oracle as O
from swann_b200 import build as B
from swann_b200 import offline as F

pytestmark = pytest.mark.gpu
DEV = "cuda"


def load(metric):
    g = np.load(Path(cases.__file__).resolve().parent / "offline.npz")
    N, D = int(g["params"][0]), int(g["params"][1])
    X = cases.build_corpus(N, D, seed=21 + metric, metric=metric)
    return g, X, ("ip" if metric == 0 else "l2")


def t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


@pytest.mark.parametrize("metric", [0, 1])
def test_mutual_rank(metric):
    g, X, name = load(metric)
    got = F.mutual_rank(t(g[f"{name}_cand"]), int(g["params"][3])).cpu().numpy().astype(np.uint8)
    assert np.array_equal(got, g[f"{name}_mutual"])


@pytest.mark.parametrize("metric", [0, 1])
@pytest.mark.parametrize("rule", ["near", "far", "bridge"])
def test_fill_degree(metric, rule):
    g, X, name = load(metric)
    chunk = int(g["params"][7])
    got = F.fill_degree(t(g[f"{name}_reverse"]), t(g[f"{name}_cand"]), rule=rule, chunk=chunk).cpu().numpy()
    assert np.array_equal(got, g[f"{name}_fill_{rule}"])


@pytest.mark.parametrize("metric", [0, 1])
def test_enforce_min_in_equals_oracle(metric):
    g, X, name = load(metric)
    min_in = int(g["params"][6])
    want, stats = R.enforce_min_in(g[f"{name}_reverse"], g[f"{name}_cand"], min_in, rounds=4)
    G = t(g[f"{name}_reverse"])
    F.enforce_min_in(t(X), G, t(g[f"{name}_cand"]), min_in, rounds=4)
    assert np.array_equal(G.cpu().numpy(), want)
    got_stats = [[s["below"], s["to_place"], s["placed"], s["already_linked"]] for s in F.enforce_min_in.last_stats]
    assert got_stats == stats


@pytest.mark.parametrize("metric", [0, 1])
def test_graph_candidates(metric):
    g, X, name = load(metric)
    idx, dst = F.candidates_from_graph(t(X), t(g[f"{name}_gc"]), 32, metric=name)
    want_i, want_d = R.graph_candidates(X, g[f"{name}_gc"], 32, metric)
    idx, dst = idx.cpu().numpy(), dst.cpu().numpy()
    tol = 4e-6 * (1.0 if metric == 0 else float((X.astype(np.float64) ** 2).sum(1).max()) * 4)
    assert np.allclose(dst, want_d, rtol=1e-5, atol=tol)
    for r in np.nonzero((idx != want_i).any(1))[0]:
        bad = idx[r] != want_i[r]
        assert np.all(np.abs(dst[r][bad] - want_d[r][bad]) <= tol + 1e-6 * np.abs(want_d[r][bad]))


@pytest.mark.parametrize("metric", [0, 1])
def test_prune_with_node_degrees_and_protection_bitexact(metric):
    g, X, name = load(metric)
    cand, cd, dpn, prot = g[f"{name}_cand"], g[f"{name}_cdist"], g[f"{name}_dpn"], g[f"{name}_mutual"]
    deg = int(g["params"][4])
    want = O.robust_prune(X, cand, cd, deg, 1.2, metric, deg_per_node=dpn, protect=prot)
    got = B.robust_prune(t(X), t(cand), t(cd), deg, alpha=1.2, deg_per_node=t(dpn), metric=name,
                         protect=t(prot).bool()).cpu().numpy()
    assert np.array_equal(got, want)


@pytest.mark.parametrize("metric", [0, 1])
def test_reverse_with_node_degrees_bitexact(metric):
    g, X, name = load(metric)
    dpn, Gp = g[f"{name}_dpn"], g[f"{name}_prune"]
    deg = int(g["params"][4])
    want = O.add_reverse(X, Gp, deg, 1.2, 64, metric, deg_per_node=dpn)
    got = B.add_reverse(t(X), t(Gp), deg, alpha=1.2, deg_per_node=t(dpn), metric=name).cpu().numpy()
    assert np.array_equal(got, want)


def test_offline_pipeline_end_to_end():
    X = cases.build_corpus(3000, 64, seed=4, metric=0)
    pool = np.arange(0, 3000, 50)
    # pool boost, mutual protection and the in-degree floor: caps hold
    G, info = F.build_graph_offline(X, D=24, cand=64, metric="ip", pool=pool, pool_boost=8, mutual=8, min_in=12)
    G = G.cpu().numpy()
    assert G.shape == (3000, 32)
    deg = (G >= 0).sum(1)
    assert deg[pool].max() > 24 and (np.delete(deg, pool) <= 24).all()
    assert all(len(set(r[r >= 0])) == (r >= 0).sum() for r in G[:200])
    rounds = info["min_in_rounds"]
    assert rounds and rounds[0]["placed"] > 0 and info["seconds"] > 0
    below_after = int((np.bincount(G[G >= 0], minlength=3000) < 12).sum())
    assert below_after < rounds[0]["below"]
    # the fill spends every empty slot of the (pool-wide) rows it can
    Gf, _ = F.build_graph_offline(X, D=24, cand=64, metric="ip", pool=pool, pool_boost=8, fill="near")
    Gf = Gf.cpu().numpy()
    assert ((Gf >= 0).sum(1) >= (G >= 0).sum(1) - 8).all() and (Gf >= 0).sum() > (G >= 0).sum()
