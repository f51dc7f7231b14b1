"""Seeded inputs shared by the golden-vector generator and the tests.

Every input is derived from ``np.random.default_rng(seed)``, so a fixture stores
only outputs plus a digest of its inputs; a test regenerates the inputs and
checks the digest before comparing, which catches a generator drift instead of
reporting it as a parity failure.
"""
from __future__ import annotations

import hashlib

import numpy as np

METRIC_IP, METRIC_L2 = 0, 1


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()[:16]


def toy(n=2000, d=64, deg=32, seed=0, metric=METRIC_IP):
    """A small corpus and its exact kNN graph (unit rows for inner product).
    The shape of the reference's own engine-test corpus."""
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((n, d), dtype=np.float32)
    if metric == METRIC_IP:
        X /= np.linalg.norm(X, axis=1, keepdims=True)
    X = np.ascontiguousarray(X, dtype=np.float32)
    if metric == METRIC_IP:
        sim = X @ X.T
    else:
        sq = (X * X).sum(1)
        sim = -(sq[:, None] - 2.0 * (X @ X.T) + sq[None, :])
    np.fill_diagonal(sim, -np.inf)
    G = np.ascontiguousarray(np.argsort(-sim, axis=1, kind="stable")[:, :deg].astype(np.int32))
    return X, G


def unit_queries(nq, d, seed):
    rng = np.random.default_rng(seed)
    Q = rng.standard_normal((nq, d), dtype=np.float32)
    Q /= np.linalg.norm(Q, axis=1, keepdims=True)
    return np.ascontiguousarray(Q)


def distance_pairs(d, seed, count=3):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((count, d), dtype=np.float32)
    x = rng.standard_normal((count, d), dtype=np.float32)
    return q, x


DIST_GRID = [(d, team, vec, metric)
             for d in (16, 48, 64, 100, 128, 960, 1536)
             for team in (4, 8, 16, 32)
             for vec in (4, 8)
             for metric in (METRIC_IP, METRIC_L2)
             if not (vec == 8 and d % 8)]


def c1_data():
    """n=10,000, d=128, fp32 N(0,1) rows, 100 queries, L2."""
    rng = np.random.default_rng(0)
    X = rng.standard_normal((10000, 128), dtype=np.float32)
    Q = rng.standard_normal((100, 128), dtype=np.float32)
    return np.ascontiguousarray(X), np.ascontiguousarray(Q)


def catalogue(n, size=4096, seed=0):
    """swann/index.py:64-69: the sorted first `size` of a seeded permutation."""
    rng = np.random.default_rng(seed)
    return np.sort(rng.permutation(n)[:min(size, n)]).astype(np.int64)


def build_corpus(n, d, seed, metric):
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((n, d), dtype=np.float32)
    if metric == METRIC_IP:
        X /= np.linalg.norm(X, axis=1, keepdims=True)
    return np.ascontiguousarray(X, dtype=np.float32)


def merge_inputs(Q=7, J=5, kk=10, seed=3):
    """Branch results with repeats across branches and empty slots: what the
    merge sees when branches share a distance table."""
    rng = np.random.default_rng(seed)
    pool = rng.integers(0, 60, size=(Q, 40))
    dpool = rng.random((Q, 60)).astype(np.float32)
    ids = np.empty((Q, J, kk), np.int32)
    dist = np.empty((Q, J, kk), np.float32)
    for q in range(Q):
        for j in range(J):
            pick = rng.choice(pool[q], size=kk, replace=False) if len(set(pool[q])) >= kk else pool[q][:kk]
            ids[q, j] = pick
            dist[q, j] = dpool[q, pick]
            o = np.lexsort((ids[q, j], dist[q, j]))
            ids[q, j], dist[q, j] = ids[q, j][o], dist[q, j][o]
            nempty = rng.integers(0, 3)
            if nempty:
                ids[q, j, kk - nempty:] = -1
                dist[q, j, kk - nempty:] = np.finfo(np.float32).max
    return ids, dist


def aniso_mixture(n, d, clusters, seed, nq=0, qseed=None):
    """BASELINE config 3's corpus model at any size: `clusters` centres
    N(0, 1)^d, per-cluster per-dimension scales exp(U(ln 0.1, ln 1)), rows
    c + s * z, L2-normalised.  Returns (X float32 [n, d], Q float32 [nq, d]),
    the queries drawn from the same mixture with their own seed."""
    g = np.random.default_rng(seed)
    centres = g.standard_normal((clusters, d), dtype=np.float32)
    scales = np.exp(np.log(0.1) + (np.log(1.0) - np.log(0.1)) * g.random((clusters, d), dtype=np.float32))

    def draw(m, rng):
        c = rng.integers(0, clusters, m)
        x = centres[c] + scales[c] * rng.standard_normal((m, d), dtype=np.float32)
        x /= np.linalg.norm(x, axis=1, keepdims=True)
        return np.ascontiguousarray(x, dtype=np.float32)

    X = draw(n, np.random.default_rng(seed + 1))
    Q = draw(nq, np.random.default_rng(seed + 2 if qseed is None else qseed)) if nq else None
    return X, Q


def iso_mixture(n, d, clusters, seed, sigma=0.3):
    """BASELINE config 5's corpus model (and config 2's): `clusters` centres
    N(0, 1)^d, isotropic sigma, float32, not normalised (an L2 corpus)."""
    g = np.random.default_rng(seed)
    centres = g.standard_normal((clusters, d), dtype=np.float32)
    c = g.integers(0, clusters, n)
    X = centres[c] + sigma * g.standard_normal((n, d), dtype=np.float32)
    return np.ascontiguousarray(X, dtype=np.float32)
