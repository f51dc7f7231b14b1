"""Corpus directories: the on-disk layout the reference's bench and offline
tools read and write (offline/prep_annbench.py:91-125, offline/prep_fvecs.py:
60-115, offline/prep_parquet.py:83-105), and the sign-code files
`swann_b200._engine.load_codes` reads (swann/_engine.py:320-337).

    X.npy                 float32 [n, d]  (d padded with zeros to a multiple of 8;
                                           rows L2-normalised for inner product)
    Q_test.npy            float32 [nq, d] (and Q_val.npy / qidx_{val,test}.npy
                                           when the queries are split)
    gt_<split>_ids.npy    int32   [nq, k] exact top-k
    gt_<split>_sim.npy    float32 [nq, k] inner product, or minus the euclidean
                                          distance (prep_fvecs.py:96-105)
    G.npy                 int32   [n, deg] a graph, when one is given
    manifest.json         corpus, n, d, d_original, k, seed, source, metric
                          ("ip_on_l2_normalised" | "sqeuclidean"), [deg, graph]
    codes_<name>.npy      int32   [n, ceil(d / 32)] sign code
    alpha_<name>.npy      float32 [n]     per-node scale
    mu_<name>.npy         float32 [d]     corpus mean

The reference ships no writer for the code files (its offline/build_codes.py
is missing); `write_codes` defines them from what the reader and the kernel
expect: b_i = +1 (bit i set) when x_i > mu_i, else -1, and alpha = |x - mu|_1 / d,
so alpha * <q, b> + <q, mu> estimates <q, x>.
"""
from __future__ import annotations

import json
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np
import torch

METRIC_NAMES = {"ip": "ip_on_l2_normalised", "l2": "sqeuclidean"}


def _device(device):
    if device is not None:
        return torch.device(device)
    return torch.device("cuda" if torch.cuda.is_available() else "cpu")


def _pad8(A: np.ndarray) -> np.ndarray:
    pad = (-A.shape[1]) % 8
    return np.pad(A, ((0, 0), (0, pad))) if pad else A


def _normalise(A: torch.Tensor) -> torch.Tensor:
    return A / A.norm(dim=1, keepdim=True).clamp(min=1e-12)


@torch.no_grad()
def exact_ground_truth(X, Q, k: int, metric: str = "ip", device=None, block: int = 256):
    """Exact top-k of every query, in blocks of queries (the score matrix never
    exists whole).  Returns (ids int32 [nq, k], sim float32 [nq, k]): the inner
    product for "ip", minus the euclidean distance for "l2"."""
    dev = _device(device)
    Xg = torch.as_tensor(np.asarray(X, dtype=np.float32)).to(dev)
    Qg = torch.as_tensor(np.asarray(Q, dtype=np.float32)).to(dev)
    nq, k = Qg.shape[0], min(k, Xg.shape[0])
    ids = np.empty((nq, k), np.int32)
    sim = np.empty((nq, k), np.float32)
    for s in range(0, nq, block):
        e = min(s + block, nq)
        if metric == "ip":
            v, i = torch.topk(Qg[s:e] @ Xg.T, k, dim=1, largest=True)
        else:
            v, i = torch.topk(torch.cdist(Qg[s:e], Xg), k, dim=1, largest=False)
            v = -v
        ids[s:e], sim[s:e] = i.cpu().numpy(), v.cpu().numpy()
    return ids, sim


def write_corpus(out, X, queries, metric: str = "ip", k: int = 100, name: str = "corpus", seed: int = 0,
                 split: bool = False, graph=None, source: str = "", device=None) -> Path:
    """Write a corpus directory.  Rows and queries are padded to a multiple of
    8 dimensions and, for inner product, L2-normalised (zero rows stay zero).
    split=True halves the queries at random (seeded) into val and test, as
    prep_annbench.py:83-97 does; otherwise they are all test queries."""
    if metric not in METRIC_NAMES:
        raise ValueError(f"metric must be one of {sorted(METRIC_NAMES)}")
    out = Path(out)
    out.mkdir(parents=True, exist_ok=True)
    X = np.ascontiguousarray(np.asarray(X, dtype=np.float32))
    Q = np.ascontiguousarray(np.asarray(queries, dtype=np.float32))
    if Q.shape[1] != X.shape[1]:
        raise ValueError(f"queries are {Q.shape[1]}-dimensional, the corpus {X.shape[1]}")
    d0 = X.shape[1]
    X, Q = _pad8(X), _pad8(Q)
    if metric == "ip":
        X = _normalise(torch.from_numpy(X)).numpy()
        Q = _normalise(torch.from_numpy(Q)).numpy()
    np.save(out / "X.npy", X)
    splits = {"test": Q}
    if split:
        perm = np.random.default_rng(seed).permutation(Q.shape[0])
        half = Q.shape[0] // 2
        val, test = np.sort(perm[:half]), np.sort(perm[half:])
        splits = {"val": Q[val], "test": Q[test]}
        np.save(out / "qidx_val.npy", val)
        np.save(out / "qidx_test.npy", test)
    for sp, Qs in splits.items():
        np.save(out / f"Q_{sp}.npy", Qs)
        gi, gv = exact_ground_truth(X, Qs, k, metric, device)
        np.save(out / f"gt_{sp}_ids.npy", gi)
        np.save(out / f"gt_{sp}_sim.npy", gv)
    man = {"corpus": name, "n": int(X.shape[0]), "d": int(X.shape[1]), "d_original": int(d0), "k": int(k),
           "seed": int(seed), "source": str(source), "metric": METRIC_NAMES[metric]}
    if graph is not None:
        G = np.ascontiguousarray(np.asarray(graph.cpu() if isinstance(graph, torch.Tensor) else graph,
                                            dtype=np.int32))
        if G.shape[0] != X.shape[0]:
            raise ValueError("the graph has a row per corpus row")
        np.save(out / "G.npy", G)
        man.update(deg=int(G.shape[1]), graph="given")
    (out / "manifest.json").write_text(json.dumps(man, indent=2))
    return out


@dataclass
class Corpus:
    path: Path
    manifest: dict
    X: np.ndarray
    queries: dict = field(default_factory=dict)        # split -> [nq, d]
    gt_ids: dict = field(default_factory=dict)         # split -> [nq, k]
    gt_sim: dict = field(default_factory=dict)
    G: np.ndarray | None = None

    @property
    def metric(self) -> str:
        """"ip" or "l2", the name swann_b200.Index takes."""
        return "ip" if self.manifest["metric"].startswith("ip") else "l2"


def read_corpus(path, mmap: bool = False) -> Corpus:
    """Load a corpus directory (numpy arrays; `mmap` maps X instead of reading it)."""
    path = Path(path)
    man = json.loads((path / "manifest.json").read_text())
    X = np.load(path / "X.npy", mmap_mode="r" if mmap else None)
    c = Corpus(path=path, manifest=man, X=X)
    for sp in ("val", "test"):
        if (path / f"Q_{sp}.npy").exists():
            c.queries[sp] = np.load(path / f"Q_{sp}.npy")
        if (path / f"gt_{sp}_ids.npy").exists():
            c.gt_ids[sp] = np.load(path / f"gt_{sp}_ids.npy")
            c.gt_sim[sp] = np.load(path / f"gt_{sp}_sim.npy")
    if (path / "G.npy").exists():
        c.G = np.load(path / "G.npy")
    return c


def read_vecs(path, n: int = 0) -> np.ndarray:
    """.fvecs (float32), .ivecs (int32) or .bvecs (uint8) rows, each prefixed by
    its int32 dimension; the first n rows (all when n = 0)."""
    path = Path(path)
    ext = path.suffix.lower()
    dt, size = {".fvecs": (np.float32, 4), ".ivecs": (np.int32, 4), ".bvecs": (np.uint8, 1)}[ext]
    raw = np.fromfile(path, dtype=np.uint8)
    if raw.size == 0:
        return np.empty((0, 0), dt)
    d = int(raw[:4].view(np.int32)[0])
    rec = 4 + d * size
    rows = raw.size // rec
    if n:
        rows = min(rows, n)
    body = raw[: rows * rec].reshape(rows, rec)
    if not (body[:, :4].copy().view(np.int32)[:, 0] == d).all():
        raise ValueError(f"{path.name}: rows of different dimensions")
    return np.ascontiguousarray(body[:, 4:]).view(dt).reshape(rows, d)


def prep_fvecs(base, queries, out, metric: str = "l2", n: int = 0, nq: int = 10000, k: int = 100,
               name: str | None = None, seed: int = 0, device=None) -> Path:
    """A corpus directory from .fvecs/.bvecs files (offline/prep_fvecs.py):
    the first n base rows, the first nq queries, exact ground truth."""
    X = read_vecs(base, n).astype(np.float32)
    Q = read_vecs(queries, nq).astype(np.float32)
    return write_corpus(out, X, Q, metric=metric, k=k, name=name or Path(base).stem, seed=seed,
                        source=str(base), device=device)


@torch.no_grad()
def build_codes(X, device=None, chunk: int = 1 << 16):
    """The 1-bit sign code of every row around the corpus mean.
    Returns (codes int32 [n, ceil(d / 32)], alpha float32 [n], mu float32 [d]):
    bit i of row v is set when x_vi > mu_i; alpha_v = |x_v - mu|_1 / d."""
    dev = _device(device)
    Xt = X if isinstance(X, torch.Tensor) else torch.from_numpy(np.asarray(X))
    n, d = Xt.shape
    words = (d + 31) // 32
    mu = torch.zeros(d, dtype=torch.float64, device=dev)
    for s in range(0, n, chunk):
        mu += Xt[s:s + chunk].to(dev, torch.float64).sum(0)
    mu = (mu / max(n, 1)).float()
    codes = torch.empty((n, words), dtype=torch.int32, device=dev)
    alpha = torch.empty(n, dtype=torch.float32, device=dev)
    weights = (torch.ones(32, dtype=torch.int64, device=dev) << torch.arange(32, device=dev))
    for s in range(0, n, chunk):
        diff = Xt[s:s + chunk].to(dev, torch.float32) - mu
        alpha[s:s + diff.shape[0]] = diff.abs().sum(1) / d
        bits = torch.zeros((diff.shape[0], words * 32), dtype=torch.int64, device=dev)
        bits[:, :d] = (diff > 0).to(torch.int64)
        packed = (bits.view(-1, words, 32) * weights).sum(-1)            # 0 .. 2^32 - 1
        codes[s:s + diff.shape[0]] = (packed - ((packed >> 31) << 32)).to(torch.int32)
    return codes, alpha, mu


def write_codes(out, X, name: str = "1bit", device=None):
    """Write codes_<name>.npy, alpha_<name>.npy, mu_<name>.npy for X into a
    corpus directory; returns the three arrays (as load_codes will read them)."""
    out = Path(out)
    codes, alpha, mu = build_codes(X, device)
    np.save(out / f"codes_{name}.npy", codes.cpu().numpy())
    np.save(out / f"alpha_{name}.npy", alpha.cpu().numpy())
    np.save(out / f"mu_{name}.npy", mu.cpu().numpy())
    return codes, alpha, mu
