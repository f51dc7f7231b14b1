"""Corpus directories and sign codes on the CPU: the layout the reference's
offline tools write (offline/prep_annbench.py:91-125, prep_fvecs.py:60-115) and
the code files load_codes reads (swann/_engine.py:320-337)."""
import json

import numpy as np
import pytest
import torch

from swann_b200 import _engine as E
from swann_b200 import corpus as C


def _data(n=200, d=13, nq=20, seed=0):
    rng = np.random.default_rng(seed)
    return rng.standard_normal((n, d)).astype(np.float32), rng.standard_normal((nq, d)).astype(np.float32)


@pytest.mark.parametrize("metric", ["ip", "l2"])
def test_corpus_round_trip(tmp_path, metric):
    X, Q = _data()
    G = np.arange(200 * 4, dtype=np.int32).reshape(200, 4) % 200
    C.write_corpus(tmp_path, X, Q, metric=metric, k=5, name="toy", graph=G, device="cpu")
    c = C.read_corpus(tmp_path)
    man = json.loads((tmp_path / "manifest.json").read_text())
    assert man["metric"] == C.METRIC_NAMES[metric] and c.metric == metric
    assert (man["n"], man["d"], man["d_original"], man["k"], man["deg"]) == (200, 16, 13, 5, 4)
    assert c.X.shape == (200, 16) and c.X.dtype == np.float32
    assert (c.X[:, 13:] == 0).all()
    Xp = np.pad(X, ((0, 0), (0, 3)))
    Qp = np.pad(Q, ((0, 0), (0, 3)))
    if metric == "ip":
        Xp /= np.linalg.norm(Xp, axis=1, keepdims=True)
        Qp /= np.linalg.norm(Qp, axis=1, keepdims=True)
        assert np.allclose(np.linalg.norm(c.X, axis=1), 1.0, atol=1e-6)
        s = Qp @ Xp.T
        truth = np.argsort(-s, axis=1, kind="stable")[:, :5]
        assert np.allclose(c.gt_sim["test"], np.take_along_axis(s, truth, 1), atol=1e-5)
    else:
        dd = np.sqrt(((Qp[:, None, :] - Xp[None]) ** 2).sum(-1))
        truth = np.argsort(dd, axis=1, kind="stable")[:, :5]
        assert np.allclose(c.gt_sim["test"], -np.take_along_axis(dd, truth, 1), atol=1e-4)
    assert (c.gt_ids["test"] == truth).all()
    assert c.gt_ids["test"].dtype == np.int32
    assert (c.G == G).all() and c.G.dtype == np.int32


def test_corpus_split_into_val_and_test(tmp_path):
    X, Q = _data(nq=21)
    C.write_corpus(tmp_path, X, Q, metric="ip", k=3, split=True, seed=4, device="cpu")
    c = C.read_corpus(tmp_path)
    val, test = np.load(tmp_path / "qidx_val.npy"), np.load(tmp_path / "qidx_test.npy")
    assert len(val) == 10 and len(test) == 11
    assert sorted(np.concatenate([val, test]).tolist()) == list(range(21))
    assert c.queries["val"].shape == (10, 16) and c.gt_ids["val"].shape == (10, 3)


def test_vecs_reader_and_prep(tmp_path):
    rng = np.random.default_rng(1)
    base = rng.standard_normal((50, 12)).astype(np.float32)
    qs = rng.standard_normal((7, 12)).astype(np.float32)

    def write(path, A, dt):
        with open(path, "wb") as f:
            for row in A:
                np.int32(A.shape[1]).tofile(f)
                row.astype(dt).tofile(f)

    write(tmp_path / "b.fvecs", base, np.float32)
    write(tmp_path / "q.fvecs", qs, np.float32)
    assert np.array_equal(C.read_vecs(tmp_path / "b.fvecs"), base)
    assert np.array_equal(C.read_vecs(tmp_path / "b.fvecs", n=9), base[:9])
    u8 = rng.integers(0, 255, (5, 16)).astype(np.uint8)
    write(tmp_path / "u.bvecs", u8, np.uint8)
    assert np.array_equal(C.read_vecs(tmp_path / "u.bvecs"), u8)
    out = C.prep_fvecs(tmp_path / "b.fvecs", tmp_path / "q.fvecs", tmp_path / "corp", metric="l2", k=4,
                       device="cpu")
    c = C.read_corpus(out)
    assert c.X.shape == (50, 16) and c.gt_ids["test"].shape == (7, 4) and c.metric == "l2"


def test_codes_match_their_definition(tmp_path):
    rng = np.random.default_rng(3)
    X = rng.standard_normal((300, 70)).astype(np.float32)   # 70 dims: 3 words, the last partly used
    X[:, 31] += 5.0                                          # bit 31 set on most rows: negative int32 words
    codes, alpha, mu = C.build_codes(X, device="cpu")
    mu_ref = X.astype(np.float64).mean(0).astype(np.float32)
    assert np.allclose(mu.numpy(), mu_ref, atol=1e-6)
    diff = X - mu.numpy()
    assert np.allclose(alpha.numpy(), np.abs(diff).sum(1) / 70, rtol=1e-6)
    words = codes.numpy().view(np.uint32)
    assert words.shape == (300, 3)
    for i in range(70):
        bit = (words[:, i // 32] >> (i % 32)) & 1
        assert (bit == (diff[:, i] > 0)).all(), i
    assert ((words[:, 2] >> 6) == 0).all()                   # dims 70..95 do not exist
    assert (codes.numpy()[:, 0] < 0).any()
    C.write_codes(tmp_path, X, device="cpu")
    (tmp_path / "manifest.json").write_text(json.dumps({"metric": "ip_on_l2_normalised"}))
    cd, al, cm, margin = E.load_codes(tmp_path, device="cpu")
    assert torch.equal(cd, codes) and torch.equal(al, alpha) and torch.equal(cm, mu) and margin == 0.20
