"""Host-side logic that needs no GPU: sizing formulas, the tensor definition of
the merge, configuration and errors, and the multi-rank drivers over gloo
(two CPU ranks, the oracle standing in for the per-rank kernels)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import cases
import swann_b200 as swann
from oracle import oracle as O
from swann_b200 import _engine as E
from swann_b200 import dist as D
from swann_b200.index import SearchConfig


def test_sizing_formulas_match_reference():
    """swann/_engine.py:73-77 and :186-198, at the configurations the
    reference and BASELINE use."""
    assert E.visited_size(64, 64) == 16384
    assert E.visited_size(16, 32) == 2048
    assert E.cache_size(32, 64, 64) == 131072
    assert E.cache_size(64, 64, 64) == 262144
    assert E.cache_size(128, 64, 64) == 524288
    assert E.cache_size(3, 12, 32) == 1024


def test_search_config_defaults():
    c = SearchConfig()
    assert (c.branches, c.queue, c.budget, c.stop_eps, c.team, c.k) == (32, 12, 64, 0.05, 16, 10)


def test_tensor_merge_matches_oracle_on_cpu():
    ids, dist_ = cases.merge_inputs(Q=25, J=7, kk=10, seed=4)
    oi, od = O.merge_branches(ids, dist_, 10)
    ti, td = E._merge_branches_tensor(torch.from_numpy(ids), torch.from_numpy(dist_), 10)
    assert np.array_equal(ti.numpy(), oi) and np.array_equal(td.numpy(), od)


def test_overflow_guard_returns_old_setting():
    was = swann.overflow_guard(False)
    try:
        assert swann.overflow_guard(False) is False
    finally:
        swann.overflow_guard(was)


def test_index_rejects_host_vectors():
    with pytest.raises(ValueError, match="GPU"):
        swann.Index(torch.zeros((10, 8)), torch.zeros((10, 4), dtype=torch.int32))


def test_shard_bounds_cover_exactly():
    for n in (0, 1, 7, 100, 65535):
        for w in (1, 2, 3, 8):
            b = D.shard_bounds(n, w)
            assert b[0][0] == 0 and b[-1][1] == n
            assert all(b[i][1] == b[i + 1][0] for i in range(w - 1))
            assert max(e - s for s, e in b) - min(e - s for s, e in b) <= 1


# -- multi-rank drivers over gloo ------------------------------------------------

def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, which, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        if which == "search":
            X, G = cases.toy(n=1500, d=32, deg=16, seed=9)
            Q = cases.unit_queries(37, 32, 9)
            seeds = np.random.default_rng(9).integers(0, X.shape[0], (37, 4)).astype(np.int32)
            Qt = torch.from_numpy(Q)
            qidx = torch.arange(37)

            def fn(Qs):
                # the shard's rows of Q identify its queries
                sel = qidx[[int(np.nonzero((Q == q.numpy()).all(1))[0][0]) for q in Qs]]
                ids, dd = O.search(X, G, Qs.numpy(), seeds[sel.numpy()], k=10, L=12, B=16, team=8)
                return torch.from_numpy(ids), torch.from_numpy(dd)

            ids, dd = D.search_sharded(fn, Qt, 10)
            if rank == 0:
                np.savez(out_path, ids=ids.numpy(), dist=dd.numpy())
        else:
            n, d = 900, 24
            X = cases.build_corpus(n, d, seed=3, metric=1)
            a, b = D.shard_bounds(n, world)[rank]
            Xl = torch.from_numpy(X[a:b].copy())

            def sweep(Xf, r0, r1):
                c, cd = O.knn_candidates(Xf.numpy(), 32, 1, rows=(r0, r1))
                return torch.from_numpy(c), torch.from_numpy(cd)

            def prune(Xf, c, cd):
                return torch.from_numpy(O.robust_prune(Xf.numpy(), c.numpy(), cd.numpy(), 16, 1.2, 1))

            def reverse(Xf, G1, r0, r1):
                return torch.from_numpy(O.add_reverse(Xf.numpy(), G1.numpy(), 16, 1.2, 64, 1)[r0:r1].copy())

            Xall, G = D.build_sharded(Xl, n, sweep, prune, reverse)
            assert torch.equal(Xall, torch.from_numpy(X))
            if rank == 0:
                np.save(out_path, G.numpy())
    finally:
        dist.destroy_process_group()


def _spawn(which, tmp_path, world=2):
    out = str(tmp_path / f"{which}.npz" if which == "search" else tmp_path / f"{which}.npy")
    port = _free_port()
    mp.start_processes(_rank_main, args=(world, port, which, out), nprocs=world, join=True, start_method="spawn")
    return out


def test_sharded_search_equals_single_process(tmp_path):
    """Two gloo ranks each search half the batch; the gathered result is the
    single-process result, in query order."""
    out = _spawn("search", tmp_path)
    got = np.load(out)
    X, G = cases.toy(n=1500, d=32, deg=16, seed=9)
    Q = cases.unit_queries(37, 32, 9)
    seeds = np.random.default_rng(9).integers(0, X.shape[0], (37, 4)).astype(np.int32)
    ids, dd = O.search(X, G, Q, seeds, k=10, L=12, B=16, team=8)
    assert np.array_equal(got["ids"], ids) and np.array_equal(got["dist"], dd)


def test_sharded_build_equals_single_process(tmp_path):
    """Row-block build over two gloo ranks (corpus tiles all-gathered, pruned
    rows all-gathered before the reverse pass) equals the one-process build."""
    out = _spawn("build", tmp_path)
    G = np.load(out)
    X = cases.build_corpus(900, 24, seed=3, metric=1)
    want = O.build_graph(X, metric=1, degree=16, candidates=32)
    assert np.array_equal(G, want)


def test_bench_corpus_row_blocks_equal_the_whole():
    """bench.py's seeded generator: the rows a rank generates for its block of a
    sharded build are exactly those rows of the single-process corpus, at
    block edges that do not fall on the generator's 65536-row chunks."""
    import bench
    full = bench.gen_mixture(150_000, 8, 7, 1, torch.device("cpu"), False, True)
    for a, b in ((0, 1), (70_000, 140_000), (65_535, 65_537), (131_071, 150_000)):
        part = bench.gen_mixture(150_000, 8, 7, 1, torch.device("cpu"), False, True, rows=(a, b))
        assert torch.equal(part, full[a:b]), (a, b)


@pytest.mark.parametrize("metric", ["ip", "l2"])
def test_two_level_tour_orders_cells_along_the_coarse_walk(monkeypatch, metric):
    """A catalogue above TOUR_MAX gets the two-level tour: a permutation in
    which every cell (the entries nearest one walked entry) is contiguous, the
    cells follow the coarse walk, and consecutive entries are near each other."""
    from swann_b200 import index as I
    monkeypatch.setattr(I, "TOUR_MAX", 300)
    monkeypatch.setattr(I, "TOUR_COARSE", 64)
    g = torch.Generator().manual_seed(3)
    centres = torch.randn((40, 16), generator=g) * 3
    V = centres[torch.randint(0, 40, (2000,), generator=g)] + 0.3 * torch.randn((2000, 16), generator=g)
    if metric == "ip":
        V = V / V.norm(dim=1, keepdim=True)
    m = I.METRICS[metric]
    pos = I._catalogue_tour(V, m)
    assert torch.equal(torch.sort(pos).values, torch.arange(2000))
    walk = torch.argsort(pos)                       # entries in tour order
    C = V[torch.linspace(0, 1999, 64).round().long()]
    cpos = torch.from_numpy(I._greedy_walk(I._entry_distances(C, C, m).numpy()))
    cell = cpos[I._entry_distances(V, C, m).argmin(1)]
    along = cell[walk]
    assert bool((along[1:] >= along[:-1]).all())    # cells in coarse-walk order, each contiguous
    D = I._entry_distances(V, V, m)
    step = D[walk[:-1], walk[1:]].mean()
    rand = D[torch.randint(0, 2000, (4000,), generator=g), torch.randint(0, 2000, (4000,), generator=g)].mean()
    assert float(step) < 0.5 * float(rand)


def test_small_catalogue_tour_is_the_greedy_walk():
    from swann_b200 import index as I
    g = torch.Generator().manual_seed(4)
    V = torch.randn((200, 8), generator=g)
    pos = I._catalogue_tour(V, I.METRICS["l2"])
    assert torch.equal(pos, torch.from_numpy(I._greedy_walk(I._entry_distances(V, V, I.METRICS["l2"]).numpy())))
