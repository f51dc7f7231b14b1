"""The search entry point that allocates nothing (swb_search_fused_static).

It serves callers that cannot give the library device memory for scratch --
a host runtime whose memory manager owns the whole device heap and forbids raw
cudaMalloc, or a latency-critical serving thread that must never call an
allocator.  Its scratch is one fixed array compiled into the library.

Checked here through the C ABI, against the existing entry point
(swb_search_fused with caller-provided scratch) on the same inputs, bit for bit
in a deterministic mode, on two calls in a row with different queries (so
scratch left over by the first call would show up in the second), plus the
clear rejection of a batch too large for the fixed array.
"""
import numpy as np
import pytest
import torch

import cases
from swann_b200 import _engine as E
from swann_b200 import _lib as N

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _static_search(Xg, Gg, Qg, seeds, k, L, B, team, Hc, shared_cache, shared_bound, exclusive, elide):
    Q, J = seeds.shape
    ids = torch.empty((Q, k), dtype=torch.int32, device=DEV)
    dist = torch.empty((Q, k), dtype=torch.float32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    rc = N.lib().swb_search_fused_static(
        N.ptr(Xg), N.dtype_code(Xg), Xg.shape[0], Xg.shape[1], N.ptr(Gg), Gg.shape[1], N.ptr(Qg), N.ptr(seeds),
        Q, J, k, L, B, 1, team, 0.05, int(shared_cache), int(shared_bound), int(exclusive), int(elide), Hc,
        N.ptr(ids), N.ptr(dist), N.ptr(status), N.stream_of(Xg))
    N.check(rc, "swb_search_fused_static")
    torch.cuda.synchronize()
    assert int(status[0]) == 0
    return ids, dist


def test_static_scratch_matches_caller_scratch_on_two_calls():
    X, G = cases.toy(n=2000, d=64, deg=32, seed=13, metric=1)
    Xg, Gg = torch.from_numpy(X).to(DEV), torch.from_numpy(G).to(DEV)
    rng = np.random.default_rng(2)
    k, L, B, team, Hc = 10, 16, 12, 16, 2048
    for call in range(2):
        # a different batch each call: stale table entries from the previous
        # call would change the second call's distances
        Q = rng.standard_normal((37 + call, X.shape[1]), dtype=np.float32)
        seeds = rng.integers(0, X.shape[0], (Q.shape[0], 6)).astype(np.int32)
        Qg, sd = torch.from_numpy(Q).to(DEV), torch.from_numpy(seeds).to(DEV)
        # deterministic mode: the shared table only changes how much is computed
        want_i, want_d, _, _ = E.search_fused_lean(Xg, Gg, Qg, sd, k=k, L=L, B=B, metric=1, team_size=team,
                                                   stop_eps=0.05, shared_cache=True, table_slots=Hc)
        got_i, got_d = _static_search(Xg, Gg, Qg, sd, k, L, B, team, Hc, True, False, 0, False)
        assert torch.equal(got_i, want_i), f"call {call}: ids differ"
        assert torch.equal(got_d, want_d), f"call {call}: distances differ"


def test_static_scratch_production_mode_returns_exact_distances():
    """Shared table, bound and strict claims (Index.search's mode): results are
    timing dependent, so they are checked for validity -- every id distinct and
    every distance the exact one -- on two calls in a row."""
    X, G = cases.toy(n=2000, d=64, deg=32, seed=17, metric=1)
    Xg, Gg = torch.from_numpy(X).to(DEV), torch.from_numpy(G).to(DEV)
    rng = np.random.default_rng(5)
    for call in range(2):
        Q = rng.standard_normal((50, X.shape[1]), dtype=np.float32)
        seeds = rng.integers(0, X.shape[0], (50, 8)).astype(np.int32)
        Qg, sd = torch.from_numpy(Q).to(DEV), torch.from_numpy(seeds).to(DEV)
        ids, dist = _static_search(Xg, Gg, Qg, sd, 10, 12, 64, 16, 4096, True, True, 2, True)
        ids, dist = ids.cpu().numpy(), dist.cpu().numpy()
        assert (ids >= 0).all()
        for q in range(50):
            assert len(set(ids[q])) == 10
            ex = ((Q[q][None, :].astype(np.float64) - X[ids[q]].astype(np.float64)) ** 2).sum(1)
            assert np.allclose(dist[q], ex, rtol=1e-5)


def test_static_scratch_rejects_oversized_batches():
    X, G = cases.toy(n=500, d=16, deg=8, seed=3, metric=1)
    Xg, Gg = torch.from_numpy(X).to(DEV), torch.from_numpy(G).to(DEV)
    Q = np.zeros((4096, 16), np.float32)
    seeds = np.zeros((4096, 32), np.int32)
    need = N.lib().swb_search_static_bytes(4096, 32, 10, 12, 64, 8, 65536, 1, 2, 1)
    assert need > (32 << 20)
    with pytest.raises(ValueError, match="fixed scratch"):
        _static_search(Xg, Gg, torch.from_numpy(Q).to(DEV), torch.from_numpy(seeds).to(DEV), 10, 12, 64, 16,
                       65536, True, True, 2, True)
