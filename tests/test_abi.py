"""The C ABI: the library loads without a GPU and exports every symbol the
headers in include/ declare, with the bindings' argument counts matching the
declarations.  No compute calls (no GPU needed)."""
import re
from pathlib import Path

import pytest

from swann_b200 import _lib as N

ROOT = Path(__file__).resolve().parent.parent


def declared():
    """(name, n_params) of every SWB_API function in include/*.h."""
    out = []
    for h in sorted((ROOT / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"SWB_API\s+[\w\s\*]+?\b(swb_\w+)\s*\(([^)]*)\)\s*;", text, flags=re.S):
            params = m.group(2).strip()
            n = 0 if params in ("", "void") else params.count(",") + 1
            out.append((m.group(1), n))
    return out


def test_headers_declare_something():
    names = [n for n, _ in declared()]
    assert "swb_search_fused" in names and "swb_prune" in names and len(names) >= 10


@pytest.mark.parametrize("name,nparams", declared())
def test_symbol_exported_and_bound(name, nparams):
    L = N.lib()
    assert hasattr(L, name), f"{name} declared but not exported"
    assert name in N.SIGNATURES, f"{name} has no ctypes binding"
    assert len(N.SIGNATURES[name][1]) == nparams, f"{name}: binding has {len(N.SIGNATURES[name][1])} params"


def test_version_and_error_string():
    L = N.lib()
    assert L.swb_version() >= 1
    assert isinstance(L.swb_last_error(), bytes)


def test_argument_errors_need_no_gpu():
    """Validation happens before any CUDA call: a bad team size or a batch
    over the limit is rejected with its own code."""
    L = N.lib()
    rc = L.swb_search_advance(1 << 20, 0, 10, 8, 1 << 20, 4, 1 << 20, 1 << 20, 1 << 20, 1 << 20, 1 << 20,
                              1, 1, 8, 1 << 20, 1, 1 << 20, 0, 12, 1, 1, 0, 1, -1.0, 10, None, 0, None, 0,
                              0, 0.0, None, 0, None, None, None, 0.0, 0, None, None)
    assert rc == N.ERR_TEAM
    assert b"team" in L.swb_last_error()
    rc = L.swb_search_init(1 << 20, 0, 10, 8, 1 << 20, 1 << 20, 70000, 1, 1, 1 << 20, 1 << 20, 1 << 20, 1 << 20, 8,
                           1 << 20, 1, 1 << 20, 0, 16, None, 0, None, None)
    assert rc == N.ERR_BATCH
    assert b"65535" in L.swb_last_error()
    rc = L.swb_search_init(1 << 20, 0, 10, 6, 1 << 20, 1 << 20, 1, 1, 1, 1 << 20, 1 << 20, 1 << 20, 1 << 20, 8,
                           1 << 20, 1, 1 << 20, 0, 16, None, 0, None, None)
    assert rc == N.ERR_ARG
    with pytest.raises(ValueError):
        N.check(rc)


def test_static_scratch_sizing_rejects_out_of_range_knobs():
    """The no-allocation entry point sizes its scratch in 64 bits and rejects
    knobs outside the kernels' limits before touching the GPU: a budget and
    degree whose visited table would pass 2^30 slots, a degree beyond the
    limit, a batch beyond 65535."""
    L = N.lib()
    assert L.swb_search_static_bytes(16, 8, 10, 12, 64, 64, 4096, 1, 2, 1) < (32 << 20)
    assert L.swb_search_static_bytes(1, 1, 10, 12, 1 << 24, 128, 0, 0, 0, 0) == 2 ** 64 - 1
    assert L.swb_search_static_bytes(1, 1, 10, 12, 64, 129, 0, 0, 0, 0) == 2 ** 64 - 1
    args = dict(X=1 << 20, G=1 << 20, Q=1 << 20, S=1 << 20)
    rc = L.swb_search_fused_static(args["X"], 0, 1000, 64, args["G"], 200, args["Q"], args["S"], 4, 4, 10, 12, 64,
                                   0, 16, 0.05, 1, 1, 2, 1, 4096, 1 << 20, 1 << 20, None, None)
    assert rc == N.ERR_ARG and b"degree" in L.swb_last_error()
    rc = L.swb_search_fused_static(args["X"], 0, 1000, 64, args["G"], 64, args["Q"], args["S"], 4, 1, 10, 12,
                                   1 << 24, 0, 16, 0.05, 0, 0, 0, 0, 0, 1 << 20, 1 << 20, None, None)
    assert rc == N.ERR_ARG and b"2^30" in L.swb_last_error()
    rc = L.swb_search_fused_static(args["X"], 0, 1000, 64, args["G"], 64, args["Q"], args["S"], 70000, 4, 10, 12,
                                   64, 0, 16, 0.05, 1, 1, 2, 1, 4096, 1 << 20, 1 << 20, None, None)
    assert rc == N.ERR_BATCH


def test_refext_keeps_the_reference_signatures():
    """swann_b200.refext exposes the reference's three pybind entry points
    (swann/csrc/local_search.cu:950-955) with their argument lists, and its
    argument errors are RuntimeErrors, as the reference's TORCH_CHECKs are."""
    import inspect

    import torch

    from swann_b200 import refext
    assert list(inspect.signature(refext.init_states).parameters) == [
        "X", "Qv", "seeds", "ids", "dist", "expd", "lin", "visited", "counters", "metric", "team_size",
        "cache_id", "cache_d", "bound"]
    assert list(inspect.signature(refext.advance).parameters) == [
        "X", "G", "Qv", "ids", "dist", "expd", "lin", "visited", "counters", "metric", "team_size", "delta",
        "max_expansions", "policy", "V_in", "stop_eps", "kstop", "cache_id", "cache_d", "bound", "exclusive",
        "stall_patience", "crowd_frac", "active", "codes", "alpha", "cmu", "code_margin"]
    assert list(inspect.signature(refext.merge_branches).parameters) == ["bids", "bdist", "k"]
    t = torch.zeros((2, 1, 4))
    with pytest.raises(RuntimeError, match="X: contiguous cuda"):
        refext.init_states(t, t, t, t, t, t, t, t, t, 0, 16, t, t, t)
