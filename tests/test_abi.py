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
