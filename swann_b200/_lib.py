"""Loads libswann_b200.so and binds its C ABI (include/swann_b200.h) with ctypes.

This module is the only place Python touches the native library.  There is no
fallback: if the library is missing or a call fails, the caller gets an
exception, never a silent CPU path.  Tensors are passed as raw device pointers
with the current torch stream of their device.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libswann_b200.so"

OK, ERR_ARG, ERR_TEAM, ERR_SMEM, ERR_BATCH, ERR_CUDA, ERR_TIMEOUT = range(7)
F32, F16 = 0, 1

_vp, _i32, _i64, _u64, _f32 = C.c_void_p, C.c_int, C.c_int64, C.c_uint64, C.c_float

# name -> (restype, argtypes), exactly the declarations of include/swann_b200.h
SIGNATURES = {
    "swb_search_init": (_i32, [_vp, _i32, _i64, _i32, _vp, _vp, _i32, _i32, _i32,
                               _vp, _vp, _vp, _vp, _i32, _vp, _i32, _vp, _i32, _i32,
                               _vp, _i32, _vp, _vp]),
    "swb_search_advance": (_i32, [_vp, _i32, _i64, _i32, _vp, _i32, _vp,
                                  _vp, _vp, _vp, _vp, _i32, _i32, _i32,
                                  _vp, _i32, _vp, _i32, _i32, _i32, _i32,
                                  _i32, _i32, _f32, _i32, _vp, _i32, _vp, _i32,
                                  _i32, _f32, _vp, _i32, _vp, _vp, _vp, _f32, _i32, _vp, _vp]),
    "swb_merge_branches": (_i32, [_vp, _vp, _i32, _i32, _i32, _i32, _vp, _vp, _vp]),
    "swb_search_prepare": (_i32, [_i32, _vp, _i32, _vp, _vp, _vp]),
    "swb_graph_candidates": (_i32, [_vp, _i64, _i32, _vp, _i32, _i32, _i32, _vp, _vp, _vp]),
    "swb_mutual_rank": (_i32, [_vp, _i64, _i32, _i32, _vp, _vp]),
    "swb_fill_degree": (_i32, [_vp, _i64, _i32, _vp, _i32, _i32, _i32, _vp, _vp]),
    "swb_min_in_workspace": (_u64, [_i64]),
    "swb_enforce_min_in": (_i32, [_vp, _i64, _i32, _vp, _i32, _i32, _i32, _vp, _u64, _vp, _vp, _vp]),
    "swb_select_topk": (_i32, [_vp, _i64, _i32, _i64, _vp, _vp, _i32, _i32, _i32, _vp, _vp, _i32, _vp]),
    "swb_search_fused": (_i32, [_vp, _i32, _i64, _i32, _vp, _i32, _vp, _vp,
                                _i32, _i32, _i32, _i32, _i32, _i32,
                                _i32, _i32, _i32, _f32, _i32, _vp, _i32,
                                _vp, _i32, _vp, _i32, _i32, _f32,
                                _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "swb_search_fused_static": (_i32, [_vp, _i32, _i64, _i32, _vp, _i32, _vp, _vp, _i32, _i32, _i32, _i32, _i32,
                                       _i32, _i32, _f32, _i32, _i32, _i32, _i32, _i32, _vp, _vp, _vp, _vp]),
    "swb_search_static_bytes": (_u64, [_i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32]),
    "swb_topc_block": (_i32, [_vp, _i64, _i64, _i64, _i64, _i64, _vp, _i32, _i32, _vp, _vp, _i32, _vp]),
    "swb_row_norms": (_i32, [_vp, _i32, _i64, _i32, _vp, _vp]),
    "swb_sweep_topc": (_i32, [_vp, _vp, _i32, _i64, _i32, _vp, _i64, _i64, _i32, _i32, _vp, _vp, _vp, _u64,
                              _vp, _vp]),
    "swb_sweep_workspace": (_u64, [_i64, _i64, _i32, _i32]),
    "swb_split_tf32": (_i32, [_vp, _i64, _vp, _vp, _vp]),
    "swb_prune": (_i32, [_vp, _i64, _i32, _vp, _vp, _i64, _i32, _i32, _f32, _i32, _vp, _vp, _vp, _vp]),
    "swb_reverse": (_i32, [_vp, _i64, _i32, _vp, _i32, _f32, _i32, _i32, _vp, _i64, _i64, _vp, _vp, _u64, _vp]),
    "swb_reverse_workspace": (_u64, [_i64, _i64, _i32, _i32]),
    "swb_prune_tc": (_i32, [_vp, _vp, _vp, _i32, _i32, _vp, _i64, _i32, _vp, _vp, _i64, _i32, _i32, _f32, _i32,
                            _vp, _vp, _vp, _vp, _vp, _vp]),
    "swb_reverse_tc": (_i32, [_vp, _vp, _vp, _i32, _i32, _vp, _i64, _i32, _vp, _i32, _f32, _i32, _i32, _vp, _i64,
                              _i64, _vp, _vp, _u64, _vp, _vp, _vp]),
    "swb_last_error": (C.c_char_p, []),
    "swb_version": (_i32, []),
}

_LIB = None


class SwannError(RuntimeError):
    """A native call failed; `code` is the SWB_ERR_* status."""

    def __init__(self, code, msg):
        super().__init__(msg)
        self.code = code


def lib():
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH.name} is not built; run `python -m swann_b200._build` "
                "(there is no CPU fallback)")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def check(rc: int, what: str = "") -> None:
    if rc == OK:
        return
    msg = lib().swb_last_error().decode(errors="replace")
    if rc in (ERR_ARG, ERR_TEAM, ERR_BATCH):
        raise ValueError(f"{what}: {msg}" if what else msg)
    raise SwannError(rc, f"{what}: {msg}" if what else msg)


def ptr(t) -> int | None:
    """Raw device pointer of a tensor (None for None or an empty tensor)."""
    if t is None or t.numel() == 0:
        return None
    return t.data_ptr()


def stream_of(t) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def dtype_code(X) -> int:
    if X.dtype == torch.float32:
        return F32
    if X.dtype == torch.float16:
        return F16
    raise ValueError("vectors must be float32 or float16")
