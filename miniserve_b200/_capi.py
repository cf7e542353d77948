"""ctypes binding of libmsattn.so (the C ABI declared in include/msattn.h).

The library is the only compute path: if it is missing or fails to load, every call raises.
There is no CPU or PyTorch fallback.
"""

from __future__ import annotations

import ctypes as C
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libmsattn.so"

MS_OK = 0
MS_ERR_ARG = 1
MS_ERR_LAYOUT = 2
MS_ERR_PLAN = 3
MS_ERR_CUDA = 4
MS_ERR_CAPACITY = 5

DEV_BAD_SLOT = 1
DEV_BAD_BLOCK = 2
DEV_TIMEOUT = 4
DEV_BAD_POSITION = 8

# Every symbol include/msattn.h declares, for the export check.
EXPORTED = (
    "ms_version",
    "ms_last_error",
    "ms_device_status",
    "ms_plan_capacity",
    "ms_plan_build",
    "ms_prepare_step",
    "ms_qk_norm_rope_scatter",
    "ms_qkv_proj_norm_rope_scatter",
    "ms_kv_scatter",
    "ms_paged_attention",
    "ms_paged_attention_noalloc",
)


class MsPlanInfo(C.Structure):
    _fields_ = [
        ("num_seqs", C.c_int32),
        ("num_tokens", C.c_int32),
        ("n_decode_items", C.c_int32),
        ("n_tile_items", C.c_int32),
        ("n_combine", C.c_int32),
        ("off_seqs", C.c_int32),
        ("off_tables", C.c_int32),
        ("off_decode", C.c_int32),
        ("off_tile", C.c_int32),
        ("off_combine", C.c_int32),
        ("total_ints", C.c_int32),
        ("pages_per_split", C.c_int32),
        ("part_rows", C.c_int64),
        ("workspace_bytes_per_kv_head", C.c_int64),
        ("total_pages", C.c_int64),
        ("n_tc_items", C.c_int32),
        ("off_tc", C.c_int32),
        ("n_cascade", C.c_int32),
        ("decode_pages", C.c_int32),
        ("combine_tokens_max", C.c_int32),
        ("reserved", C.c_int32 * 3),
    ]


_P = C.c_void_p
_I32 = C.c_int32
_I64 = C.c_int64

_SIGNATURES = {
    "ms_version": (C.c_int, []),
    "ms_last_error": (C.c_char_p, []),
    "ms_device_status": (C.c_int, [_P, C.POINTER(C.c_uint32), C.c_int]),
    "ms_plan_capacity": (_I64, [_I32, _I32, _I64]),
    "ms_plan_build": (
        C.c_int,
        [_I32, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _P, _I64, C.POINTER(MsPlanInfo)],
    ),
    "ms_prepare_step": (C.c_int, [_I32, _P, _P, _P, _P, _I32, _P, _P, _P, _I64, _P]),
    "ms_qk_norm_rope_scatter": (
        C.c_int,
        [_P, _I64, _I32, _I32, _I32, _P, _P, C.c_float, _P, _P, _I64, _P, _I64, _P, _P, _I64,
         _P, _P, _I32, _P],
    ),
    "ms_qkv_proj_norm_rope_scatter": (
        C.c_int,
        [_P, _I64, _I32, _I32, _P, _I64, _I32, _I32, _P, _P, C.c_float, _P, _P, _I64, _P, _I64,
         _P, _P, _I64, _P, _P, _I32, _P],
    ),
    "ms_kv_scatter": (C.c_int, [_P, _I64, _P, _I64, _I32, _I32, _P, _P, _P, _I32, _P]),
    "ms_paged_attention": (
        C.c_int,
        [_P, _I64, _P, _I64, _I32, _I32, _P, _P, _I32, _P, C.POINTER(MsPlanInfo), _P, _I64,
         C.c_float, _P],
    ),
    "ms_paged_attention_noalloc": (
        C.c_int,
        [_P, _I64, _P, _I64, _I32, _I32, _P, _P, _I32, _P, C.POINTER(MsPlanInfo), C.c_float, _P],
    ),
}

_lock = threading.Lock()
_lib: C.CDLL | None = None


def load(path: str | os.PathLike[str] | None = None) -> C.CDLL:
    """Load (once) and return the library; raises if it is missing."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"{p} is missing: build it with `python -m miniserve_b200.build` "
                "(this package has no fallback path)"
            )
        lib = C.CDLL(str(p))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


_EXC = {
    MS_ERR_ARG: ValueError,
    MS_ERR_LAYOUT: ValueError,
    MS_ERR_PLAN: ValueError,
    MS_ERR_CAPACITY: RuntimeError,
    MS_ERR_CUDA: RuntimeError,
}


def check(rc: int, what: str) -> None:
    """Raise the Python exception matching a non-zero status code."""
    if rc == MS_OK:
        return
    msg = load().ms_last_error().decode(errors="replace")
    raise _EXC.get(rc, RuntimeError)(f"{what} failed (code {rc}): {msg}")


def device_status(stream: int = 0, clear: bool = True) -> int:
    """Synchronise `stream` and return (and by default clear) the device status bits."""
    flags = C.c_uint32(0)
    check(load().ms_device_status(_P(stream), C.byref(flags), 1 if clear else 0), "ms_device_status")
    return int(flags.value)
