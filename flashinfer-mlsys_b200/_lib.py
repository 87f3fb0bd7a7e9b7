"""ctypes view of ``libmoe_fp8_ds.so`` (declarations: include/moe_fp8_ds.h).

Loading never touches the GPU. There is no fallback: if the library is
missing the import of the op fails with an error naming the build step.
"""
from __future__ import annotations

import ctypes
import os
import threading

from . import build as _build

_c_int64 = ctypes.c_int64
_vp = ctypes.c_void_p

# name -> (restype, argtypes)
SIGNATURES = {
    "moe_fp8_ds_kernel": (ctypes.c_int, [_vp] * 8 + [_c_int64, ctypes.c_double, _vp, _c_int64, _c_int64, _vp]),
    "moe_fp8_ds_kernel_ex": (
        ctypes.c_int,
        [_vp] * 8 + [_c_int64, ctypes.c_double, _vp, _c_int64, _c_int64, _vp, _vp, _vp, _vp],
    ),
    "moe_fp8_ds_kernel_shared": (
        ctypes.c_int,
        [_vp] * 8 + [_c_int64, ctypes.c_double] + [_vp] * 5 + [_c_int64, _c_int64, _vp],
    ),
    "moe_fp8_ds_route": (ctypes.c_int, [_vp, _vp, _c_int64, _c_int64, _c_int64, ctypes.c_double, _vp, _vp, _vp, _vp]),
    "moe_fp8_ds_route_noalloc": (
        ctypes.c_int, [_vp, _vp, _c_int64, _c_int64, _c_int64, ctypes.c_double, _vp, _vp, _vp, _vp]),
    "moe_fp8_ds_experts": (
        ctypes.c_int,
        [_vp] * 8 + [_c_int64, _c_int64, _c_int64, _vp, ctypes.c_int, _vp],
    ),
    "moe_fp8_ds_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "moe_fp8_ds_device_status": (ctypes.c_int, [_vp]),
    "moe_fp8_ds_workspace_bytes": (ctypes.c_size_t, [_c_int64, _c_int64]),
    "moe_fp8_ds_last_rows": (ctypes.c_int, [_c_int64, _c_int64, _vp, _vp]),
    "moe_fp8_ds_release_workspace": (ctypes.c_int, []),
    "moe_fp8_ds_version": (ctypes.c_char_p, []),
    "moe_fp8_ds_profile_enable": (ctypes.c_int, [ctypes.c_int]),
    "moe_fp8_ds_profile_last": (ctypes.c_int, [ctypes.POINTER(ctypes.c_float), ctypes.c_int]),
    "moe_fp8_ds_set_fused_decode": (ctypes.c_int, [ctypes.c_int]),
    "moe_fp8_ds_test_route_barrier": (ctypes.c_int, [ctypes.c_uint64, ctypes.c_int]),
    "moe_fp8_ds_quantize_act": (ctypes.c_int, [_vp, _c_int64, _vp, _vp, _vp]),
    "moe_fp8_ds_add_norm_quant": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_float, _c_int64, _vp, _vp, _vp]),
    "moe_fp8_ds_ep_pack": (ctypes.c_int, [_vp, _vp, _vp, _vp, _c_int64, _vp, _c_int64, _vp, _vp]),
    "moe_fp8_ds_ep_unpack": (ctypes.c_int, [_vp, _c_int64, _vp, _vp, _vp, _vp, _vp]),
    "moe_fp8_ds_ep_combine": (ctypes.c_int, [_vp, _vp, _c_int64, _c_int64, _vp, _vp]),
    "moe_fp8_ds_ep_plan": (ctypes.c_int, [_vp, _c_int64, _c_int64, _vp, _vp, _vp, _vp]),
}

_lib = None
_load_lock = threading.Lock()


def lib_path() -> str:
    """The in-tree library, or the file named by MOE_FP8_DS_LIBRARY (an
    alternative build of the same sources, e.g. for side-by-side timing)."""
    return os.environ.get("MOE_FP8_DS_LIBRARY") or _build.LIB_PATH


def load(build_if_missing: bool = True) -> ctypes.CDLL:
    """Load (building first if needed) the sm_100a library and bind signatures.
    Thread-safe: concurrent first calls build and load once."""
    global _lib
    if _lib is not None:
        return _lib
    with _load_lock:
        if _lib is not None:
            return _lib
        path = lib_path()
        if path == _build.LIB_PATH and (not os.path.exists(path) or (build_if_missing and _build.is_stale())):
            if not build_if_missing:
                raise RuntimeError(f"{path} is missing: build it with `python flashinfer-mlsys_b200/build.py`")
            _build.build()
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return lib


class MoeError(RuntimeError):
    """A nonzero status from the C ABI."""

    def __init__(self, status: int, where: str):
        msg = load().moe_fp8_ds_status_string(status).decode()
        super().__init__(f"{where}: status {status} ({msg})")
        self.status = status


def check(status: int, where: str) -> None:
    if status != 0:
        raise MoeError(status, where)
