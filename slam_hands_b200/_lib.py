"""ctypes binding of libdroidcorr.so (the C ABI declared in include/droidcorr.h).

The library is built in-tree (slam_hands_b200/libdroidcorr.so, see build()).
There is no fallback: if the library is missing or cannot be loaded, load()
raises, so no caller can silently run anything but the CUDA kernels.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libdroidcorr.so")
CSRC = os.path.join(PKG_DIR, "csrc")
HEADER = os.path.join(os.path.dirname(PKG_DIR), "include", "droidcorr.h")

DC_OK = 0
DC_ERR_INVALID_ARG = 1
DC_ERR_CUDA = 2
DC_ERR_UNSUPPORTED = 3
DC_ERR_NO_MEMORY = 4
DC_ERR_DEVICE_TIMEOUT = 5
DC_ERR_NOT_READY = 6

DC_PREC_FP32 = 0
DC_PREC_TF32 = 1
DC_PREC_BF16 = 2
DC_PREC_FP16 = 3
DC_PREC_FP32X3 = 4
PRECISIONS = {"fp32": DC_PREC_FP32, "tf32": DC_PREC_TF32, "bf16": DC_PREC_BF16,
              "fp16": DC_PREC_FP16, "fp32x3": DC_PREC_FP32X3}

DC_ORDER_SOURCE = 0
DC_ORDER_WINDOW_ROW = 1
DC_ORDER_AUTO = 2
TILE_ORDERS = {"source": DC_ORDER_SOURCE, "window_row": DC_ORDER_WINDOW_ROW,
               "auto": DC_ORDER_AUTO}

DC_DTYPE_F32 = 0
DC_DTYPE_F16 = 1

# Every function the header declares, with (restype, argtypes).
_vp = ctypes.c_void_p
_i = ctypes.c_int
_ll = ctypes.c_longlong
_f = ctypes.c_float


class DcConfig(ctypes.Structure):
    _fields_ = [("h", _i), ("w", _i), ("channels", _i), ("levels", _i), ("radius", _i),
                ("max_frames", _i), ("max_edges", _i), ("precision", _i), ("alpha", _f)]


_PP = ctypes.POINTER(_vp)
SIGNATURES = {
    "dc_default_config": (None, [ctypes.POINTER(DcConfig), _i, _i]),
    "dc_create": (_i, [ctypes.POINTER(DcConfig), ctypes.POINTER(_vp)]),
    "dc_destroy": (_i, [_vp]),
    "dc_last_error": (ctypes.c_char_p, [_vp]),
    "dc_status_string": (ctypes.c_char_p, [_i]),
    "dc_context_bytes": (_ll, [_vp]),
    "dc_set_frames": (_i, [_vp, _vp, _i, _i, _i, _vp]),
    "dc_build_volume": (_i, [_vp, _vp, _vp, _i, _PP, _vp]),
    "dc_pool_2x2": (_i, [_vp, _vp, _ll, _i, _i, _vp]),
    "dc_lookup": (_i, [_vp, _PP, _vp, _vp, _i, _vp]),
    "dc_lookup_single": (_i, [_vp, _PP, _vp, _vp, _vp]),
    "dc_build_and_lookup": (_i, [_vp, _vp, _vp, _i, _vp, _vp, _vp]),
    "dc_alt_lookup": (_i, [_vp, _vp, _vp, _i, _vp, _vp, _vp]),
    "dc_launch_count": (_ll, [_vp]),
    "dc_device_status": (_i, [_vp, _vp]),
    "dc_store_slots": (_i, [_vp, _i, _i, ctypes.POINTER(_vp), ctypes.POINTER(_ll)]),
    "dc_project": (_i, [_vp, _vp, _vp, _vp, _i, _vp, _vp, _i, _vp, _vp, _vp]),
    "dc_project_build_and_lookup": (_i, [_vp, _vp, _vp, _vp, _i, _vp, _vp, _i, _vp, _vp, _vp,
                                         _vp]),
    "dc_scatter_mean": (_i, [_vp, _vp, _ll, _vp, _i, _vp, _vp, _vp, _vp]),
    "dc_gather_rows": (_i, [_vp, _vp, _ll, _i, _vp, _i, _vp, _vp]),
    "dc_build_and_lookup_static": (_i, [ctypes.POINTER(DcConfig), _vp, _i, _i, _vp, _vp, _i,
                                        _vp, _vp, _vp]),
    "dc_static_device_status": (_i, [_vp]),
    "dc_set_max_ctas": (_i, [_vp, _i]),
    "dc_set_tile_order": (_i, [_vp, _i]),
    "dc_store_ipc_handle": (_i, [_vp, _vp]),
    "dc_store_attach_source": (_i, [_vp, _vp]),
    "dc_store_pull_slots": (_i, [_vp, _i, _i, _vp]),
    "dc_sync_signal": (_i, [_vp, _i, ctypes.c_uint, _i, _vp]),
    "dc_sync_wait": (_i, [_vp, _i, ctypes.c_uint, _i, _vp]),
    "dc_set_corr_encoder": (_i, [_vp, _vp, _vp, _i, _vp]),
    "dc_corr_encode": (_i, [_vp, _vp, _i, _vp, _vp]),
    "dc_build_lookup_encode": (_i, [_vp, _vp, _vp, _i, _vp, _vp, _vp, _vp]),
    "dc_debug_inject_stall": (_i, [_ll]),
}

_lib = None


def build(jobs: int = 8) -> str:
    """Compile libdroidcorr.so for sm_100a with the committed Makefile (nvcc)."""
    subprocess.run(["make", "-s", "-C", CSRC, f"-j{jobs}"], check=True)
    return LIB_PATH


def load() -> ctypes.CDLL:
    """Load the in-tree library and bind every declared entry point."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"libdroidcorr.so not found at {LIB_PATH}; build it with "
            "`python -c 'import __graft_entry__ as g; g.build()'` (nvcc, sm_100a). "
            "There is no CPU fallback.")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


class DroidCorrError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"droidcorr status {status}: {msg}")
        self.status = status
