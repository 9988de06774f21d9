"""ctypes binding of ``libmxg.so`` (the C ABI declared in ``include/mxg.h``).

The library is the only compute path: if it is missing or fails to load the
functions below raise; there is no CPU or library fallback.
"""
from __future__ import annotations

import ctypes
import os
import re
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmxg.so")
HEADER_PATH = os.path.join(os.path.dirname(_HERE), "include", "mxg.h")

MXG_OK = 0
MXG_ERR_INVALID_ARGUMENT = 1
MXG_ERR_BAD_SHAPE = 2
MXG_ERR_MISALIGNED = 3
MXG_ERR_WORKSPACE_TOO_SMALL = 4
MXG_ERR_CUDA = 5
MXG_ERR_DEVICE_TIMEOUT = 6
MXG_ERR_BAD_OFFSETS = 7
MXG_ERR_UNSUPPORTED_DEVICE = 8
MXG_ERR_TOO_MANY_GROUPS = 9
OFFS_LEADING_ZERO, OFFS_CUMULATIVE, OFFS_SIZES, OFFS_AUTO = 0, 1, 2, 3
DTYPE_BF16, DTYPE_F32 = 0, 1
MAX_GROUPS = 256

_c_i64, _c_int, _c_size, _vp = ctypes.c_int64, ctypes.c_int, ctypes.c_size_t, ctypes.c_void_p
_i32p = ctypes.POINTER(ctypes.c_int32)

_PROTOS = {
    "mxg_error_string": (ctypes.c_char_p, [_c_int]),
    "mxg_version": (_c_int, []),
    "mxg_get_device_error": (_c_int, [ctypes.POINTER(ctypes.c_int), _c_int]),
    "mxg_quantize_rowwise": (_c_int, [_vp, _c_i64, _c_i64, _vp, _vp, _vp]),
    "mxg_quantize_colwise": (_c_int, [_vp, _c_i64, _c_i64, _vp, _vp, _vp]),
    "mxg_grouped_fwd_workspace_size": (_c_size, [_c_int, _c_i64, _c_i64, _c_i64]),
    "mxg_grouped_fwd": (_c_int, [_vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_i64, _c_i64,
                                 _c_i64, _vp, _c_int, _vp, _c_size, _vp]),
    "mxg_grouped_fwd_prepare": (_c_int, [_vp, _vp, _vp, _c_int, _c_int, _c_int, _c_i64, _c_i64,
                                         _c_i64, _vp, _c_size, _vp]),
    "mxg_grouped_fwd_run": (_c_int, [_vp, _vp, _c_int, _c_i64, _c_i64, _c_i64, _vp, _c_int, _vp,
                                     _c_size, _vp]),
    "mxg_grouped_fwd_run_scatter": (_c_int, [_vp, _vp, _c_int, _c_i64, _c_i64, _c_i64, _vp, _c_int, _vp,
                                             _vp, _c_i64, _vp, _c_size, _vp]),
    "mxg_grouped_wgrad_prepare": (_c_int, [_vp, _vp, _vp, _c_int, _c_int, _c_int, _c_i64, _c_i64,
                                           _c_i64, _vp, _c_size, _vp]),
    "mxg_grouped_wgrad_run": (_c_int, [_vp, _vp, _c_int, _c_i64, _c_i64, _c_i64, _vp, _c_int, _vp,
                                       _c_size, _vp]),
    "mxg_grouped_fwd_noalloc": (_c_int, [_vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_i64,
                                         _c_i64, _c_i64, _vp, _c_int, _vp]),
    "mxg_dense_fwd_kn_workspace_size": (_c_size, [_c_i64, _c_i64, _c_i64]),
    "mxg_dense_fwd_kn": (_c_int, [_vp, _vp, _c_i64, _c_i64, _c_i64, _vp, _c_int, _vp, _c_size, _vp]),
    "mxg_grouped_wgrad_workspace_size": (_c_size, [_c_int, _c_i64, _c_i64, _c_i64]),
    "mxg_grouped_wgrad": (_c_int, [_vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_i64, _c_i64,
                                   _c_i64, _vp, _c_int, _vp, _c_size, _vp]),
    "mxg_transpose_u8": (_c_int, [_vp, _c_i64, _c_i64, _vp, _vp]),
    "mxg_ep_route_workspace_size": (_c_size, [_c_i64, _c_int]),
    "mxg_ep_route": (_c_int, [_vp, _vp, _c_i64, _c_int, _c_int, _vp, _vp, _vp, _vp, _c_size, _vp]),
    "mxg_gather_rows": (_c_int, [_vp, _c_i64, _c_i64, _vp, _c_i64, _vp, _vp]),
    "mxg_ep_regroup": (_c_int, [_vp, _c_int, _c_int, _c_int, _vp, _vp, _vp, _vp]),
    "mxg_ep_combine": (_c_int, [_vp, _vp, _vp, _c_i64, _c_int, _c_i64, _vp, _vp]),
    "mxg_swiglu": (_c_int, [_vp, _c_i64, _c_i64, _vp, _vp]),
    "mxg_swiglu_bwd": (_c_int, [_vp, _vp, _c_i64, _c_i64, _vp, _vp]),
    "mxg_peer_alloc": (_c_int, [_c_size, ctypes.POINTER(_vp), _vp]),
    "mxg_peer_open": (_c_int, [_vp, ctypes.POINTER(_vp)]),
    "mxg_peer_close": (_c_int, [_vp]),
    "mxg_peer_free": (_c_int, [_vp]),
    "mxg_ep_p2p_plan_workspace_size": (_c_size, [_c_int, _c_int]),
    "mxg_ep_p2p_plan": (_c_int, [_vp, _c_int, _c_int, _c_int, _c_int, _c_i64, _vp, _vp, _vp, _vp,
                                 _vp, _vp, _vp, _vp, _c_size, _vp]),
    "mxg_ep_dispatch_p2p": (_c_int, [_vp, _c_i64, _c_i64, _vp, _c_i64, _vp, _vp, _c_int, _c_int,
                                     _c_int, _vp, _c_i64, _c_int, _vp]),
    "mxg_ep_dispatch_p2p_gather": (_c_int, [_vp, _c_i64, _c_i64, _vp, _c_i64, _vp, _vp, _c_int, _c_int,
                                            _c_int, _vp, _c_i64, _vp, _vp, _c_int, _vp, _vp]),
    "mxg_ep_return_p2p": (_c_int, [_vp, _c_i64, _vp, _c_i64, _vp, _vp, _vp, _c_int, _c_i64, _c_int,
                                   _vp]),
    "mxg_ep_zero_pad_rows": (_c_int, [_vp, _c_i64, _vp, _c_i64, _vp]),
    "mxg_copy_runs": (_c_int, [_vp, _c_i64, _c_i64, _vp, _vp, _vp, _vp, _c_i64, _vp, _c_int, _c_i64,
                               _vp]),
    "mxg_set_gemm_sm_limit": (_c_int, [_c_int]),
    "mxg_get_gemm_sm_limit": (_c_int, []),
    "mxg_quantize_dual": (_c_int, [_vp, _c_i64, _c_i64, _vp, _vp, _vp, _vp, _vp]),
    "mxg_quantize_dual_rows": (_c_int, [_vp, _c_i64, _c_i64, _c_i64, _c_i64, _vp, _vp, _vp, _vp, _vp]),
    "mxg_swiglu_quantize": (_c_int, [_vp, _c_i64, _c_i64, _vp, _vp, _vp, _vp, _vp]),
    "mxg_swiglu_bwd_quantize": (_c_int, [_vp, _vp, _c_i64, _c_i64, _vp, _vp, _vp, _vp, _vp]),
    "mxg_debug_inject_stall": (_c_int, [_c_i64]),
}

_lock = threading.Lock()
_lib = None


class MxgError(RuntimeError):
    """A non-zero status from the C ABI (host validation, CUDA, or a device-side error)."""

    def __init__(self, code: int, where: str):
        self.code = code
        super().__init__(f"{where}: {error_string(code)} (code {code})")


def header_symbols() -> list[str]:
    """Every entry point ``include/mxg.h`` declares."""
    txt = open(HEADER_PATH).read()
    return sorted(set(re.findall(r"^MXG_API [^;(]*?\b(mxg_\w+)\s*\(", txt, flags=re.M)))


def load() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is not built; run `python mxfp8-grouped-gemm_b200/build.py`")
            L = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in _PROTOS.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def error_string(code: int) -> str:
    return load().mxg_error_string(int(code)).decode()


def check(code: int, where: str) -> None:
    if code != MXG_OK:
        raise MxgError(code, where)


def device_error(clear: bool = True) -> int:
    """Synchronise and return the device error word (0 = no error)."""
    v = ctypes.c_int(0)
    check(load().mxg_get_device_error(ctypes.byref(v), 1 if clear else 0), "mxg_get_device_error")
    return v.value


def raise_device_error() -> None:
    code = device_error(clear=True)
    if code:
        raise MxgError(code, "device")


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


# ---------------------------------------------------------------- workspaces
_ws_cache: dict = {}


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """A cached uint8 device buffer of at least ``nbytes`` for the current
    stream (calls on one stream run in order, so they may share it)."""
    key = (device.index if device.index is not None else torch.cuda.current_device(), stream_ptr(device))
    buf = _ws_cache.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(int(nbytes), 1024), dtype=torch.uint8, device=device)
        _ws_cache[key] = buf
    return buf
