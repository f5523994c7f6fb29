"""ctypes binding of the C ABI in include/rep_b200.h (librep_b200.so).

Every device entry point of the package goes through ``call``: it passes raw
device pointers and torch's current CUDA stream, and turns a non-zero status
into the exception type the reference raises for the same condition
(ValueError for shapes/arguments, RuntimeError for CUDA/device failures).
There is no fallback: if the library is missing or the device is not an
sm_100 part, the call raises.
"""

from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "librep_b200.so")

RB_F32, RB_BF16, RB_F16, RB_I32, RB_I8, RB_I64 = 0, 1, 2, 3, 4, 5
RB_ACT_DYNAMIC, RB_ACT_STATIC, RB_ACT_NONE = 0, 1, 2
RB_OK, RB_ERR_VALUE, RB_ERR_UNSUPPORTED, RB_ERR_CUDA, RB_ERR_DEVICE = 0, 1, 2, 3, 4
RB_MAX_SLOTS = 32
RB_MAX_DEST = 8
RB_IPC_HANDLE_BYTES = 64

_vp, _i64, _i32, _f32, _u64 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_uint64
_pp = ctypes.POINTER(ctypes.c_void_p)

# name -> argtypes (every entry point returns int)
SIGNATURES = {
    "rb_rep_gather_ln_quant": [_vp, _i32, _i64, _i32, _vp, _vp, _vp, _i32, _i64, _vp, _vp, _i32, _f32,
                               _i32, _vp, _i32, _vp, _i64, _vp, _vp, _vp, _vp],
    "rb_rep_gather_ln_quant_idx": [_vp, _i32, _i64, _i32, _i32, _vp, _vp, _vp, _i32, _i64, _vp, _vp, _i32, _f32,
                                   _i32, _vp, _i32, _vp, _i64, _vp, _vp, _vp, _vp],
    "rb_rep_gather_pool": [_vp, _i32, _i64, _i32, _vp, _vp, _vp, _vp, _i32, _i64, _vp, _i64, _vp],
    "rb_layernorm_quant": [_vp, _i32, _i64, _i32, _i64, _vp, _vp, _i32, _f32, _i32, _vp, _i32, _vp, _i64,
                           _vp, _vp, _vp],
    "rb_layernorm_quant_slots": [_vp, _i32, _i64, _i32, _i64, _vp, _vp, _i32, _f32, _i32, _vp, _i32, _vp, _i64,
                                 _vp, _vp, _vp],
    "rb_quant_dynamic_per_token": [_vp, _i32, _i64, _i64, _i64, _vp, _i64, _vp, _vp],
    "rb_quant_static": [_vp, _i32, _i64, _vp, _i32, _vp, _vp],
    "rb_quant_rows_v1": [_vp, _i32, _i64, _i64, _i64, _vp, _i64, _vp, _vp],
    "rb_quantize_weight_per_channel": [_vp, _i32, _i64, _i64, _i64, _vp, _vp, _vp],
    "rb_pack_weight_nk": [_vp, _i64, _i64, _i64, _i64, _vp, _vp],
    "rb_w8a8_gemm": [_vp, _i64, _vp, _i64, _i64, _i64, _i64, _vp, _i32, _i32, _vp, _i32, _vp, _i32, _vp,
                     _i64, _i32, _vp],
    "rb_w8a8_gemm_ws": [_vp, _i64, _vp, _i64, _i64, _i64, _i64, _vp, _i32, _i32, _vp, _i32, _vp, _i32, _vp,
                        _i64, _i32, _vp, _i64, _vp],
    "rb_w8a8_gemm_workspace_size": [_i64, _i64, _i64],
    "rb_w8a8_gemm_noalloc": [_vp, _i64, _vp, _i64, _i64, _i64, _i64, _vp, _i32, _i32, _vp, _i32, _vp, _i32, _vp,
                             _i64, _i32, _vp],
    "rb_w8a8_gemm_ln": [_vp, _i64, _vp, _i64, _i64, _i64, _i64, _vp, _i32, _i32, _vp, _i32, _vp, _i32, _vp,
                        _i64, _i32, _vp, _vp, _i32, _f32, _vp, _i64, _vp],
    "rb_fp_gemm": [_vp, _i32, _i64, _vp, _i64, _i64, _i64, _i64, _vp, _i32, _vp, _i64, _i32, _vp],
    "rb_smoe_workspace_size": [_i64, _i32, _i32, _i32, _i32, _i32],
    "rb_smoe_experts": [_vp, _i32, _i64, _i64, _i32, _vp, _i32, _vp, _i32, _i32, _vp, _vp, _vp, _vp, _i32, _vp,
                        _i64, _vp, _i64, _vp],
    "rb_rep_gather_pool_scatter": [_vp, _i32, _i64, _i32, _vp, _vp, _vp, _vp, _i32, _i64, _vp, _vp, _i32, _i64,
                                   _i64, _vp],
    "rb_ipc_export": [_vp, _vp, _vp],
    "rb_ipc_import": [_vp, _i64, _vp],
    "rb_ipc_close": [_vp, _i64],
    "rb_device_supported": [],
    "rb_device_error": [_i32],
    "rb_selftest_wait_timeout": [_u64, _vp],
    "rb_version": [],
}

RETURNS_I64 = {"rb_w8a8_gemm_workspace_size", "rb_smoe_workspace_size"}

_lock = threading.Lock()
_lib: Optional[ctypes.CDLL] = None
_load_error: Optional[str] = None


def load() -> ctypes.CDLL:
    """Load librep_b200.so (raises RuntimeError if it is missing or broken)."""
    global _lib, _load_error
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            _load_error = (f"{LIB_PATH} is missing; build it with "
                           "`python -m baidu_cti_grab_b200.build`")
            raise RuntimeError(_load_error)
        try:
            lib = ctypes.CDLL(LIB_PATH)
        except OSError as exc:
            _load_error = f"cannot load {LIB_PATH}: {exc}"
            raise RuntimeError(_load_error) from exc
        for name, argtypes in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = ctypes.c_int64 if name in RETURNS_I64 else ctypes.c_int
        lib.rb_last_error.argtypes = []
        lib.rb_last_error.restype = ctypes.c_char_p
        _lib = lib
        return lib


def is_available() -> bool:
    try:
        load()
        return True
    except RuntimeError:
        return False


def load_error_message() -> Optional[str]:
    return _load_error


def last_error() -> str:
    msg = load().rb_last_error()
    return msg.decode() if msg else ""


def call(name: str, *args) -> None:
    """Invoke an entry point and raise on a non-zero status."""
    rc = getattr(load(), name)(*args)
    if rc == RB_OK:
        return
    msg = f"{name}: {last_error()}"
    if rc in (RB_ERR_VALUE, RB_ERR_UNSUPPORTED):
        raise ValueError(msg)
    raise RuntimeError(msg)


def device_error(reset: bool = False) -> int:
    """Watchdog status of the library's kernels (synchronous; 0 = healthy)."""
    v = load().rb_device_error(1 if reset else 0)
    if v < 0:
        raise RuntimeError(f"rb_device_error: {last_error()}")
    return v


def ptr_array(values) -> "ctypes.Array":
    """Host array of device pointers (one per slot)."""
    arr = (ctypes.c_void_p * len(values))()
    for i, v in enumerate(values):
        arr[i] = v
    return arr


def i64_array(values) -> "ctypes.Array":
    arr = (ctypes.c_int64 * len(values))()
    for i, v in enumerate(values):
        arr[i] = int(v)
    return arr


def i32_array(values) -> "ctypes.Array":
    arr = (ctypes.c_int * len(values))()
    for i, v in enumerate(values):
        arr[i] = int(v)
    return arr
