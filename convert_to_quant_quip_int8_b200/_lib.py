"""ctypes binding of libqi8.so (the C ABI declared in include/qi8.h).

The library is built in-tree (``convert_to_quant_quip_int8_b200/libqi8.so``).
There is no fallback: if the library is missing or the current device is not
an sm_100 part, every kernel call raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libqi8.so")

# status codes (qi8.h)
QI8_OK = 0
QI8_EINVAL = -1
QI8_ESHAPE = -2
QI8_EALIGN = -3
QI8_EDTYPE = -4
QI8_ECUDA = -5
QI8_ETIMEOUT = -6
QI8_EUNSUPPORTED = -7

# element types
QI8_BF16, QI8_F16, QI8_F32, QI8_I8, QI8_I32 = 0, 1, 2, 3, 4
# row quantization modes
QI8_Q_TOKEN, QI8_Q_BLOCK, QI8_Q_GELU = 0, 1, 0x100
# scale kinds
QI8_S_NONE, QI8_S_SCALAR, QI8_S_ROW, QI8_S_ROW_KBLOCK, QI8_S_TILE128 = 0, 1, 2, 3, 4
QI8_MAX_PEERS = 8
# epilogue activation
QI8_ACT_NONE, QI8_ACT_GELU = 0, 1
# weight requant schemes
QI8_REQ_ROW, QI8_REQ_GLOBAL, QI8_REQ_BLOCK = 0, 1, 2

_DTYPE = {torch.bfloat16: QI8_BF16, torch.float16: QI8_F16, torch.float32: QI8_F32,
          torch.int8: QI8_I8, torch.int32: QI8_I32}

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int

# name -> (restype, argtypes); must match include/qi8.h
SIGNATURES = {
    "qi8_version": (_I, []),
    "qi8_last_error": (ctypes.c_char_p, []),
    "qi8_device_supported": (_I, [_I]),
    "qi8_device_status": (_I, [_I]),
    "qi8_quant_rows": (_I, [_P, _I, _I64, _I64, _I64, _I, _I, _P, _I64, _P, _P]),
    "qi8_rotate_quant_rows": (_I, [_P, _I, _I64, _I64, _I64, _I64, _P, _I, _I, _P, _P, _P]),
    "qi8_fwht_rows": (_I, [_P, _I, _I64, _I64, _I64, _I64, _P, _P, _I, _P, _P]),
    "qi8_fwht_cols": (_I, [_P, _I64, _I64, _I64, _I, ctypes.c_float, _P]),
    "qi8_unrotate_rows": (_I, [_P, _I64, _I64, _P, _P, _I, _I64, _P, _I, _I64, _P]),
    "qi8_gemm_i8": (_I, [_P, _P, _I64, _I64, _I64, _P, _I, _P, _I, _P, _I, _P, _I, _I64, _I, _P]),
    "qi8_dequant": (_I, [_P, _I64, _I64, _P, _I, _I, _P, _I, _P]),
    "qi8_quant_weight": (_I, [_P, _I, _I64, _I64, _I, _P, _P, _P, _I64, _P]),
    "qi8_quip_workspace_bytes": (_I64, [_I64, _I64]),
    "qi8_quip_convert": (_I, [_P, _I, _I64, _I64, _P, _P, _I, _I, _I, _P, _P, _P, _P, _I64, _P]),
    "qi8_quip_convert_noalloc": (_I, [_P, _I, _I64, _I64, _P, _P, _I, _I, _I, _P, _P, _P, _P]),
    "qi8_requant_weight": (_I, [_P, _I, _I64, _I64, _I64, _I, _I, _P, _P, _P, _I64, _P]),
    "qi8_weight_rotate2d": (_I, [_P, _I, _I64, _I64, _I64, _I64, _P, _P, _I, _P, _P, _I64, _P]),
    "qi8_allgather_cols": (_I, [_P, _I, _I64, _I64, _P, _I64, _P, _P, _I64, _P]),
    "qi8_gather_layout": (_I, [_P, _I, _I, _I64, _I64, _P, _I64, _P]),
    "qi8_gemm_workspace_bytes": (_I64, [_I64, _I64, _I64, _I, _I]),
    "qi8_gemm_i8_ws": (_I, [_P, _P, _I64, _I64, _I64, _P, _I, _P, _I, _P, _I, _P, _I, _I64, _I, _P, _I64, _P]),
    "qi8_gemm_i8_gather": (_I, [_P, _P, _I64, _I64, _I64, _P, _I, _P, _I, _P, _I, _P, _I, _I, _I, _I64, _I, _P]),
    "qi8_gemm_i8_quant": (_I, [_P, _P, _I64, _I64, _I64, _P, _I, _P, _I, _P, _I, _P, _I64, _P, _I, _P]),
    "qi8_int8_gelu": (_I, [_P, _P, _I64, _I64, _I, _P, _P, _P]),
    "qi8_gptq_quant_block": (_I, [_P, _I64, _I64, _I64, _P, _I64, _P, _I, _P, _I64, _P, _I64, _P]),
    "qi8_col_sumsq": (_I, [_P, _I, _I64, _I64, _I64, _P, _P]),
    "qi8_scale2d": (_I, [_P, _I, _I64, _I64, _I64, _P, _P, _I, _P, _I64, _P]),
    "qi8_ldlq_prepare": (_I, [_P, _P, _I64, _I64, _P, _P, _P, _P, _P, _P, _P]),
    "qi8_hinv_workspace_bytes": (_I64, [_I64]),
    "qi8_hinv_upper": (_I, [_P, _I64, _P, _P, _P, _I64, _P]),
    "qi8_eye_f32": (_I, [_P, _I64, _P]),
    "qi8_ldlq_workspace_bytes": (_I64, [_I64, _I64, _I]),
    "qi8_ldlq": (_I, [_P, _I64, _I64, _P, _P, _I, _P, _P, _I64, _P]),
    "qi8_ldlq_finish": (_I, [_P, _I64, _I64, _P, _P, _P, _P, _P]),
    "qi8_ipc_handle": (_I, [_P, _P, ctypes.POINTER(_I64)]),
    "qi8_ipc_open": (_I, [_P, _I64, ctypes.POINTER(_P)]),
    "qi8_ipc_close": (_I, [_P, _I64]),
    "qi8_peer_barrier": (_I, [_P, _I, _I, _P]),
}

_lib = None
_lock = threading.Lock()


class QI8Error(RuntimeError):
    """A libqi8 call failed (CUDA error, timeout, unsupported device)."""


def load() -> ctypes.CDLL:
    """Load libqi8.so (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(f"{LIB_PATH} is not built; run "
                                  "`python -m convert_to_quant_quip_int8_b200.build`")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def last_error() -> str:
    return load().qi8_last_error().decode(errors="replace")


def check(rc: int, what: str = "") -> None:
    """Map a qi8 status code onto the exception types the reference raises
    (AssertionError for shape/contiguity/alignment checks, TypeError for
    dtypes, RuntimeError for CUDA failures)."""
    if rc == QI8_OK:
        return
    msg = f"{what}: {last_error()}" if what else last_error()
    if rc in (QI8_ESHAPE, QI8_EALIGN, QI8_EINVAL):
        raise AssertionError(msg)
    if rc == QI8_EDTYPE:
        raise TypeError(msg)
    raise QI8Error(f"[{rc}] {msg}")


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE[dt]
    except KeyError:
        raise TypeError(f"unsupported dtype {dt}") from None


def ptr(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def stream_ptr(device=None):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def require_cuda(*tensors) -> None:
    """Fail loudly for non-CUDA inputs: this package has no CPU path."""
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("convert_to_quant_quip_int8_b200 kernels run on CUDA (sm_100a) only; "
                               f"got a tensor on {t.device}")
