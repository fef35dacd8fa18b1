"""ctypes binding of ``libscalesweep_b200.so`` (the C ABI in include/scalesweep_b200.h).

There is no fallback: if the library is missing or the tensors are not on a
CUDA device, calls raise.  Build the library with
``python -m test_speed_scalesweep_b200.build``.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

from . import build as _build

_c_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_f32 = ctypes.c_float

_SIGNATURES = {
    "ssw_abi_version": (_int, []),
    "ssw_status_string": (ctypes.c_char_p, [_int]),
    "ssw_last_error": (ctypes.c_char_p, []),
    "ssw_scalesweep_mse_nvfp4_quant_out": (_int, [_c_p, _int, _i64, _i64, _i64, _c_p, _c_p, _c_p, _int, _c_p]),
    "ssw_scalesweep_mse128_nvfp4_quant_out": (_int, [_c_p, _int, _i64, _i64, _i64, _c_p, _c_p, _c_p, _int, _c_p]),
    "ssw_scalesweep_mse_reference_nvfp4_quant_out": (_int, [_c_p, _int, _i64, _i64, _i64, _c_p, _c_p, _c_p, _int, _c_p]),
    "ssw_scalesweep_nvfp4_quant_out": (_int, [_c_p, _int, _i64, _i64, _i64, _c_p, _c_p, _c_p, _int, _c_p]),
    "ssw_scalesweep128_nvfp4_quant_out": (_int, [_c_p, _int, _i64, _i64, _i64, _c_p, _c_p, _c_p, _int, _c_p]),
    "ssw_rtn_nvfp4_quant_out": (_int, [_c_p, _int, _i64, _i64, _i64, _c_p, _c_p, _c_p, _int, _c_p]),
    "ssw_silu_and_mul": (_int, [_c_p, _int, _i64, _i64, _c_p, _c_p]),
    "ssw_rms_norm_scalesweep_mse_nvfp4_quant_out": (_int, [_c_p, _c_p, _c_p, _f32, _i64, _i64, _c_p,
                                                           _c_p, _c_p, _int, _c_p, _c_p]),
    "ssw_silu_and_mul_scalesweep_mse_nvfp4_quant_out": (_int, [_c_p, _int, _i64, _i64, _c_p, _c_p,
                                                               _c_p, _int, _c_p]),
    "ssw_absmax_workspace_bytes": (_i64, []),
    "ssw_absmax": (_int, [_c_p, _int, _i64, _c_p, _c_p, _c_p]),
    "ssw_global_scale_from_amax": (_int, [_c_p, _f32, _c_p, _c_p]),
    "ssw_global_scale_inv": (_int, [_c_p, _int, _i64, _f32, _c_p, _c_p, _c_p, _c_p]),
    "ssw_nvfp4_gemm_workspace_bytes": (_i64, [_i64, _i64, _i64]),
    "ssw_nvfp4_quant_gemm_workspace_bytes": (_i64, [_i64, _i64, _i64]),
    "ssw_nvfp4_quant_gemm": (_int, [_c_p, _int, _c_p, _c_p, _c_p, _c_p, _c_p, _i64, _i64, _i64,
                                    _c_p, _i64, _c_p, _c_p]),
    "ssw_nvfp4_gemm": (_int, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _i64, _i64, _i64, _c_p, _i64,
                              _c_p, _c_p]),
    "ssw_nvfp4_gemm_dependent": (_int, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _i64, _i64, _i64,
                                        _c_p, _i64, _c_p, _c_p]),
    "ssw_nvfp4_mma_rate_probe": (_int, [_int, _int, _c_p, _c_p, _c_p]),
    "ssw_global_scale_inv_noalloc_max_numel": (_i64, []),
    "ssw_global_scale_inv_noalloc": (_int, [_c_p, _int, _i64, _f32, _c_p, _c_p, _c_p]),
}

ABI_VERSION = 1
SSW_OK, SSW_ERR_INVALID_ARGUMENT, SSW_ERR_UNSUPPORTED, SSW_ERR_CUDA, SSW_ERR_TIMEOUT = range(5)

_lock = threading.Lock()
_handle = None


def library_path() -> str:
    return _build.LIB_PATH


def lib() -> ctypes.CDLL:
    """Load the CUDA library (once).  Raises if it has not been built."""
    global _handle
    if _handle is not None:
        return _handle
    with _lock:
        if _handle is None:
            path = library_path()
            if not os.path.exists(path):
                raise RuntimeError(
                    f"{path} is missing: the scale-sweep CUDA library must be built "
                    "(python -m test_speed_scalesweep_b200.build); there is no CPU fallback")
            h = ctypes.CDLL(path)
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(h, name)
                fn.restype = res
                fn.argtypes = args
            if h.ssw_abi_version() != ABI_VERSION:
                raise RuntimeError("libscalesweep_b200.so ABI version mismatch; rebuild it")
            _handle = h
    return _handle


def check(status: int) -> None:
    if status == SSW_OK:
        return
    h = lib()
    msg = (h.ssw_last_error() or b"").decode() or h.ssw_status_string(status).decode()
    if status == SSW_ERR_INVALID_ARGUMENT:
        raise ValueError(msg)
    if status == SSW_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    if status == SSW_ERR_TIMEOUT:
        raise TimeoutError(msg)
    raise RuntimeError(msg)


DTYPE_CODES = {torch.bfloat16: 0, torch.float16: 1}


def dtype_code(t: torch.Tensor) -> int:
    try:
        return DTYPE_CODES[t.dtype]
    except KeyError:
        raise ValueError(f"input dtype must be torch.bfloat16 or torch.float16, got {t.dtype}") from None


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream
