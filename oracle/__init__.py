"""CPU ORACLE -- test infrastructure, never product code.

Python bindings (ctypes) for ``scalesweep_oracle.c``, the plain-C restatement
of the reference's scale-sweep NVFP4 quantizer (K1 ``scalesweep_mse``, K2
``scalesweep_mse_reference``, the full-range ``mse128`` mode, the RTN
comparator, the global amax/scale), plus a numpy GEMM reference for the NVFP4
linear layer.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline leg may import this package, and only as the checker or as the
timed CPU baseline; the product path never routes through it.

Parity pin: the restatement is checked bit-for-bit against golden vectors
produced by the reference's own Triton kernels (``tests/golden/``), and the
hardware conversion semantics it assumes were measured on a B200.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import build as _build

_VARIANTS = {"mse": 0, "reference": 1, "weighted": 2}
_MODES = {"window": 0, "full_range": 1, "rtn": 2}
_DTYPES = {"bf16": 0, "f16": 1}
SENTINEL = 0xA5

_lib = None


def lib():
    global _lib
    if _lib is None:
        path = _build.LIB
        if not os.path.exists(path):
            path = _build.build()
        L = ctypes.CDLL(path)
        L.orc_quantize.restype = ctypes.c_int
        L.orc_quantize.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int64,
                                   ctypes.c_int64, ctypes.c_float, ctypes.c_void_p,
                                   ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_int]
        L.orc_absmax.restype = ctypes.c_float
        L.orc_absmax.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int]
        L.orc_global_scale_inv.restype = ctypes.c_float
        L.orc_global_scale_inv.argtypes = [ctypes.c_float, ctypes.c_float]
        L.orc_dequantize.restype = ctypes.c_int
        L.orc_dequantize.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                     ctypes.c_int64, ctypes.c_int, ctypes.c_void_p]
        L.orc_swizzled_offset.restype = ctypes.c_int64
        L.orc_swizzled_offset.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64]
        L.orc_e2m1_encode.restype = ctypes.c_uint8
        L.orc_e2m1_encode.argtypes = [ctypes.c_float]
        L.orc_e4m3_encode.restype = ctypes.c_uint8
        L.orc_e4m3_encode.argtypes = [ctypes.c_float]
        L.orc_e4m3_decode.restype = ctypes.c_float
        L.orc_e4m3_decode.argtypes = [ctypes.c_uint8]
        L.orc_silu_mul.restype = ctypes.c_int
        L.orc_silu_mul.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int64,
                                   ctypes.c_void_p, ctypes.c_int]
        L.orc_rms_sumsq.restype = ctypes.c_int
        L.orc_rms_sumsq.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                    ctypes.c_int64, ctypes.c_void_p]
        L.orc_rms_apply.restype = ctypes.c_int
        L.orc_rms_apply.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                    ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p]
        _lib = L
    return _lib


def round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


def scale_shape(m: int, n_out: int, swizzled: bool) -> tuple[int, int]:
    if swizzled:
        return round_up(m, 128), round_up(n_out // 16, 4)
    return m, n_out // 16


def quantize(bits: np.ndarray, gsi: float, *, dtype: str = "bf16", padded_n: int | None = None,
             swizzled: bool = True, variant: str = "mse", mode: str = "window",
             nthreads: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """Oracle quantization of a [m, n] bf16/f16 tensor given as uint16 bits.

    Returns (codes uint8 [m, n_out/2], scales uint8) with the unwritten scale
    padding left at ``SENTINEL``.
    """
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    m, n = bits.shape
    n_out = padded_n if padded_n is not None else n
    codes = np.full((m, n_out // 2), SENTINEL, np.uint8)
    scales = np.full(scale_shape(m, n_out, swizzled), SENTINEL, np.uint8)
    rc = lib().orc_quantize(bits.ctypes.data, _DTYPES[dtype], m, n, n_out, float(gsi),
                            codes.ctypes.data, scales.ctypes.data, int(swizzled),
                            _VARIANTS[variant], _MODES[mode], int(nthreads))
    if rc != 0:
        raise ValueError("oracle rejected the shape")
    return codes, scales


def silu_mul(bits: np.ndarray, dtype: str = "bf16", nthreads: int = 0) -> np.ndarray:
    """vLLM's silu_and_mul on a [m, 2n] bf16/f16 tensor given as uint16 bits:
    returns the [m, n] bits of RN(RN(silu(gate)) * up) (``orc_silu_mul``)."""
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    m, n2 = bits.shape
    if n2 % 2:
        raise ValueError("the last dimension must be even (gate, then up)")
    out = np.empty((m, n2 // 2), np.uint16)
    if lib().orc_silu_mul(bits.ctypes.data, _DTYPES[dtype], m, n2 // 2, out.ctypes.data,
                          int(nthreads)) != 0:
        raise ValueError("oracle rejected the shape")
    return out


def silu_mul_quantize(bits: np.ndarray, gsi: float, *, dtype: str = "bf16",
                      swizzled: bool = True) -> tuple[np.ndarray, np.ndarray]:
    """The fused SiLU-and-mul quantizer: ``quantize(silu_mul(bits))`` with the
    scalesweep_mse window."""
    return quantize(silu_mul(bits, dtype), gsi, dtype=dtype, swizzled=swizzled)


def rms_sumsq(bits: np.ndarray, residual: np.ndarray | None = None):
    """vLLM's RMSNorm sum of squares per row of a [m, n] bf16 tensor given as
    uint16 bits (``orc_rms_sumsq``).  With ``residual`` (fused_add_rms_norm)
    the rows summed are bf16(x + residual); returns (acc float32 [m], the
    updated residual bits or None)."""
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    m, n = bits.shape
    acc = np.empty(m, np.float32)
    res = None if residual is None else np.array(residual, dtype=np.uint16, order="C", copy=True)
    if lib().orc_rms_sumsq(bits.ctypes.data, 0 if res is None else res.ctypes.data, m, n,
                           acc.ctypes.data) != 0:
        raise ValueError("oracle rejected the shape")
    return acc, res


def rms_apply(bits: np.ndarray, weight: np.ndarray, rstd: np.ndarray) -> np.ndarray:
    """RMSNorm's output bits bf16(RN(RN(x * rstd[row]) * weight)) (``orc_rms_apply``)."""
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    weight = np.ascontiguousarray(weight, dtype=np.uint16)
    rstd = np.ascontiguousarray(rstd, dtype=np.float32)
    m, n = bits.shape
    if weight.shape != (n,) or rstd.shape != (m,):
        raise ValueError("weight must be [n] and rstd [m]")
    out = np.empty_like(bits)
    if lib().orc_rms_apply(bits.ctypes.data, weight.ctypes.data, rstd.ctypes.data, m, n,
                           out.ctypes.data) != 0:
        raise ValueError("oracle rejected the shape")
    return out


def rms_rsqrt_bound(acc: np.ndarray, n: int, eps: float) -> np.ndarray:
    """1/sqrt(RN(RN(acc / n) + eps)) in float64: the value the device's rsqrtf
    approximates (to within 2 ulp, CUDA's stated bound)."""
    mean = np.float32(acc) / np.float32(n)
    return 1.0 / np.sqrt((mean + np.float32(eps)).astype(np.float64))


def absmax(bits: np.ndarray, dtype: str = "bf16", nthreads: int = 0) -> float:
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    return float(lib().orc_absmax(bits.ctypes.data, _DTYPES[dtype], bits.size, int(nthreads)))


def global_scale_inv(amax: float, fp8_max: float) -> float:
    return float(lib().orc_global_scale_inv(float(amax), float(np.float32(fp8_max * 6.0))))


def dequantize(codes: np.ndarray, scales: np.ndarray, m: int, n: int,
               swizzled: bool = True) -> np.ndarray:
    """e2m1 * e4m3 per element (global scale not applied), float32 [m, n]."""
    codes = np.ascontiguousarray(codes, np.uint8)
    scales = np.ascontiguousarray(scales, np.uint8)
    out = np.empty((m, n), np.float32)
    rc = lib().orc_dequantize(codes.ctypes.data, scales.ctypes.data, m, n, int(swizzled),
                              out.ctypes.data)
    if rc != 0:
        raise ValueError("oracle rejected the shape")
    return out


def gemm(a_codes, a_scales, b_codes, b_scales, m: int, n: int, k: int,
         alpha: float) -> np.ndarray:
    """NVFP4 linear layer reference: alpha * deq(A) @ deq(B)^T in float64.

    Follows the dequantize-then-matmul fallback of
    ``benchmark_nvfp4_tokens.py:84-106`` (global scale 1 on both operands,
    ``alpha`` applied to the product), without the bf16 rounding of the
    operands, which is exact anyway because e2m1*e4m3 products are exact.
    """
    a = dequantize(a_codes, a_scales, m, k).astype(np.float64)
    b = dequantize(b_codes, b_scales, n, k).astype(np.float64)
    return (a @ b.T) * float(alpha)


def e2m1_encode(x: float) -> int:
    return int(lib().orc_e2m1_encode(float(x)))


def e4m3_encode(x: float) -> int:
    return int(lib().orc_e4m3_encode(float(x)))


def e4m3_decode(raw: int) -> float:
    return float(lib().orc_e4m3_decode(int(raw)))
