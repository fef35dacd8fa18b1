"""Per-tensor amax and the global-scale multiplier on the GPU.

The reference computes, per call and outside its kernels,
``(fp8_max * 6) / x.abs().max().float()`` with torch
(``bench_kernel/test_kernel_latency.py:65-75``), where fp8_max is 256 for the
scale-sweep backends and 448 for RTN.  torch evaluates that division as
``reciprocal(amax) * (fp8_max*6)`` (two roundings); the kernels here do the
same, in one pass over the tensor, without a host synchronisation, so the
result can stay on the device and the sequence is CUDA-graph capturable.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

SCALESWEEP_BACKENDS = frozenset({"scalesweep_mse", "scalesweep_mse_reference"})
FP4_E2M1_MAX = 6.0


def fp8_scale_max(backend: str) -> float:
    """FP8 range used to derive a backend's global-scale multiplier (reference :73-75)."""
    return 256.0 if backend in SCALESWEEP_BACKENDS else 448.0


def _workspace(device: torch.device) -> torch.Tensor:
    n = int(_lib.lib().ssw_absmax_workspace_bytes())
    return torch.empty((n + 3) // 4, dtype=torch.int32, device=device)


def _check_input(x: torch.Tensor) -> None:
    if not x.is_cuda:
        raise ValueError("input must be a CUDA tensor (there is no CPU implementation)")
    if not x.is_contiguous():
        raise ValueError("input must be contiguous")


def absmax(x: torch.Tensor, *, out: torch.Tensor | None = None) -> torch.Tensor:
    """max |x| as a float32 tensor of shape [1] (NaN if x holds a NaN)."""
    _check_input(x)
    dev = x.device
    if out is None:
        out = torch.empty(1, dtype=torch.float32, device=dev)
    ws = _workspace(dev)
    with torch.cuda.device(dev):
        st = _lib.lib().ssw_absmax(ctypes.c_void_p(x.data_ptr()), _lib.dtype_code(x), x.numel(),
                                   ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(ws.data_ptr()),
                                   ctypes.c_void_p(_lib.stream_handle(dev)))
    _lib.check(st)
    return out


def global_scale_from_amax(amax: torch.Tensor, fp8_max: float, *,
                           out: torch.Tensor | None = None) -> torch.Tensor:
    """(fp8_max*6) / amax, torch's rounding, on the device."""
    if amax.dtype != torch.float32 or not amax.is_cuda:
        raise ValueError("amax must be a float32 CUDA tensor")
    dev = amax.device
    if out is None:
        out = torch.empty(1, dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        st = _lib.lib().ssw_global_scale_from_amax(
            ctypes.c_void_p(amax.data_ptr()), float(fp8_max), ctypes.c_void_p(out.data_ptr()),
            ctypes.c_void_p(_lib.stream_handle(dev)))
    _lib.check(st)
    return out


def global_scale_inv_from_max(x: torch.Tensor, fp8_max: float, *,
                              out: torch.Tensor | None = None,
                              amax_out: torch.Tensor | None = None) -> torch.Tensor:
    """Fused amax + multiplier in one launch; returns a float32 tensor [1]."""
    _check_input(x)
    dev = x.device
    if out is None:
        out = torch.empty(1, dtype=torch.float32, device=dev)
    ws = _workspace(dev)
    amax_ptr = ctypes.c_void_p(amax_out.data_ptr()) if amax_out is not None else None
    with torch.cuda.device(dev):
        st = _lib.lib().ssw_global_scale_inv(
            ctypes.c_void_p(x.data_ptr()), _lib.dtype_code(x), x.numel(), float(fp8_max),
            ctypes.c_void_p(out.data_ptr()), amax_ptr, ctypes.c_void_p(ws.data_ptr()),
            ctypes.c_void_p(_lib.stream_handle(dev)))
    _lib.check(st)
    return out


def global_scale_inv(activations: torch.Tensor, backend: str) -> torch.Tensor:
    """Drop-in for ``bench_kernel/test_kernel_latency.py:65-70``."""
    return global_scale_inv_from_max(activations, fp8_scale_max(backend))
