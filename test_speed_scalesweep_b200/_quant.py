"""Shared host launcher: validates torch tensors and calls one C-ABI entry point."""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .custom import BLOCK_SIZE, round_up

_ENTRY = {
    "mse": "ssw_scalesweep_mse_nvfp4_quant_out",
    "mse128": "ssw_scalesweep_mse128_nvfp4_quant_out",
    "reference": "ssw_scalesweep_mse_reference_nvfp4_quant_out",
    "rtn": "ssw_rtn_nvfp4_quant_out",
    "weighted": "ssw_scalesweep_nvfp4_quant_out",
    "weighted128": "ssw_scalesweep128_nvfp4_quant_out",
}


def required_scale_bytes(m: int, physical_n: int, swizzled: bool) -> int:
    bpc = physical_n // BLOCK_SIZE
    if swizzled:
        return round_up(m, 128) * round_up(bpc, 4)
    return m * bpc


def launch(kind: str, input: torch.Tensor, input_scale: torch.Tensor, is_sf_swizzled_layout: bool,
           output: torch.Tensor, output_scale: torch.Tensor) -> None:
    """Quantize ``input`` [m, n] into ``output`` [m, physical_n/2] and ``output_scale``.

    ``physical_n = output.shape[-1] * 2`` exactly as the reference's launcher
    derives it (``bench_kernel/scalesweep_mse_nvfp4_utils.py:432-436``).
    """
    if input.dim() != 2:
        raise ValueError(f"input must be 2-D [m, n], got shape {tuple(input.shape)}")
    if not input.is_cuda:
        raise ValueError("input must be a CUDA tensor (there is no CPU implementation)")
    num_row, n = input.shape
    physical_n = output.shape[-1] * 2
    dev = input.device
    for name, t in (("input_scale", input_scale), ("output", output), ("output_scale", output_scale)):
        if t.device != dev:
            raise ValueError(f"{name} must be on {dev}, got {t.device}")
    if input_scale.dtype != torch.float32 or input_scale.numel() < 1:
        raise ValueError("input_scale must be a float32 tensor with at least one element")
    if not input.is_contiguous():
        raise ValueError("input must be contiguous")
    if not (output.is_contiguous() and output_scale.is_contiguous()):
        raise ValueError("output and output_scale must be contiguous")
    if output.element_size() != 1 or output.numel() != num_row * (physical_n // 2):
        raise ValueError(f"output must be a 1-byte tensor of shape [{num_row}, {physical_n // 2}]")
    need = required_scale_bytes(num_row, physical_n, is_sf_swizzled_layout)
    have = output_scale.numel() * output_scale.element_size()
    if have < need:
        raise ValueError(f"output_scale holds {have} bytes, the layout needs {need}")
    h = _lib.lib()
    fn = getattr(h, _ENTRY[kind])
    with torch.cuda.device(dev):
        st = fn(ctypes.c_void_p(input.data_ptr()), _lib.dtype_code(input), num_row, n, physical_n,
                ctypes.c_void_p(input_scale.data_ptr()), ctypes.c_void_p(output.data_ptr()),
                ctypes.c_void_p(output_scale.data_ptr()), int(bool(is_sf_swizzled_layout)),
                ctypes.c_void_p(_lib.stream_handle(dev)))
    _lib.check(st)
