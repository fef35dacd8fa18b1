"""SiLU-and-mul and its fusion into the scale-sweep quantizer.

In a SwiGLU MLP the down projection's activation is ``silu(gate) * up``.
vLLM computes it with ``silu_and_mul`` and, when its ``fuse_act_quant``
compile pass is on, replaces ``silu_and_mul`` + ``scaled_fp4_quant`` with the
fused ``silu_and_mul_nvfp4_quant`` (vllm 0.22
``compilation/passes/fusion/act_quant_fusion.py:124-172``).  The reference
turns that pass off (``run_bench_tune.sh:24,31``) so that its own quantizer
runs, at the price of writing and re-reading the bf16 intermediate.

This module provides the scale-sweep version of the fused op: the same codes
and scales as ``scalesweep_mse_nvfp4_quant`` applied to ``silu_and_mul``'s
output, from one kernel that never writes the intermediate.  ``silu_and_mul``
itself is here too; it equals vLLM's bit for bit (every bf16 and f16 gate
value was checked on a B200).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._quant import required_scale_bytes
from .custom import BLOCK_SIZE, round_up


def _rows(input: torch.Tensor) -> tuple[torch.Tensor, int, int]:
    if input.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError(f"input must be bf16 or f16, got {input.dtype}")
    if input.dim() < 1 or input.shape[-1] % 2:
        raise ValueError("the last dimension of input holds gate and up halves and must be even")
    n = input.shape[-1] // 2
    if n % BLOCK_SIZE:
        raise ValueError(f"the output width ({n}) must be a multiple of {BLOCK_SIZE}")
    if not input.is_cuda:
        raise ValueError("input must be a CUDA tensor (there is no CPU implementation)")
    if not input.is_contiguous():
        raise ValueError("input must be contiguous")
    m = input.numel() // input.shape[-1] if input.shape[-1] else 0
    return input.reshape(m, 2 * n), m, n


def silu_and_mul(input: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """``silu(input[..., :n]) * input[..., n:]`` as vLLM's ``silu_and_mul``
    computes it (silu in fp32 rounded to the input type, times up)."""
    x, m, n = _rows(input)
    if out is None:
        out = torch.empty(input.shape[:-1] + (n,), dtype=input.dtype, device=input.device)
    if out.dtype != input.dtype or out.device != input.device or not out.is_contiguous():
        raise ValueError("out must be a contiguous tensor of the input's dtype and device")
    if out.numel() != m * n:
        raise ValueError(f"out must hold {m} x {n} elements")
    h = _lib.lib()
    with torch.cuda.device(input.device):
        st = h.ssw_silu_and_mul(ctypes.c_void_p(x.data_ptr()), _lib.dtype_code(input), m, n,
                                ctypes.c_void_p(out.data_ptr()),
                                ctypes.c_void_p(_lib.stream_handle(input.device)))
    _lib.check(st)
    return out


def silu_and_mul_scalesweep_mse_nvfp4_quant_out(input: torch.Tensor, input_scale: torch.Tensor,
                                                is_sf_swizzled_layout: bool = True, *,
                                                output: torch.Tensor,
                                                output_scale: torch.Tensor) -> None:
    """Quantize ``silu_and_mul(input)`` with the scalesweep_mse sweep into
    ``output`` [m, n/2] and ``output_scale`` without materialising it."""
    x, m, n = _rows(input)
    dev = input.device
    for name, t in (("input_scale", input_scale), ("output", output),
                    ("output_scale", output_scale)):
        if t.device != dev:
            raise ValueError(f"{name} must be on {dev}, got {t.device}")
    if input_scale.dtype != torch.float32 or input_scale.numel() < 1:
        raise ValueError("input_scale must be a float32 tensor with at least one element")
    if not (output.is_contiguous() and output_scale.is_contiguous()):
        raise ValueError("output and output_scale must be contiguous")
    if output.element_size() != 1 or output.numel() != m * (n // 2):
        raise ValueError(f"output must be a 1-byte tensor of shape [{m}, {n // 2}]")
    need = required_scale_bytes(m, n, is_sf_swizzled_layout)
    have = output_scale.numel() * output_scale.element_size()
    if have < need:
        raise ValueError(f"output_scale holds {have} bytes, the layout needs {need}")
    h = _lib.lib()
    with torch.cuda.device(dev):
        st = h.ssw_silu_and_mul_scalesweep_mse_nvfp4_quant_out(
            ctypes.c_void_p(x.data_ptr()), _lib.dtype_code(input), m, n,
            ctypes.c_void_p(input_scale.data_ptr()), ctypes.c_void_p(output.data_ptr()),
            ctypes.c_void_p(output_scale.data_ptr()), int(bool(is_sf_swizzled_layout)),
            ctypes.c_void_p(_lib.stream_handle(dev)))
    _lib.check(st)


def alloc_outputs(input: torch.Tensor, is_sf_swizzled_layout: bool = True):
    """Codes uint8 [m, n/2] and scales float8_e4m3fn ([round_up(m,128),
    round_up(n/16,4)] swizzled, else [m, n/16]) for a [.., 2n] input."""
    n = input.shape[-1] // 2
    m = input.numel() // input.shape[-1] if input.shape[-1] else 0
    codes = input.new_empty((m, n // 2), dtype=torch.uint8)
    bpc = n // BLOCK_SIZE
    shape = (round_up(m, 128), round_up(bpc, 4)) if is_sf_swizzled_layout else (m, bpc)
    return codes, input.new_empty(shape, dtype=torch.float8_e4m3fn)


def silu_and_mul_scalesweep_mse_nvfp4_quant(input: torch.Tensor, input_scale: torch.Tensor,
                                            is_sf_swizzled_layout: bool = True):
    """Functional form: returns (codes, scales)."""
    codes, scales = alloc_outputs(input, is_sf_swizzled_layout)
    silu_and_mul_scalesweep_mse_nvfp4_quant_out(input, input_scale, is_sf_swizzled_layout,
                                                output=codes, output_scale=scales)
    return codes, scales


def silu_and_mul_nvfp4_quant(result: torch.Tensor, result_block_scale: torch.Tensor,
                             input: torch.Tensor, input_global_scale: torch.Tensor) -> None:
    """vLLM's fused-op signature (``torch.ops._C.silu_and_mul_nvfp4_quant``:
    result, swizzled result_block_scale, input, input_global_scale), with the
    scale-sweep quantizer behind it."""
    silu_and_mul_scalesweep_mse_nvfp4_quant_out(input, input_global_scale, True, output=result,
                                                output_scale=result_block_scale)
