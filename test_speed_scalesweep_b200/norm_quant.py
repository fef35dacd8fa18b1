"""RMSNorm fused into the scale-sweep quantizer.

In a Llama decoder layer the qkv and gate_up projections read RMSNorm's
output.  vLLM's ``fuse_norm_quant`` compile pass replaces ``rms_norm`` (or
``fused_add_rms_norm``) followed by a quant op with one fused op (vllm 0.22
``compilation/passes/fusion/rms_quant_fusion.py:103-128``, FP8 keys only);
the reference switches that pass off (``run_bench_tune.sh:24,31``) so that
its own quantizer runs on the normalised bf16 tensor.

This module gives the scale-sweep form: the same codes and scales as
``scalesweep_mse_nvfp4_quant`` applied to vLLM's RMSNorm output, without
writing that output.  A row-statistics kernel forms ``1/rms`` exactly as
vLLM's kernels do (block size, vector order and reduction tree), then the
quantizer normalises each 16-element block while it loads it.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._quant import required_scale_bytes
from .custom import BLOCK_SIZE, round_up


def _check(input: torch.Tensor, weight: torch.Tensor, residual: torch.Tensor | None):
    if input.dtype != torch.bfloat16:
        raise ValueError(f"input must be bf16, got {input.dtype}")
    if input.dim() < 1 or input.shape[-1] % BLOCK_SIZE:
        raise ValueError(f"the last dimension of input must be a multiple of {BLOCK_SIZE}")
    n = input.shape[-1]
    if weight.dtype != torch.bfloat16 or weight.shape != (n,):
        raise ValueError(f"weight must be a bf16 tensor of shape [{n}]")
    if residual is not None and (residual.dtype != torch.bfloat16 or residual.shape != input.shape):
        raise ValueError("residual must be a bf16 tensor of the input's shape")
    tensors = (input, weight) + ((residual,) if residual is not None else ())
    if not all(t.is_cuda for t in tensors):
        raise ValueError("input, weight and residual must be CUDA tensors "
                         "(there is no CPU implementation)")
    if any(t.device != input.device for t in tensors):
        raise ValueError("input, weight and residual must be on one device")
    if not all(t.is_contiguous() for t in tensors):
        raise ValueError("input, weight and residual must be contiguous")
    m = input.numel() // n if n else 0
    return m, n


def alloc_outputs(input: torch.Tensor, is_sf_swizzled_layout: bool = True):
    """Codes uint8 [m, n/2] and scales float8_e4m3fn ([round_up(m,128),
    round_up(n/16,4)] swizzled, else [m, n/16]) for an [.., n] input."""
    n = input.shape[-1]
    m = input.numel() // n if n else 0
    codes = input.new_empty((m, n // 2), dtype=torch.uint8)
    bpc = n // BLOCK_SIZE
    shape = (round_up(m, 128), round_up(bpc, 4)) if is_sf_swizzled_layout else (m, bpc)
    return codes, input.new_empty(shape, dtype=torch.float8_e4m3fn)


def rms_norm_scalesweep_mse_nvfp4_quant_out(input: torch.Tensor, weight: torch.Tensor,
                                            epsilon: float, input_scale: torch.Tensor,
                                            is_sf_swizzled_layout: bool = True, *,
                                            output: torch.Tensor, output_scale: torch.Tensor,
                                            residual: torch.Tensor | None = None,
                                            rstd: torch.Tensor | None = None) -> None:
    """Quantize vLLM's RMSNorm output with the scalesweep_mse sweep into
    ``output`` [m, n/2] and ``output_scale``.

    ``residual`` None: the normalised tensor is ``rms_norm(input, weight,
    epsilon)``.  Otherwise it is ``fused_add_rms_norm``'s: ``residual`` is
    updated in place to ``bf16(input + residual)`` and that is normalised;
    ``input`` is left as it is (vLLM would overwrite it with the normalised
    bf16 values, which nothing here needs).

    ``rstd``: optional float32 device workspace of at least m elements; it is
    left holding each row's 1/rms.  One is allocated when it is None."""
    m, n = _check(input, weight, residual)
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
    if rstd is None:
        rstd = torch.empty(max(m, 1), dtype=torch.float32, device=dev)
    elif (rstd.device != dev or rstd.dtype != torch.float32 or not rstd.is_contiguous()
          or rstd.numel() < m):
        raise ValueError(f"rstd must be a contiguous float32 tensor of at least {m} elements "
                         f"on {dev}")
    h = _lib.lib()
    with torch.cuda.device(dev):
        st = h.ssw_rms_norm_scalesweep_mse_nvfp4_quant_out(
            ctypes.c_void_p(input.data_ptr()),
            ctypes.c_void_p(residual.data_ptr() if residual is not None else 0),
            ctypes.c_void_p(weight.data_ptr()), float(epsilon), m, n,
            ctypes.c_void_p(input_scale.data_ptr()), ctypes.c_void_p(output.data_ptr()),
            ctypes.c_void_p(output_scale.data_ptr()), int(bool(is_sf_swizzled_layout)),
            ctypes.c_void_p(rstd.data_ptr()), ctypes.c_void_p(_lib.stream_handle(dev)))
    _lib.check(st)


def rms_norm_scalesweep_mse_nvfp4_quant(input: torch.Tensor, weight: torch.Tensor,
                                        epsilon: float, input_scale: torch.Tensor,
                                        is_sf_swizzled_layout: bool = True,
                                        residual: torch.Tensor | None = None):
    """Functional form: returns (codes, scales); updates ``residual`` in place
    when one is given."""
    codes, scales = alloc_outputs(input, is_sf_swizzled_layout)
    rms_norm_scalesweep_mse_nvfp4_quant_out(input, weight, epsilon, input_scale,
                                            is_sf_swizzled_layout, output=codes,
                                            output_scale=scales, residual=residual)
    return codes, scales
