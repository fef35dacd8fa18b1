"""Block-scaled NVFP4 GEMM (tcgen05, sm_100a) with the signature of vLLM's
``cutlass_scaled_fp4_mm`` (vllm 0.22 ``_custom_ops.py:741-753``), the consumer
of the quantizer's codes and swizzled scales in a W4A4 linear layer
(``model_executor/kernels/linear/nvfp4/cutlass.py:64-71``)."""
from __future__ import annotations

import ctypes

import torch

from . import _lib


def cutlass_scaled_fp4_mm(a: torch.Tensor, b: torch.Tensor, block_scale_a: torch.Tensor,
                          block_scale_b: torch.Tensor, alpha: torch.Tensor,
                          out_dtype: torch.dtype = torch.bfloat16,
                          status: torch.Tensor | None = None,
                          split_k: bool = True,
                          dependent_launch: bool = False) -> torch.Tensor:
    """``alpha * (A ⊙ sfA) @ (B ⊙ sfB)^T`` in bf16.

    a: uint8 [M, K/2] E2M1 codes; b: uint8 [N, K/2]; block_scale_a/b: E4M3
    scales in the 128x4-swizzled layout; alpha: float32 device scalar.
    K must be a multiple of 256 and N a multiple of 64.  When the output has
    too few tiles to fill the GPU the K loop is split across CTAs (workspace
    from torch's caching allocator); ``split_k=False`` forces one pass.
    ``dependent_launch=True`` launches it as a programmatic dependent of the
    kernel before it on the stream (``ssw_nvfp4_gemm_dependent``): its
    prologue and weight loads overlap that kernel, and A is read only after it.
    """
    if out_dtype != torch.bfloat16:
        raise ValueError("only bf16 output is implemented")
    for name, t in (("a", a), ("b", b), ("block_scale_a", block_scale_a),
                    ("block_scale_b", block_scale_b), ("alpha", alpha)):
        if not t.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor")
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
        if t.device != a.device:
            raise ValueError(f"{name} must be on {a.device}, got {t.device}")
    if status is not None and (status.device != a.device or status.dtype != torch.int32):
        raise ValueError(f"status must be an int32 tensor on {a.device}")
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[1]:
        raise ValueError("a [M, K/2] and b [N, K/2] must share K")
    m, n, k = a.shape[0], b.shape[0], a.shape[1] * 2
    kpad = (k // 16 + 3) // 4 * 4
    if block_scale_a.numel() * block_scale_a.element_size() < (m + 127) // 128 * 128 * kpad:
        raise ValueError("block_scale_a is smaller than the swizzled layout of A")
    if block_scale_b.numel() * block_scale_b.element_size() < (n + 127) // 128 * 128 * kpad:
        raise ValueError("block_scale_b is smaller than the swizzled layout of B")
    if alpha.dtype != torch.float32:
        raise ValueError("alpha must be float32")
    out = torch.empty((m, n), dtype=torch.bfloat16, device=a.device)
    st_ptr = ctypes.c_void_p(status.data_ptr()) if status is not None else None
    h = _lib.lib()
    with torch.cuda.device(a.device):
        ws_bytes = int(h.ssw_nvfp4_gemm_workspace_bytes(m, n, k)) if split_k else 0
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=a.device) if ws_bytes else None
        fn = h.ssw_nvfp4_gemm_dependent if dependent_launch else h.ssw_nvfp4_gemm
        st = fn(
            ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(b.data_ptr()),
            ctypes.c_void_p(block_scale_a.data_ptr()), ctypes.c_void_p(block_scale_b.data_ptr()),
            ctypes.c_void_p(alpha.data_ptr()), ctypes.c_void_p(out.data_ptr()), m, n, k,
            ctypes.c_void_p(ws.data_ptr()) if ws is not None else None, ws_bytes, st_ptr,
            ctypes.c_void_p(_lib.stream_handle(a.device)))
    _lib.check(st)
    return out


def scalesweep_nvfp4_linear(x: torch.Tensor, input_scale: torch.Tensor, weight: torch.Tensor,
                            weight_scale: torch.Tensor, alpha: torch.Tensor,
                            out_dtype: torch.dtype = torch.bfloat16,
                            status: torch.Tensor | None = None) -> torch.Tensor:
    """A W4A4 linear layer in one call: scale-sweep MSE quantization of the
    activation ``x`` [M, K] (bf16/f16) with ``input_scale`` (its
    global-scale inverse), then the NVFP4 GEMM against ``weight`` [N, K/2]
    and its swizzled ``weight_scale``.  The result equals
    ``cutlass_scaled_fp4_mm(*scalesweep_mse_nvfp4_quant(x, input_scale), ...)``
    bit for bit; the GEMM is launched as a programmatic dependent of the
    quantizer, so its prologue and first weight loads overlap it.  This is
    the scaled_fp4_quant + cutlass_scaled_fp4_mm pair of vLLM's W4A4 linear
    layer (vllm 0.22 ``model_executor/kernels/linear/nvfp4/cutlass.py:56-71``)."""
    if out_dtype != torch.bfloat16:
        raise ValueError("only bf16 output is implemented")
    if x.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError(f"x must be bf16 or f16, got {x.dtype}")
    for name, t in (("x", x), ("input_scale", input_scale), ("weight", weight),
                    ("weight_scale", weight_scale), ("alpha", alpha)):
        if not t.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor")
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
        if t.device != x.device:
            raise ValueError(f"{name} must be on {x.device}, got {t.device}")
    if input_scale.dtype != torch.float32 or alpha.dtype != torch.float32:
        raise ValueError("input_scale and alpha must be float32")
    if status is not None and (status.device != x.device or status.dtype != torch.int32):
        raise ValueError(f"status must be an int32 tensor on {x.device}")
    k = x.shape[-1]
    m = x.numel() // k if k else 0
    if weight.dim() != 2 or weight.shape[1] * 2 != k:
        raise ValueError("weight must be [N, K/2] codes matching x's K")
    n = weight.shape[0]
    kpad = (k // 16 + 3) // 4 * 4
    if weight_scale.numel() * weight_scale.element_size() < (n + 127) // 128 * 128 * kpad:
        raise ValueError("weight_scale is smaller than the swizzled layout of the weight")
    out = torch.empty(x.shape[:-1] + (n,), dtype=torch.bfloat16, device=x.device)
    h = _lib.lib()
    st_ptr = ctypes.c_void_p(status.data_ptr()) if status is not None else None
    with torch.cuda.device(x.device):
        ws_bytes = int(h.ssw_nvfp4_quant_gemm_workspace_bytes(m, n, k)) if m else 0
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device)
        st = h.ssw_nvfp4_quant_gemm(
            ctypes.c_void_p(x.data_ptr()), _lib.dtype_code(x), ctypes.c_void_p(input_scale.data_ptr()),
            ctypes.c_void_p(weight.data_ptr()), ctypes.c_void_p(weight_scale.data_ptr()),
            ctypes.c_void_p(alpha.data_ptr()), ctypes.c_void_p(out.data_ptr()), m, n, k,
            ctypes.c_void_p(ws.data_ptr()), ws_bytes, st_ptr,
            ctypes.c_void_p(_lib.stream_handle(x.device)))
    _lib.check(st)
    return out
