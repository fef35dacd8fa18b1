"""Scale-sweep MSE NVFP4 activation quantizer -- B200 drop-in for the reference's
``bench_kernel/scalesweep_mse_nvfp4_utils.py`` (same names, signatures,
outputs and errors).

Per 16-element block: normalise by the global-scale multiplier, take the block
amax, build the 11-candidate E4M3 scale window [code-3, code+7] around the
nearest-even code of amax/6 (clamped to [1, 126]), E2M1-round-trip each
candidate, keep the smallest fp32 squared error (sequential FMA chain; first
index wins ties), then store the packed codes and the swizzled scale.  The
work runs in hand-written sm_100a CUDA (``csrc/quant.cu``) through the C ABI;
there is no CPU fallback.
"""
from __future__ import annotations

import torch

from . import _quant
from .custom import create_fp4_output_tensors

BLOCK_SIZE = 16
LOWER_BOUND = -3
UPPER_BOUND = 7
FP4_E2M1_MAX = 6.0
REF_MAX_SCALE_RAW = 126


def _scalesweep_mse_nvfp4_quant_out(input: torch.Tensor, input_scale: torch.Tensor,
                                    is_sf_swizzled_layout: bool, output: torch.Tensor,
                                    output_scale: torch.Tensor, use_full_range: bool) -> None:
    """Launcher (reference :424-459)."""
    _quant.launch("mse128" if use_full_range else "mse", input, input_scale,
                  is_sf_swizzled_layout, output, output_scale)


def scalesweep_mse_nvfp4_quant_out(input: torch.Tensor, input_scale: torch.Tensor,
                                   is_sf_swizzled_layout: bool = True, *, output: torch.Tensor,
                                   output_scale: torch.Tensor) -> None:
    """In-place variant (reference :462-477)."""
    _scalesweep_mse_nvfp4_quant_out(input, input_scale, is_sf_swizzled_layout, output,
                                    output_scale, use_full_range=False)


def scalesweep_mse128_nvfp4_quant_out(input: torch.Tensor, input_scale: torch.Tensor,
                                      is_sf_swizzled_layout: bool = True, *, output: torch.Tensor,
                                      output_scale: torch.Tensor) -> None:
    """Full-range (126 candidates) in-place variant (reference :480-495)."""
    _scalesweep_mse_nvfp4_quant_out(input, input_scale, is_sf_swizzled_layout, output,
                                    output_scale, use_full_range=True)


def scalesweep_mse_nvfp4_quant_impl(input: torch.Tensor, input_scale: torch.Tensor,
                                    is_sf_swizzled_layout: bool = True,
                                    padded_n: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Allocating variant (reference :498-519): returns (codes uint8, scales float8_e4m3fn)."""
    m, n = input.shape
    output, output_scale = create_fp4_output_tensors(m, n, input.device, is_sf_swizzled_layout,
                                                     padded_n=padded_n)
    scalesweep_mse_nvfp4_quant_out(input, input_scale, is_sf_swizzled_layout, output=output,
                                   output_scale=output_scale)
    return output, output_scale.view(torch.float8_e4m3fn)


def scalesweep_mse128_nvfp4_quant_impl(input: torch.Tensor, input_scale: torch.Tensor,
                                       is_sf_swizzled_layout: bool = True,
                                       padded_n: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Allocating full-range variant (reference :522-543)."""
    m, n = input.shape
    output, output_scale = create_fp4_output_tensors(m, n, input.device, is_sf_swizzled_layout,
                                                     padded_n=padded_n)
    scalesweep_mse128_nvfp4_quant_out(input, input_scale, is_sf_swizzled_layout, output=output,
                                      output_scale=output_scale)
    return output, output_scale.view(torch.float8_e4m3fn)


def rtn_nvfp4_quant_out(input: torch.Tensor, input_scale: torch.Tensor,
                        is_sf_swizzled_layout: bool = True, *, output: torch.Tensor,
                        output_scale: torch.Tensor) -> None:
    """Plain round-to-nearest comparator: the window's base code, no sweep."""
    _quant.launch("rtn", input, input_scale, is_sf_swizzled_layout, output, output_scale)


def rtn_nvfp4_quant_impl(input: torch.Tensor, input_scale: torch.Tensor,
                         is_sf_swizzled_layout: bool = True,
                         padded_n: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    m, n = input.shape
    output, output_scale = create_fp4_output_tensors(m, n, input.device, is_sf_swizzled_layout,
                                                     padded_n=padded_n)
    rtn_nvfp4_quant_out(input, input_scale, is_sf_swizzled_layout, output=output,
                        output_scale=output_scale)
    return output, output_scale.view(torch.float8_e4m3fn)


def _scalesweep_mse_nvfp4_quant_fake(input: torch.Tensor, input_scale: torch.Tensor,
                                     is_sf_swizzled_layout: bool = True,
                                     padded_n: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Shape function for op registration (reference :546-561)."""
    n = input.shape[-1]
    m = input.numel() // n
    output, output_scale = create_fp4_output_tensors(m, n, input.device, is_sf_swizzled_layout,
                                                     padded_n=padded_n)
    return output, output_scale.view(torch.float8_e4m3fn)


def _scalesweep_mse_nvfp4_quant_out_fake(input: torch.Tensor, input_scale: torch.Tensor,
                                         is_sf_swizzled_layout: bool = True, *,
                                         output: torch.Tensor, output_scale: torch.Tensor) -> None:
    """(reference :564-572)"""
    return None
