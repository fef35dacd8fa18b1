"""Importance-weighted scale-sweep NVFP4 quantizer -- B200 drop-in for the
reference's ``bench_kernel/scalesweep_nvfp4_utils.py`` (backends
``scalesweep`` and ``scalesweep128``).

Same sweep as ``scalesweep_mse``, but each element's squared error is rounded
on its own and multiplied by a per-column importance weight before it is
accumulated (``:40-149``).  The reference's host code always passes weights
of one (``:314``), so the kernel sums the rounded squares in element order.
"""
from __future__ import annotations

import torch

from . import _quant
from .custom import create_fp4_output_tensors
from .scalesweep_mse_nvfp4_utils import (  # noqa: F401  (re-exported like the reference)
    BLOCK_SIZE, LOWER_BOUND, REF_MAX_SCALE_RAW, UPPER_BOUND, _scalesweep_mse_nvfp4_quant_fake,
    _scalesweep_mse_nvfp4_quant_out_fake)


def _scalesweep_nvfp4_quant_out(input: torch.Tensor, input_scale: torch.Tensor,
                                is_sf_swizzled_layout: bool, output: torch.Tensor,
                                output_scale: torch.Tensor, use_full_range: bool) -> None:
    """Launcher (reference :305-341)."""
    _quant.launch("weighted128" if use_full_range else "weighted", input, input_scale,
                  is_sf_swizzled_layout, output, output_scale)


def scalesweep_nvfp4_quant_out(input: torch.Tensor, input_scale: torch.Tensor,
                               is_sf_swizzled_layout: bool = True, *, output: torch.Tensor,
                               output_scale: torch.Tensor) -> None:
    """(reference :344-354)"""
    _scalesweep_nvfp4_quant_out(input, input_scale, is_sf_swizzled_layout, output, output_scale,
                                False)


def scalesweep128_nvfp4_quant_out(input: torch.Tensor, input_scale: torch.Tensor,
                                  is_sf_swizzled_layout: bool = True, *, output: torch.Tensor,
                                  output_scale: torch.Tensor) -> None:
    """(reference :357-367)"""
    _scalesweep_nvfp4_quant_out(input, input_scale, is_sf_swizzled_layout, output, output_scale,
                                True)


def _scalesweep_nvfp4_quant_impl(input: torch.Tensor, input_scale: torch.Tensor,
                                 is_sf_swizzled_layout: bool, padded_n: int | None,
                                 use_full_range: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """(reference :370-389)"""
    m, n = input.shape
    output, output_scale = create_fp4_output_tensors(m, n, input.device, is_sf_swizzled_layout,
                                                     padded_n=padded_n)
    _scalesweep_nvfp4_quant_out(input, input_scale, is_sf_swizzled_layout, output, output_scale,
                                use_full_range)
    return output, output_scale.view(torch.float8_e4m3fn)


def scalesweep_nvfp4_quant_impl(input: torch.Tensor, input_scale: torch.Tensor,
                                is_sf_swizzled_layout: bool = True,
                                padded_n: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """(reference :392-400)"""
    return _scalesweep_nvfp4_quant_impl(input, input_scale, is_sf_swizzled_layout, padded_n, False)


def scalesweep128_nvfp4_quant_impl(input: torch.Tensor, input_scale: torch.Tensor,
                                   is_sf_swizzled_layout: bool = True,
                                   padded_n: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """(reference :403-411)"""
    return _scalesweep_nvfp4_quant_impl(input, input_scale, is_sf_swizzled_layout, padded_n, True)
