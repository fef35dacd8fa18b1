"""Scale-sweep MSE NVFP4 quantizer, "reference" variant -- B200 drop-in for the
reference's ``bench_kernel/scalesweep_mse_reference_nvfp4_utils.py``.

Differs from ``scalesweep_mse_nvfp4_utils`` in two numerically visible ways,
reproduced bit-exactly: the base code is the largest E4M3 value not above
amax/6 (:347-351), and the 16 squared errors are summed as a pairwise tree
(:91-143).  ``padded_n`` other than the input width is rejected (:420-426,
:455-459).
"""
from __future__ import annotations

import torch

from . import _quant
from .custom import create_fp4_output_tensors

BLOCK_SIZE = 16
LOWER_BOUND = -3
UPPER_BOUND = 7

_PADDED_N_MSG = ("The reference ScaleSweep kernel does not support padded_n different "
                 "from the input width.")


def scalesweep_mse_nvfp4_quant_out(input: torch.Tensor, input_scale: torch.Tensor,
                                   is_sf_swizzled_layout: bool = True, *, output: torch.Tensor,
                                   output_scale: torch.Tensor) -> None:
    """In-place variant (reference :412-445)."""
    _, n = input.shape
    physical_n = output.shape[-1] * 2
    if physical_n != n:
        raise ValueError(_PADDED_N_MSG)
    _quant.launch("reference", input, input_scale, is_sf_swizzled_layout, output, output_scale)


def scalesweep_mse_nvfp4_quant_impl(input: torch.Tensor, input_scale: torch.Tensor,
                                    is_sf_swizzled_layout: bool = True,
                                    padded_n: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Allocating variant (reference :448-474)."""
    m, n = input.shape
    if padded_n is not None and padded_n != n:
        raise ValueError(_PADDED_N_MSG)
    output, output_scale = create_fp4_output_tensors(m, n, input.device, is_sf_swizzled_layout,
                                                     padded_n=padded_n)
    scalesweep_mse_nvfp4_quant_out(input, input_scale, is_sf_swizzled_layout, output=output,
                                   output_scale=output_scale)
    return output, output_scale.view(torch.float8_e4m3fn)


def _scalesweep_mse_reference_nvfp4_quant_fake(
        input: torch.Tensor, input_scale: torch.Tensor, is_sf_swizzled_layout: bool = True,
        padded_n: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Shape function (reference :477-497)."""
    n = input.shape[-1]
    m = input.numel() // n
    if padded_n is not None and padded_n != n:
        raise ValueError(_PADDED_N_MSG)
    output, output_scale = create_fp4_output_tensors(m, n, input.device, is_sf_swizzled_layout,
                                                     padded_n=padded_n)
    return output, output_scale.view(torch.float8_e4m3fn)


def _scalesweep_mse_reference_nvfp4_quant_out_fake(input: torch.Tensor, input_scale: torch.Tensor,
                                                   is_sf_swizzled_layout: bool = True, *,
                                                   output: torch.Tensor,
                                                   output_scale: torch.Tensor) -> None:
    """(reference :500-508)"""
    return None
