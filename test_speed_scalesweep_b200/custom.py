"""NVFP4 quantization dispatch -- drop-in for the reference's ``bench_kernel/custom.py``.

``nvfp4_quant`` keeps the reference's signature, reshaping and errors
(``bench_kernel/custom.py:10-53``) and maps backend names to the B200 kernels
of this package.  ``create_fp4_output_tensors`` allocates exactly what
vLLM's helper of the same name allocates (the reference imports it from
``vllm._custom_ops``): codes ``uint8 [m, physical_n/2]`` and scales either
``int32 [round_up(m,128), round_up(physical_n/16,4)/4]`` (swizzled) or
``uint8 [m, physical_n/16]``.
"""
from __future__ import annotations

import torch

BLOCK_SIZE = 16


def round_up(x: int, y: int) -> int:
    return (x + y - 1) // y * y


def create_fp4_scale_tensor(m: int, n: int, device: torch.device,
                            is_sf_swizzled_layout: bool) -> torch.Tensor:
    if is_sf_swizzled_layout:
        return torch.empty((round_up(m, 128), round_up(n // BLOCK_SIZE, 4) // 4), device=device,
                           dtype=torch.int32)
    return torch.empty((m, n // BLOCK_SIZE), device=device, dtype=torch.uint8)


def create_fp4_output_tensors(m: int, n: int, device: torch.device, is_sf_swizzled_layout: bool,
                              padded_n: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    physical_n = padded_n if padded_n is not None else n
    output = torch.empty((m, physical_n // 2), device=device, dtype=torch.uint8)
    output_scale = create_fp4_scale_tensor(m, physical_n, device, is_sf_swizzled_layout)
    return output, output_scale


def _vllm_rtn(input, input_global_scale, is_sf_swizzled_layout, padded_n):
    try:
        from vllm import _custom_ops as vllm_ops
    except Exception as exc:  # pragma: no cover - depends on the vLLM install
        raise RuntimeError("backend 'cutlass'/'vllm' needs vLLM's compiled ops") from exc
    return vllm_ops.scaled_fp4_quant(input, input_global_scale, is_sf_swizzled_layout,
                                     backend="cutlass", padded_n=padded_n)


def nvfp4_quant(input: torch.Tensor, input_global_scale: torch.Tensor,
                is_sf_swizzled_layout: bool = True, backend: str = "scalesweep_mse",
                padded_n: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Quantize ``input`` to NVFP4 with the selected backend.

    Same contract as the reference dispatcher: any-rank input is flattened to
    ``[-1, K]``; ``K`` must be a multiple of 16.
    """
    if input.ndim < 1:
        raise ValueError("input must have at least one dimension")
    input = input.reshape(1 if input.ndim == 1 else -1, input.shape[-1])
    if input.shape[-1] % 16:
        raise ValueError("the last input dimension must be a multiple of 16")

    if backend in {"cutlass", "vllm"}:
        return _vllm_rtn(input, input_global_scale, is_sf_swizzled_layout, padded_n)

    from . import scalesweep_mse_nvfp4_utils as mse
    from . import scalesweep_mse_reference_nvfp4_utils as mse_reference
    from . import scalesweep_nvfp4_utils as sweep

    implementations = {
        "scalesweep": sweep.scalesweep_nvfp4_quant_impl,
        "scalesweep128": sweep.scalesweep128_nvfp4_quant_impl,
        "scalesweep_mse": mse.scalesweep_mse_nvfp4_quant_impl,
        "scalesweep_mse_reference": mse_reference.scalesweep_mse_nvfp4_quant_impl,
        "scalesweep_mse128": mse.scalesweep_mse128_nvfp4_quant_impl,
        "rtn": mse.rtn_nvfp4_quant_impl,
    }
    try:
        implementation = implementations[backend]
    except KeyError as exc:
        raise ValueError(f"Unsupported backend: {backend}") from exc
    return implementation(input, input_global_scale, is_sf_swizzled_layout, padded_n)


__all__ = ["create_fp4_output_tensors", "nvfp4_quant"]
