"""torch.library registration of the quantizer ops (functional + ``.out``) with
fake (meta) implementations, so the ops work under torch.compile and inside
CUDA graphs exactly like the ops the reference's vLLM fork registered
(``torch.ops.vllm.scalesweep_mse_nvfp4_quant``, ...; the fake functions of
``bench_kernel/scalesweep_mse_nvfp4_utils.py:546-572`` are their shape
functions).

Ops live in the ``scalesweep_b200`` namespace.  ``register_vllm_aliases()``
additionally defines the same schemas under the ``vllm`` namespace for a
vLLM build that looks them up there.
"""
from __future__ import annotations

import torch

from . import act_quant
from . import norm_quant
from . import scalesweep_mse_nvfp4_utils as mse
from . import scalesweep_mse_reference_nvfp4_utils as mse_ref
from . import scalesweep_nvfp4_utils as sweep

NAMESPACE = "scalesweep_b200"

_FUNCTIONAL = ("(Tensor input, Tensor input_scale, bool is_sf_swizzled_layout=True, "
               "SymInt? padded_n=None) -> (Tensor, Tensor)")
_OUT = ("(Tensor input, Tensor input_scale, bool is_sf_swizzled_layout=True, *, "
        "Tensor(a!) output, Tensor(b!) output_scale) -> ()")

_OPS = {
    "scalesweep_mse_nvfp4_quant": (mse.scalesweep_mse_nvfp4_quant_impl,
                                   mse.scalesweep_mse_nvfp4_quant_out,
                                   mse._scalesweep_mse_nvfp4_quant_fake),
    "scalesweep_mse128_nvfp4_quant": (mse.scalesweep_mse128_nvfp4_quant_impl,
                                      mse.scalesweep_mse128_nvfp4_quant_out,
                                      mse._scalesweep_mse_nvfp4_quant_fake),
    "scalesweep_mse_reference_nvfp4_quant": (
        mse_ref.scalesweep_mse_nvfp4_quant_impl, mse_ref.scalesweep_mse_nvfp4_quant_out,
        mse_ref._scalesweep_mse_reference_nvfp4_quant_fake),
    "rtn_nvfp4_quant": (mse.rtn_nvfp4_quant_impl, mse.rtn_nvfp4_quant_out,
                        mse._scalesweep_mse_nvfp4_quant_fake),
    "scalesweep_nvfp4_quant": (sweep.scalesweep_nvfp4_quant_impl, sweep.scalesweep_nvfp4_quant_out,
                               mse._scalesweep_mse_nvfp4_quant_fake),
    "scalesweep128_nvfp4_quant": (sweep.scalesweep128_nvfp4_quant_impl,
                                  sweep.scalesweep128_nvfp4_quant_out,
                                  mse._scalesweep_mse_nvfp4_quant_fake),
}

_libs: dict[str, torch.library.Library] = {}


def _alloc(input, swizzled, padded_n):
    """Outputs in their final dtypes (no aliasing views): codes uint8
    [m, physical_n/2]; scales float8_e4m3fn [round_up(m,128), round_up(bpc,4)]
    when swizzled, else [m, bpc]."""
    n = input.shape[-1]
    m = input.numel() // n if n else 0
    pn = padded_n if padded_n is not None else n
    codes = input.new_empty((m, pn // 2), dtype=torch.uint8)
    bpc = pn // 16
    shape = ((m + 127) // 128 * 128, (bpc + 3) // 4 * 4) if swizzled else (m, bpc)
    return codes, input.new_empty(shape, dtype=torch.float8_e4m3fn)


def _register(namespace: str, kind: str) -> None:
    if namespace in _libs:
        return
    lib = torch.library.Library(namespace, kind)
    for name, (_impl, out, fake) in _OPS.items():
        lib.define(name + _FUNCTIONAL)
        lib.define(name + ".out" + _OUT)

        def functional(input, input_scale, is_sf_swizzled_layout=True, padded_n=None, _out=out):
            codes, scales = _alloc(input, is_sf_swizzled_layout, padded_n)
            _out(input, input_scale, is_sf_swizzled_layout, output=codes, output_scale=scales)
            return codes, scales

        def out_variant(input, input_scale, is_sf_swizzled_layout=True, *, output, output_scale,
                        _out=out):
            _out(input, input_scale, is_sf_swizzled_layout, output=output,
                 output_scale=output_scale)

        def fake_functional(input, input_scale, is_sf_swizzled_layout=True, padded_n=None,
                            _fake=fake):
            _fake(input, input_scale, is_sf_swizzled_layout, padded_n)  # argument checks
            return _alloc(input, is_sf_swizzled_layout, padded_n)

        def fake_out(input, input_scale, is_sf_swizzled_layout=True, *, output, output_scale):
            return None

        lib.impl(name, functional, "CUDA")
        lib.impl(name + ".out", out_variant, "CUDA")
        torch.library.register_fake(f"{namespace}::{name}", fake_functional, lib=lib)
        torch.library.register_fake(f"{namespace}::{name}.out", fake_out, lib=lib)
    if namespace == NAMESPACE:
        _register_act_quant(lib, namespace)
        _register_norm_quant(lib, namespace)
        _register_linear(lib, namespace)
    _libs[namespace] = lib


def _register_linear(lib: torch.library.Library, namespace: str) -> None:
    """The W4A4 linear layer in one op (``gemm.scalesweep_nvfp4_linear``):
    scale-sweep quantization of ``x`` [M, K] and the NVFP4 GEMM against
    ``weight`` [N, K/2], bf16 [M, N] out."""
    from . import gemm

    lib.define("scalesweep_nvfp4_linear(Tensor x, Tensor input_scale, Tensor weight, "
               "Tensor weight_scale, Tensor alpha) -> Tensor")

    def linear(x, input_scale, weight, weight_scale, alpha):
        return gemm.scalesweep_nvfp4_linear(x, input_scale, weight, weight_scale, alpha)

    def fake_linear(x, input_scale, weight, weight_scale, alpha):
        return x.new_empty(tuple(x.shape[:-1]) + (weight.shape[0],), dtype=torch.bfloat16)

    lib.impl("scalesweep_nvfp4_linear", linear, "CUDA")
    torch.library.register_fake(f"{namespace}::scalesweep_nvfp4_linear", fake_linear, lib=lib)


def _register_act_quant(lib: torch.library.Library, namespace: str) -> None:
    """SiLU-and-mul and the fused SiLU-and-mul quantizer (act_quant.py).
    ``silu_and_mul`` and ``silu_and_mul_nvfp4_quant`` take vLLM's schemas
    (``torch.ops._C.silu_and_mul(out, input)``,
    ``torch.ops._C.silu_and_mul_nvfp4_quant(result, result_block_scale, input,
    input_global_scale)``), so a fusion pass can target them unchanged."""
    fused = "silu_and_mul_scalesweep_mse_nvfp4_quant"
    lib.define(fused + "(Tensor input, Tensor input_scale, bool is_sf_swizzled_layout=True) "
               "-> (Tensor, Tensor)")
    lib.define(fused + ".out(Tensor input, Tensor input_scale, bool is_sf_swizzled_layout=True, "
               "*, Tensor(a!) output, Tensor(b!) output_scale) -> ()")
    lib.define("silu_and_mul(Tensor(a!) out, Tensor input) -> ()")
    lib.define("silu_and_mul_nvfp4_quant(Tensor(a!) result, Tensor(b!) result_block_scale, "
               "Tensor input, Tensor input_global_scale) -> ()")

    def fused_functional(input, input_scale, is_sf_swizzled_layout=True):
        return act_quant.silu_and_mul_scalesweep_mse_nvfp4_quant(input, input_scale,
                                                                 is_sf_swizzled_layout)

    def fused_out(input, input_scale, is_sf_swizzled_layout=True, *, output, output_scale):
        act_quant.silu_and_mul_scalesweep_mse_nvfp4_quant_out(
            input, input_scale, is_sf_swizzled_layout, output=output, output_scale=output_scale)

    def silu_mul(out, input):
        act_quant.silu_and_mul(input, out)

    def fake_fused(input, input_scale, is_sf_swizzled_layout=True):
        return act_quant.alloc_outputs(input, is_sf_swizzled_layout)

    def fake_none(*args, **kwargs):
        return None

    lib.impl(fused, fused_functional, "CUDA")
    lib.impl(fused + ".out", fused_out, "CUDA")
    lib.impl("silu_and_mul", silu_mul, "CUDA")
    lib.impl("silu_and_mul_nvfp4_quant", act_quant.silu_and_mul_nvfp4_quant, "CUDA")
    torch.library.register_fake(f"{namespace}::{fused}", fake_fused, lib=lib)
    torch.library.register_fake(f"{namespace}::{fused}.out", fake_none, lib=lib)
    torch.library.register_fake(f"{namespace}::silu_and_mul", fake_none, lib=lib)
    torch.library.register_fake(f"{namespace}::silu_and_mul_nvfp4_quant", fake_none, lib=lib)


def _register_norm_quant(lib: torch.library.Library, namespace: str) -> None:
    """RMSNorm fused into the scale-sweep quantizer (norm_quant.py).  The
    in-place forms follow vLLM's fused RMSNorm + quant schemas
    (``rms_norm_static_fp8_quant(result, input, weight, scale, epsilon)``,
    ``fused_add_rms_norm_static_fp8_quant(result, input, residual, weight,
    scale, epsilon)``) with the swizzled block-scale tensor after ``result``,
    as in ``silu_and_mul_nvfp4_quant``."""
    fn = "rms_norm_scalesweep_mse_nvfp4_quant"
    lib.define(fn + "(Tensor input, Tensor weight, float epsilon, Tensor input_scale, "
               "bool is_sf_swizzled_layout=True) -> (Tensor, Tensor)")
    lib.define("rms_norm_nvfp4_quant(Tensor(a!) result, Tensor(b!) result_block_scale, "
               "Tensor input, Tensor weight, Tensor input_global_scale, float epsilon) -> ()")
    lib.define("fused_add_rms_norm_nvfp4_quant(Tensor(a!) result, Tensor(b!) result_block_scale, "
               "Tensor input, Tensor(c!) residual, Tensor weight, Tensor input_global_scale, "
               "float epsilon) -> ()")

    def functional(input, weight, epsilon, input_scale, is_sf_swizzled_layout=True):
        return norm_quant.rms_norm_scalesweep_mse_nvfp4_quant(input, weight, epsilon, input_scale,
                                                              is_sf_swizzled_layout)

    def norm_q(result, result_block_scale, input, weight, input_global_scale, epsilon):
        norm_quant.rms_norm_scalesweep_mse_nvfp4_quant_out(
            input, weight, epsilon, input_global_scale, True, output=result,
            output_scale=result_block_scale)

    def add_norm_q(result, result_block_scale, input, residual, weight, input_global_scale,
                   epsilon):
        norm_quant.rms_norm_scalesweep_mse_nvfp4_quant_out(
            input, weight, epsilon, input_global_scale, True, output=result,
            output_scale=result_block_scale, residual=residual)

    def fake_functional(input, weight, epsilon, input_scale, is_sf_swizzled_layout=True):
        return norm_quant.alloc_outputs(input, is_sf_swizzled_layout)

    def fake_none(*args, **kwargs):
        return None

    lib.impl(fn, functional, "CUDA")
    lib.impl("rms_norm_nvfp4_quant", norm_q, "CUDA")
    lib.impl("fused_add_rms_norm_nvfp4_quant", add_norm_q, "CUDA")
    torch.library.register_fake(f"{namespace}::{fn}", fake_functional, lib=lib)
    torch.library.register_fake(f"{namespace}::rms_norm_nvfp4_quant", fake_none, lib=lib)
    torch.library.register_fake(f"{namespace}::fused_add_rms_norm_nvfp4_quant", fake_none, lib=lib)


def register() -> None:
    """Define the ops under ``torch.ops.scalesweep_b200`` (idempotent)."""
    _register(NAMESPACE, "DEF")


def register_vllm_aliases() -> None:
    """Also define them under ``torch.ops.vllm`` (for a vLLM build that expects them)."""
    _register("vllm", "FRAGMENT")


register()
