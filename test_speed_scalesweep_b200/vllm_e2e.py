"""vLLM integration: the scale-sweep quantizer as vLLM's NVFP4 activation
quantizer, plus the end-to-end Llama-3.1-8B W4A4 throughput benchmark.

The reference runs its quantizers inside an unpublished vLLM fork that takes
an ``act_quant_backend`` argument (``run_bench_tune.sh:24,31``,
``benchmark_nvfp4_tokens.py:117-118``).  Stock vLLM has no such argument.  Its
W4A4 linear layer (``CutlassNvFp4LinearKernel.apply_weights``, vLLM 0.22
``model_executor/kernels/linear/nvfp4/cutlass.py:45-77``) calls the
module-local name ``scaled_fp4_quant``.  ``install_act_quant_hook`` rebinds
that name, the same monkey-patch pattern the reference applies to the same
module in ``benchmark_nvfp4_tokens.py:191-211``.  The replacement calls this
package's registered torch op, so it traces under torch.compile (fake
implementation) and runs inside vLLM's CUDA graphs.

The benchmark mirrors ``benchmark_nvfp4_tokens.py``:
- synthetic prompts of uniform-random token ids, with ``ignore_eos``;
- a fixed number of output tokens;
- output tok/s.

It uses the Llama-3.1-8B architecture with random N(0, 0.02) weights,
RTN-quantized to NVFP4 in-process, because there is no checkpoint.

    python -m test_speed_scalesweep_b200.vllm_e2e --backend scalesweep_mse \
        --batch-sizes 1 16 64 256 --input-len 1024 --output-len 256
"""
from __future__ import annotations

import argparse
import json
import os
import tempfile
import time

import torch

# Llama-3.1-8B architecture hyper-parameters (public model card values).
LLAMA31_8B = {
    "architectures": ["LlamaForCausalLM"],
    "model_type": "llama",
    "hidden_size": 4096,
    "intermediate_size": 14336,
    "num_hidden_layers": 32,
    "num_attention_heads": 32,
    "num_key_value_heads": 8,
    "head_dim": 128,
    "vocab_size": 128256,
    "max_position_embeddings": 131072,
    "rms_norm_eps": 1e-05,
    "rope_theta": 500000.0,
    "rope_scaling": {"factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                     "original_max_position_embeddings": 8192, "rope_type": "llama3"},
    "hidden_act": "silu",
    "attention_bias": False,
    "mlp_bias": False,
    "tie_word_embeddings": False,
    "torch_dtype": "bfloat16",
    "bos_token_id": 128000,
    "eos_token_id": 128009,
}

# compressed-tensors NVFP4 W4A4: 16-element float4 groups with per-tensor
# global scales for weights and activations, lm_head left in bf16
# (quant_model_nvfp4.py:65-87 produces this scheme with llmcompressor).
_FP4_ARGS = {"num_bits": 4, "type": "float", "strategy": "tensor_group", "group_size": 16,
             "symmetric": True, "dynamic": False, "observer": "minmax"}
NVFP4_QUANT_CONFIG = {
    "quant_method": "compressed-tensors",
    "format": "nvfp4-pack-quantized",
    "quantization_status": "compressed",
    "ignore": ["lm_head"],
    "config_groups": {
        "group_0": {
            "targets": ["Linear"],
            "format": "nvfp4-pack-quantized",
            "weights": dict(_FP4_ARGS),
            "input_activations": dict(_FP4_ARGS, dynamic="local"),
        }
    },
}

# "scalesweep_mse_linear": the whole W4A4 linear layer from this package --
# scale-sweep quantization and this package's NVFP4 GEMM in one op
# (install_linear_hook); the others swap only the activation quantizer.
# "scalesweep_mse_fused_act": additionally, each MLP's SiLU-and-mul and the
# down projection's activation quantizer run as one fused kernel
# (install_fused_act_hook), with vLLM's GEMM.
# "scalesweep_mse_fused_norm_act": also each decoder layer's two RMSNorms are
# fused into the qkv and gate_up projections' quantizers
# (install_fused_norm_hook).
# "scalesweep_mse_fusion_pass": the same fusions as scalesweep_mse_fused_norm_act,
# reached through vLLM's compile passes instead of module hooks
# (vllm_fusion.install_fusion_pass), so they apply to any model's graph.
# "..._dispatch": as without the suffix, but each GEMM (with its quantizer,
# where the hook issues both) is this package's where it is faster than vLLM's
# at the call's token count (OURS_M_RANGES), vLLM's elsewhere.  With the
# compile pass, only the GEMM is dispatched (install_gemm_hook), so the
# quantizer stays visible to the pass.
BACKENDS = ("scalesweep_mse", "scalesweep_mse_reference", "rtn", "cutlass",
            "scalesweep_mse_linear", "scalesweep_mse_fused_act",
            "scalesweep_mse_fused_norm_act", "scalesweep_mse_fusion_pass",
            "scalesweep_mse_dispatch", "scalesweep_mse_fused_norm_act_dispatch",
            "scalesweep_mse_fusion_pass_dispatch")
_OP_FOR_BACKEND = {"scalesweep_mse": "scalesweep_mse_nvfp4_quant",
                   "scalesweep_mse_reference": "scalesweep_mse_reference_nvfp4_quant",
                   "rtn": "rtn_nvfp4_quant"}


def write_model_dir(path: str) -> str:
    """A model directory holding only config.json (weights come from the dummy loader)."""
    os.makedirs(path, exist_ok=True)
    cfg = dict(LLAMA31_8B, quantization_config=NVFP4_QUANT_CONFIG)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    return path


HOOK_CALLS = {"count": 0}


def install_act_quant_hook(backend: str, op=None) -> int:
    """Route vLLM's W4A4 activation quantization through this package's kernels.

    Every vLLM module that imported ``scaled_fp4_quant`` by name (the CUTLASS
    and FlashInfer NVFP4 linear kernels among them) gets the replacement, so
    the hook holds whichever linear backend vLLM picks.  ``backend="cutlass"``
    leaves vLLM's own quantizer in place (the baseline).  ``op``, when given,
    replaces this package's op: any registered op with the signature
    ``op(x2d, input_global_scale, is_sf_swizzled_layout, padded_n) ->
    (codes, scales)``, such as another implementation of the same quantizer
    timed under the same hook.  Returns the number of module-level names
    rebound.
    """
    if backend == "cutlass" and op is None:
        return 0
    import importlib
    import sys

    from . import ops  # noqa: F401  (registers torch.ops.scalesweep_b200.*)
    import vllm._custom_ops as vllm_ops

    for mod_name in ("vllm.model_executor.kernels.linear.nvfp4.cutlass",
                     "vllm.model_executor.kernels.linear.nvfp4.flashinfer"):
        try:
            importlib.import_module(mod_name)
        except Exception:  # pragma: no cover - depends on the vLLM build
            pass
    original = vllm_ops.scaled_fp4_quant
    if op is None:
        op = getattr(torch.ops.scalesweep_b200, _OP_FOR_BACKEND[backend])

    def scaled_fp4_quant(input, input_global_scale, is_sf_swizzled_layout=True,
                         backend="none", padded_n=None):
        HOOK_CALLS["count"] += 1
        # no view node for the usual 2-D input, so a fusion pass sees the
        # producer feed the quantizer directly
        x = input if input.dim() == 2 else input.reshape(-1, input.shape[-1])
        if padded_n is not None and padded_n == x.shape[-1]:
            padded_n = None
        return op(x, input_global_scale, is_sf_swizzled_layout, padded_n)

    rebound = 0
    for name, mod in list(sys.modules.items()):
        if name.startswith("vllm") and getattr(mod, "scaled_fp4_quant", None) is original:
            setattr(mod, "scaled_fp4_quant", scaled_fp4_quant)
            rebound += 1
    return rebound


GEMM_HOOK_CALLS = {"count": 0}


def install_gemm_hook() -> int:
    """Route the GEMM of vLLM's W4A4 linear layer through
    ``scalesweep_b200::nvfp4_mm_dispatch`` (this package's GEMM where it is
    faster at the call's token count, vLLM's elsewhere) and leave the rest of
    ``CutlassNvFp4LinearKernel.apply_weights`` as it is.

    ``apply_weights`` calls the module-local name ``cutlass_scaled_fp4_mm``
    (vllm 0.22 ``model_executor/kernels/linear/nvfp4/cutlass.py:64-71``); this
    rebinds it, the pattern the reference applies to the same name in
    ``benchmark_nvfp4_tokens.py:195``.  The activation quantizer stays a
    separate op in the graph, so ``vllm_fusion``'s pass can still fuse its
    producer into it.  bf16 outputs only; others keep vLLM's GEMM.  Returns
    the number of module-level names rebound."""
    import importlib
    import sys

    import vllm._custom_ops as vllm_ops

    register_dispatch_ops()
    for mod_name in ("vllm.model_executor.kernels.linear.nvfp4.cutlass",):
        try:
            importlib.import_module(mod_name)
        except Exception:  # pragma: no cover - depends on the vLLM build
            pass
    original = vllm_ops.cutlass_scaled_fp4_mm

    def cutlass_scaled_fp4_mm(a, b, block_scale_a, block_scale_b, alpha, out_dtype):
        GEMM_HOOK_CALLS["count"] += 1
        if out_dtype != torch.bfloat16:
            return original(a, b, block_scale_a, block_scale_b, alpha, out_dtype)
        return torch.ops.scalesweep_b200.nvfp4_mm_dispatch(a, b, block_scale_a, block_scale_b,
                                                           alpha)

    # the callers' module-local names only: vllm._custom_ops keeps its own
    rebound = 0
    for name, mod in list(sys.modules.items()):
        if (name.startswith("vllm") and name != "vllm._custom_ops"
                and getattr(mod, "cutlass_scaled_fp4_mm", None) is original):
            setattr(mod, "cutlass_scaled_fp4_mm", cutlass_scaled_fp4_mm)
            rebound += 1
    return rebound


LINEAR_CALLS = {"ours": 0, "fallback": 0}

# Token-count ranges (inclusive) in which this package's GEMM (with the
# quantizer as its programmatic dependent launch, for the whole linear layer)
# beats scale-sweep quantization followed by vLLM's CUTLASS NVFP4 GEMM, per
# Llama-3.1-8B shape (K, N); measured on B200 with
# ``python bench.py --gemm-crossover`` (vLLM time / this package's, one CUDA
# graph of 20 launches):
#   qkv     (4096, 6144):  1.05-1.32 up to M=64, 0.67-0.99 above;
#   o       (4096, 4096):  1.09-1.35 up to M=64, 0.91-0.96 from 96 to 512;
#   gate_up (4096, 28672): 1.19-2.05 up to M=128, 0.85-0.88 at 192-256,
#                          1.06 at 384-512, 0.87-1.01 from 1024;
#   down    (14336, 4096): 1.02-1.69 up to M=128, 0.94-0.96 at 192-256,
#                          1.11-1.15 at 384-1024, 0.99-1.02 from 2048.
# Other shapes and token counts use vLLM's GEMM.
OURS_M_RANGES = {(4096, 6144): ((1, 64),), (4096, 4096): ((1, 64),),
                 (4096, 28672): ((1, 128), (384, 512)),
                 (14336, 4096): ((1, 128), (384, 1024))}
GEMM_DISPATCH = {"on": False, "ours": 0, "vllm": 0}


def _ours_for(m: int, n: int, k: int) -> bool:
    return (k % 256 == 0 and n % 64 == 0 and
            any(lo <= m <= hi for lo, hi in OURS_M_RANGES.get((k, n), ())))


_DISPATCH_LIB = None


def register_dispatch_ops() -> None:
    """``scalesweep_b200::nvfp4_mm_dispatch`` and
    ``scalesweep_b200::scalesweep_nvfp4_linear_dispatch``: the GEMM, or the
    whole W4A4 linear layer, from this package where it is faster
    (``OURS_M_RANGES``) and from vLLM's CUTLASS kernel elsewhere.  The choice
    is made at run time from the actual token count, inside an op that
    torch.compile treats as opaque, so one compiled graph serves every M.
    Idempotent."""
    global _DISPATCH_LIB
    if _DISPATCH_LIB is not None:
        return
    import vllm._custom_ops as vllm_ops

    from . import ops  # noqa: F401  (registers torch.ops.scalesweep_b200.*)
    from .gemm import cutlass_scaled_fp4_mm, scalesweep_nvfp4_linear
    from .scalesweep_mse_nvfp4_utils import scalesweep_mse_nvfp4_quant_impl

    # vLLM's own GEMM, bound now: the GEMM hook may later rebind the name
    # in vLLM's modules to a function that calls back into this op
    vllm_mm = vllm_ops.cutlass_scaled_fp4_mm
    lib = torch.library.Library("scalesweep_b200", "FRAGMENT")
    lib.define("nvfp4_mm_dispatch(Tensor a, Tensor b, Tensor a_scale, Tensor b_scale, "
               "Tensor alpha) -> Tensor")
    lib.define("scalesweep_nvfp4_linear_dispatch(Tensor x, Tensor input_scale, Tensor weight, "
               "Tensor weight_scale, Tensor alpha) -> Tensor")

    def mm(a, b, a_scale, b_scale, alpha):
        m, n, k = a.shape[0], b.shape[0], a.shape[1] * 2
        if _ours_for(m, n, k):
            GEMM_DISPATCH["ours"] += 1
            # the codes come from the quantizer launched just before: start
            # the prologue and weight loads while it finishes
            return cutlass_scaled_fp4_mm(a, b, a_scale, b_scale, alpha, dependent_launch=True)
        GEMM_DISPATCH["vllm"] += 1
        return vllm_mm(a, b, a_scale, b_scale, alpha, torch.bfloat16)

    def linear(x, input_scale, weight, weight_scale, alpha):
        m, k, n = x.shape[0], x.shape[1], weight.shape[0]
        if _ours_for(m, n, k) and x.dtype == torch.bfloat16:
            GEMM_DISPATCH["ours"] += 1
            return scalesweep_nvfp4_linear(x, input_scale, weight, weight_scale, alpha)
        GEMM_DISPATCH["vllm"] += 1
        codes, scales = scalesweep_mse_nvfp4_quant_impl(x, input_scale, True)
        return vllm_mm(codes, weight, scales, weight_scale, alpha, x.dtype)

    def fake_mm(a, b, a_scale, b_scale, alpha):
        return a.new_empty((a.shape[0], b.shape[0]), dtype=torch.bfloat16)

    def fake_linear(x, input_scale, weight, weight_scale, alpha):
        return x.new_empty((x.shape[0], weight.shape[0]))

    lib.impl("nvfp4_mm_dispatch", mm, "CUDA")
    lib.impl("scalesweep_nvfp4_linear_dispatch", linear, "CUDA")
    torch.library.register_fake("scalesweep_b200::nvfp4_mm_dispatch", fake_mm, lib=lib)
    torch.library.register_fake("scalesweep_b200::scalesweep_nvfp4_linear_dispatch", fake_linear,
                                lib=lib)
    _DISPATCH_LIB = lib


def install_linear_hook(dispatch: bool = False) -> None:
    """Route vLLM's W4A4 linear layer through ``scalesweep_nvfp4_linear``
    (with ``dispatch``: through ``scalesweep_nvfp4_linear_dispatch``, which
    keeps vLLM's GEMM where it is the faster one).

    ``CutlassNvFp4LinearKernel.apply_weights`` (vllm 0.22
    ``model_executor/kernels/linear/nvfp4/cutlass.py:45-77``) calls
    ``scaled_fp4_quant`` and then ``cutlass_scaled_fp4_mm``.  The replacement
    makes one call of the registered op
    ``torch.ops.scalesweep_b200.scalesweep_nvfp4_linear``: this package's
    quantizer, then its GEMM as a programmatic dependent launch.  Layers the
    GEMM does not take (K-padded weights, K % 256, N % 64, non-bf16
    activations) keep vLLM's method.
    """
    from . import ops  # noqa: F401  (registers torch.ops.scalesweep_b200.*)
    from vllm.model_executor.kernels.linear.nvfp4.cutlass import CutlassNvFp4LinearKernel

    original = CutlassNvFp4LinearKernel.apply_weights
    if getattr(original, "_scalesweep_b200", False):
        return
    if dispatch:
        register_dispatch_ops()
    linear_op = (torch.ops.scalesweep_b200.scalesweep_nvfp4_linear_dispatch if dispatch
                 else torch.ops.scalesweep_b200.scalesweep_nvfp4_linear)

    def apply_weights(self, layer, x, bias=None):
        k = x.shape[-1]
        n = layer.weight.shape[0]
        if (getattr(layer, "weights_padding_cols", 0) or k % 256 or n % 64
                or x.dtype != torch.bfloat16):
            LINEAR_CALLS["fallback"] += 1
            return original(self, layer, x, bias)
        LINEAR_CALLS["ours"] += 1
        out = linear_op(x.reshape(-1, k), layer.input_global_scale_inv, layer.weight,
                        layer.weight_scale, layer.alpha)
        output_size = layer.output_size_per_partition
        if n != output_size:
            out = out[:, :output_size]
        if bias is not None:
            out = out + bias
        return out.view(*x.shape[:-1], output_size)

    apply_weights._scalesweep_b200 = True
    CutlassNvFp4LinearKernel.apply_weights = apply_weights


MLP_CALLS = {"fused": 0, "fallback": 0}


def install_fused_act_hook() -> None:
    """Fuse each Llama MLP's SiLU-and-mul into the down projection's
    activation quantizer.

    ``LlamaMLP.forward`` (vllm 0.22 ``model_executor/models/llama.py:117-121``)
    runs gate_up_proj, ``SiluAndMul`` and down_proj; down_proj quantizes the
    bf16 ``silu(gate) * up`` it is given.  The replacement hands gate_up_proj's
    output straight to ``silu_and_mul_scalesweep_mse_nvfp4_quant`` with
    down_proj's activation global scale, then runs vLLM's
    ``cutlass_scaled_fp4_mm`` with down_proj's weights: the role vLLM's
    ``fuse_act_quant`` pass plays for its own quantizer.  Layers that are not
    single-GPU NVFP4 W4A4 linears without weight padding keep the original
    forward.
    """
    from . import ops  # noqa: F401  (registers torch.ops.scalesweep_b200.*)
    from vllm.model_executor.models.llama import LlamaMLP

    original = LlamaMLP.forward
    if getattr(original, "_scalesweep_b200", False):
        return

    def forward(self, x):
        if not _single_gpu_w4a4(self.down_proj):
            MLP_CALLS["fallback"] += 1
            return original(self, x)
        MLP_CALLS["fused"] += 1
        gate_up, _ = self.gate_up_proj(x)
        return _silu_mul_down(self.down_proj, gate_up)

    forward._scalesweep_b200 = True
    LlamaMLP.forward = forward


def _single_gpu_w4a4(lin) -> bool:
    """A vLLM NVFP4 W4A4 linear layer without tensor parallelism or weight
    padding: the layers whose quantize + GEMM the hooks can issue themselves."""
    return (getattr(lin, "tp_size", 1) == 1 and not getattr(lin, "weights_padding_cols", 0)
            and all(hasattr(lin, a) for a in ("input_global_scale_inv", "weight_scale", "alpha"))
            and lin.weight.dtype == torch.uint8)


def _fp4_linear(lin, codes, scales, lead_shape, dtype):
    """vLLM's CUTLASS NVFP4 GEMM on already-quantized activations, as
    ``CutlassNvFp4LinearKernel.apply_weights`` runs it after quantizing
    (vllm 0.22 ``model_executor/kernels/linear/nvfp4/cutlass.py:64-77``)."""
    import vllm._custom_ops as vllm_ops
    if GEMM_DISPATCH["on"] and dtype == torch.bfloat16:
        out = torch.ops.scalesweep_b200.nvfp4_mm_dispatch(codes, lin.weight, scales,
                                                          lin.weight_scale, lin.alpha)
    else:
        out = vllm_ops.cutlass_scaled_fp4_mm(codes, lin.weight, scales, lin.weight_scale,
                                             lin.alpha, dtype)
    out = out[:, :lin.output_size_per_partition]
    if lin.bias is not None:
        out = out + lin.bias
    return out.view(*lead_shape, lin.output_size_per_partition)


def _silu_mul_down(down, gate_up):
    """down_proj(silu_and_mul(gate_up)) with the SiLU-and-mul fused into the
    down projection's scale-sweep quantizer."""
    codes, scales = torch.ops.scalesweep_b200.silu_and_mul_scalesweep_mse_nvfp4_quant(
        gate_up.reshape(-1, gate_up.shape[-1]), down.input_global_scale_inv, True)
    return _fp4_linear(down, codes, scales, gate_up.shape[:-1], gate_up.dtype)


DECODER_CALLS = {"fused": 0, "fallback": 0}


def install_fused_norm_hook() -> None:
    """Fuse each Llama decoder layer's RMSNorms into the next projection's
    activation quantizer, and its SiLU-and-mul into the down projection's.

    ``LlamaDecoderLayer.forward`` (vllm 0.22 ``model_executor/models/llama.py:316-333``)
    runs input_layernorm, attention (qkv_proj, rotary, attention, o_proj:
    ``:223-233``), post_attention_layernorm and the MLP.  The replacement
    hands each norm's input (and the residual) to ``rms_norm_nvfp4_quant`` /
    ``fused_add_rms_norm_nvfp4_quant`` with the qkv or gate_up projection's
    activation global scale, then runs vLLM's GEMM on the codes: the role
    vLLM's ``fuse_norm_quant`` pass plays for its FP8 quantizers.  The
    residual is updated in place, as ``fused_add_rms_norm`` updates it.

    The normalised values are those of vLLM's ``vllm_c`` RMSNorm kernels.
    Under Inductor vLLM runs its native RMSNorm, compiled by Inductor, whose
    reduction order may differ in the last bits.  Layers whose projections
    are not single-GPU NVFP4 W4A4 linears keep the original forward.
    """
    from . import ops  # noqa: F401  (registers torch.ops.scalesweep_b200.*)
    from vllm.model_executor.models.llama import LlamaDecoderLayer

    original = LlamaDecoderLayer.forward
    if getattr(original, "_scalesweep_b200", False):
        return

    def norm_quant(norm, lin, x2, residual2):
        m, n = x2.shape
        codes = x2.new_empty((m, n // 2), dtype=torch.uint8)
        scales = x2.new_empty(((m + 127) // 128 * 128, (n // 16 + 3) // 4 * 4),
                              dtype=torch.float8_e4m3fn)
        if residual2 is None:
            torch.ops.scalesweep_b200.rms_norm_nvfp4_quant(
                codes, scales, x2, norm.weight, lin.input_global_scale_inv,
                norm.variance_epsilon)
        else:
            torch.ops.scalesweep_b200.fused_add_rms_norm_nvfp4_quant(
                codes, scales, x2, residual2, norm.weight, lin.input_global_scale_inv,
                norm.variance_epsilon)
        return codes, scales

    def plain_norm(norm) -> bool:
        return (getattr(norm, "variance_size_override", None) is None
                and getattr(norm, "has_weight", True) and norm.weight.dtype == torch.bfloat16)

    def forward(self, positions, hidden_states, residual):
        attn, mlp = self.self_attn, self.mlp
        if not (hidden_states.dtype == torch.bfloat16 and _single_gpu_w4a4(attn.qkv_proj)
                and _single_gpu_w4a4(mlp.gate_up_proj) and _single_gpu_w4a4(mlp.down_proj)
                and plain_norm(self.input_layernorm)
                and plain_norm(self.post_attention_layernorm)):
            DECODER_CALLS["fallback"] += 1
            return original(self, positions, hidden_states, residual)
        DECODER_CALLS["fused"] += 1
        lead, hidden = hidden_states.shape[:-1], hidden_states.shape[-1]
        x2 = hidden_states.reshape(-1, hidden)
        if residual is None:
            residual = hidden_states
            codes, scales = norm_quant(self.input_layernorm, attn.qkv_proj, x2, None)
        else:
            codes, scales = norm_quant(self.input_layernorm, attn.qkv_proj, x2,
                                       residual.view(-1, hidden))
        qkv = _fp4_linear(attn.qkv_proj, codes, scales, lead, hidden_states.dtype)
        q, k, v = qkv.split([attn.q_size, attn.kv_size, attn.kv_size], dim=-1)
        q, k = attn.rotary_emb(positions, q, k)
        attn_out, _ = attn.o_proj(attn.attn(q, k, v))
        codes, scales = norm_quant(self.post_attention_layernorm, mlp.gate_up_proj,
                                   attn_out.reshape(-1, hidden), residual.view(-1, hidden))
        gate_up = _fp4_linear(mlp.gate_up_proj, codes, scales, lead, hidden_states.dtype)
        return _silu_mul_down(mlp.down_proj, gate_up), residual

    forward._scalesweep_b200 = True
    LlamaDecoderLayer.forward = forward


def init_random_nvfp4_weights(model: torch.nn.Module, act_amax: float = 16.0,
                              seed: int = 0) -> int:
    """Give every W4A4 linear layer seeded N(0, 0.02) weights, RTN-quantized to
    NVFP4 by this package's RTN kernel, and a static activation global scale
    ``2688 / act_amax``.  Writes in place, so tensors captured by CUDA graphs
    stay valid.  Returns the number of layers initialised."""
    from . import global_scale
    from .scalesweep_mse_nvfp4_utils import rtn_nvfp4_quant_impl

    gen = torch.Generator(device="cuda").manual_seed(seed)
    act_gsi = 448.0 * 6.0 / act_amax
    count = 0
    for mod in model.modules():
        if not (hasattr(mod, "weight_scale") and hasattr(mod, "alpha")
                and hasattr(mod, "input_global_scale_inv")):
            continue
        n = mod.output_size_per_partition
        k = mod.input_size_per_partition
        w = torch.empty(n, k, device="cuda", dtype=torch.float32).normal_(0.0, 0.02,
                                                                          generator=gen)
        w = w.to(torch.bfloat16)
        w_gsi = global_scale.global_scale_inv_from_max(w, 448.0)
        codes, scales = rtn_nvfp4_quant_impl(w, w_gsi, True)
        mod.weight.data.zero_()
        mod.weight.data[:, : k // 2].copy_(codes)
        sc = mod.weight_scale.data
        sc.view(torch.uint8).zero_()
        sc.view(torch.uint8)[: scales.shape[0], : scales.shape[1]].copy_(scales.view(torch.uint8))
        mod.input_global_scale_inv.data.fill_(act_gsi)
        mod.alpha.data.copy_((1.0 / (act_gsi * w_gsi)).reshape(mod.alpha.shape))
        count += 1
    torch.cuda.synchronize()
    return count


def run(backend: str, batch_sizes, input_len: int, output_len: int, seed: int = 0,
        gpu_memory_utilization: float = 0.85, enforce_eager: bool = False,
        quant_op=None) -> dict:
    """One vLLM engine, one backend: output tok/s for each batch size.

    ``quant_op`` (with ``backend="cutlass"``) installs another registered
    activation quantizer under the same hook, so two implementations of the
    quantizer are timed through the same integration."""
    os.environ.setdefault("VLLM_ENABLE_V1_MULTIPROCESSING", "0")
    dispatch = backend.endswith("_dispatch")
    if dispatch:
        backend = backend[: -len("_dispatch")]
    linear_ours = backend == "scalesweep_mse_linear"
    fused_norm = backend == "scalesweep_mse_fused_norm_act"
    fused_act = backend == "scalesweep_mse_fused_act" or fused_norm
    fusion_pass = backend == "scalesweep_mse_fusion_pass"
    rebound = install_act_quant_hook(
        "scalesweep_mse" if (linear_ours or fused_act or fusion_pass) else backend, op=quant_op)
    if dispatch:
        register_dispatch_ops()
        GEMM_DISPATCH["on"] = True
        if fusion_pass:
            # keep the quantizer visible to the pass; dispatch the GEMM alone
            install_gemm_hook()
        else:
            install_linear_hook(dispatch=True)
    if fusion_pass:
        from . import vllm_fusion
        vllm_fusion.install_fusion_pass()
    if linear_ours:
        install_linear_hook()
    if fused_act:
        install_fused_act_hook()
    if fused_norm:
        install_fused_norm_hook()
    from vllm import LLM, SamplingParams
    from vllm.inputs import TokensPrompt

    model_dir = write_model_dir(tempfile.mkdtemp(prefix="llama31_8b_nvfp4_"))
    max_bs = max(batch_sizes)
    llm = LLM(model=model_dir, skip_tokenizer_init=True, load_format="dummy",
              dtype="bfloat16", max_model_len=input_len + output_len + 16,
              max_num_seqs=max_bs, max_num_batched_tokens=max(8192, input_len),
              gpu_memory_utilization=gpu_memory_utilization, enforce_eager=enforce_eager,
              seed=seed,
              # the CUTLASS W4A4 linear kernel for every backend, and no
              # norm/activation-quant fusion, so the activation quantizer under
              # test is the one that runs (as in the reference's runs,
              # run_bench_tune.sh:24,31)
              kernel_config={"linear_backend": "cutlass"},
              compilation_config={"pass_config": {"fuse_act_quant": False,
                                                  "fuse_norm_quant": False}})
    n_layers = llm.apply_model(lambda m: init_random_nvfp4_weights(m, seed=seed))
    gen = torch.Generator().manual_seed(seed)
    params = SamplingParams(max_tokens=output_len, ignore_eos=True, temperature=1.0,
                            detokenize=False, seed=seed)
    results = {"backend": backend + ("_dispatch" if dispatch else ""),
               "input_len": input_len, "output_len": output_len,
               "quantized_layers": n_layers, "hook_rebound_names": rebound, "batch": {},
               "linear_backend": ("scalesweep_b200 quantizer + GEMM (one op)" if linear_ours
                                  else "vLLM CUTLASS"), "fusion": "off",
               "weights": "random N(0, 0.02), RTN-quantized to NVFP4 in-process",
               "prompts": "uniform-random token ids, ignore_eos"}
    warm = [TokensPrompt(prompt_token_ids=torch.randint(0, 128000, (input_len,),
                                                        generator=gen).tolist())
            for _ in range(min(16, max_bs))]
    llm.generate(warm, params, use_tqdm=False)
    for bs in batch_sizes:
        prompts = [TokensPrompt(prompt_token_ids=torch.randint(0, 128000, (input_len,),
                                                               generator=gen).tolist())
                   for _ in range(bs)]
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        outs = llm.generate(prompts, params, use_tqdm=False)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        n_out = sum(len(o.outputs[0].token_ids) for o in outs)
        results["batch"][str(bs)] = {
            "output_tok_s": round(n_out / dt, 2),
            "total_tok_s": round((n_out + bs * input_len) / dt, 2),
            "seconds": round(dt, 3), "output_tokens": n_out}
    results["hook_calls_during_compile_and_capture"] = HOOK_CALLS["count"]
    if linear_ours:
        results["linear_hook_calls"] = dict(LINEAR_CALLS)
    if fused_act:
        results["mlp_hook_calls"] = dict(MLP_CALLS)
        results["fusion"] = "SiLU-and-mul + scale-sweep quant fused (this package)"
    if dispatch:
        results["gemm_dispatch_calls"] = {"ours": GEMM_DISPATCH["ours"],
                                          "vllm": GEMM_DISPATCH["vllm"]}
        if fusion_pass:
            results["gemm_hook_calls"] = dict(GEMM_HOOK_CALLS)
        results["linear_backend"] = ("this package's GEMM in the OURS_M_RANGES token counts, "
                                     "vLLM CUTLASS elsewhere")
    if fusion_pass:
        results["fusion_pass_matches"] = dict(vllm_fusion.MATCHES)
        results["fusion"] = ("RMSNorm / fused-add RMSNorm / SiLU-and-mul + scale-sweep quant "
                             "fused by a vLLM compile pass (this package)")
    if fused_norm or fusion_pass:
        results["numerics"] = (
            "the fused RMSNorm equals vLLM's vllm_c rms_norm / fused_add_rms_norm kernels bit "
            "for bit; under Inductor vLLM runs a generated native RMSNorm instead, so the "
            "normalised values (and then codes) can differ from an unfused compiled run in the "
            "last bits; in eager mode both generate the same tokens")
    if fused_norm:
        results["decoder_hook_calls"] = dict(DECODER_CALLS)
        results["fusion"] = ("RMSNorm + scale-sweep quant (qkv, gate_up) and SiLU-and-mul + "
                             "scale-sweep quant (down) fused (this package)")
    return results


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--backend", choices=BACKENDS, default="scalesweep_mse")
    ap.add_argument("--batch-sizes", type=int, nargs="+", default=[1, 16, 64, 256])
    ap.add_argument("--input-len", type=int, default=1024)
    ap.add_argument("--output-len", type=int, default=256)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--enforce-eager", action="store_true")
    ap.add_argument("--out", default=None)
    args = ap.parse_args()
    res = run(args.backend, args.batch_sizes, args.input_len, args.output_len, args.seed,
              enforce_eager=args.enforce_eager)
    line = json.dumps(res)
    print(line, flush=True)
    if args.out:
        with open(args.out, "w") as f:
            f.write(line + "\n")


if __name__ == "__main__":
    main()
