"""The vLLM hooks' routing, without a GPU: with meta tensors this package's
ops run their fake implementations, so the tests check which layers take the
package's path, which fall back to vLLM's, and the shapes that come out."""
import types

import pytest
import torch

vllm_cutlass = pytest.importorskip("vllm.model_executor.kernels.linear.nvfp4.cutlass")
vllm_llama = pytest.importorskip("vllm.model_executor.models.llama")

from test_speed_scalesweep_b200 import vllm_e2e  # noqa: E402


def _layer(n=6144, k=4096, padding=0):
    meta = dict(device="meta")
    return types.SimpleNamespace(
        weight=torch.empty(n, k // 2, dtype=torch.uint8, **meta),
        weight_scale=torch.empty(n, k // 16, dtype=torch.float8_e4m3fn, **meta),
        alpha=torch.empty(1, **meta), input_global_scale_inv=torch.empty(1, **meta),
        output_size_per_partition=n, weights_padding_cols=padding, bias=None, tp_size=1)


def test_linear_hook_routes_supported_layers_and_falls_back(monkeypatch):
    seen = []

    def original(self, layer, x, bias=None):
        seen.append(layer)
        return "vllm"

    monkeypatch.setattr(vllm_cutlass.CutlassNvFp4LinearKernel, "apply_weights", original)
    monkeypatch.setattr(vllm_e2e, "LINEAR_CALLS", {"ours": 0, "fallback": 0})
    vllm_e2e.install_linear_hook()
    apply = vllm_cutlass.CutlassNvFp4LinearKernel.apply_weights
    x = torch.empty(2, 5, 4096, dtype=torch.bfloat16, device="meta")
    out = apply(None, _layer(), x)
    assert out.shape == (2, 5, 6144) and out.dtype == torch.bfloat16
    padded = _layer(padding=8)
    assert apply(None, padded, x) == "vllm" and seen == [padded]
    assert apply(None, _layer(), x.float()) == "vllm"            # not bf16
    assert apply(None, _layer(n=6144 + 32), x) == "vllm"         # N % 64
    assert apply(None, _layer(n=6144 + 64), x).shape == (2, 5, 6144 + 64)  # 64-wide tiles
    assert vllm_e2e.LINEAR_CALLS == {"ours": 2, "fallback": 3}


def test_fused_act_hook_feeds_gate_up_to_the_fused_quantizer(monkeypatch):
    def original(self, x):
        return "vllm"

    monkeypatch.setattr(vllm_llama.LlamaMLP, "forward", original)
    monkeypatch.setattr(vllm_e2e, "MLP_CALLS", {"fused": 0, "fallback": 0})
    calls = {}

    def fake_mm(a, b, sa, sb, alpha, dtype):
        calls["a"], calls["sa"] = a.shape, sa.shape
        return torch.empty(a.shape[0], b.shape[0], dtype=dtype, device="meta")

    import vllm._custom_ops as vllm_ops
    monkeypatch.setattr(vllm_ops, "cutlass_scaled_fp4_mm", fake_mm)
    vllm_e2e.install_fused_act_hook()
    down = _layer(n=4096, k=14336)
    gate_up = torch.empty(7, 2 * 14336, dtype=torch.bfloat16, device="meta")
    mlp = types.SimpleNamespace(gate_up_proj=lambda x: (gate_up, None), down_proj=down)
    out = vllm_llama.LlamaMLP.forward(mlp, torch.empty(7, 4096, device="meta"))
    assert out.shape == (7, 4096)
    assert calls["a"] == (7, 14336 // 2) and calls["sa"] == (128, 14336 // 16)
    down.tp_size = 2                                             # tensor parallel: vLLM's path
    assert vllm_llama.LlamaMLP.forward(mlp, gate_up) == "vllm"
    assert vllm_e2e.MLP_CALLS == {"fused": 1, "fallback": 1}


def test_fused_norm_hook_feeds_each_norm_to_the_next_projections_quantizer(monkeypatch):
    """Layer 0 (no residual yet) takes rms_norm_nvfp4_quant, later layers
    fused_add_rms_norm_nvfp4_quant; each GEMM sees codes of its own input
    width, and the residual comes back."""
    def original(self, positions, hidden_states, residual):
        return "vllm"

    monkeypatch.setattr(vllm_llama.LlamaDecoderLayer, "forward", original)
    monkeypatch.setattr(vllm_e2e, "DECODER_CALLS", {"fused": 0, "fallback": 0})
    mms = []

    def fake_mm(a, b, sa, sb, alpha, dtype):
        mms.append((tuple(a.shape), tuple(sa.shape), b.shape[0]))
        return torch.empty(a.shape[0], b.shape[0], dtype=dtype, device="meta")

    import vllm._custom_ops as vllm_ops
    monkeypatch.setattr(vllm_ops, "cutlass_scaled_fp4_mm", fake_mm)
    vllm_e2e.install_fused_norm_hook()
    meta = dict(device="meta")
    t, h, inter, q, kv = 5, 4096, 14336, 4096, 1024

    def norm():
        return types.SimpleNamespace(weight=torch.empty(h, dtype=torch.bfloat16, **meta),
                                     variance_epsilon=1e-5, variance_size_override=None,
                                     has_weight=True)

    o_out = torch.empty(t, h, dtype=torch.bfloat16, **meta)
    attn = types.SimpleNamespace(qkv_proj=_layer(n=q + 2 * kv, k=h), q_size=q, kv_size=kv,
                                 rotary_emb=lambda pos, a, b: (a, b),
                                 attn=lambda a, b, c: a, o_proj=lambda x: (o_out, None))
    mlp = types.SimpleNamespace(gate_up_proj=_layer(n=2 * inter, k=h), down_proj=_layer(n=h, k=inter))
    layer = types.SimpleNamespace(self_attn=attn, mlp=mlp, input_layernorm=norm(),
                                  post_attention_layernorm=norm())
    x = torch.empty(t, h, dtype=torch.bfloat16, **meta)
    pos = torch.empty(t, dtype=torch.int64, **meta)
    fwd = vllm_llama.LlamaDecoderLayer.forward
    out, res = fwd(layer, pos, x, None)                    # first layer: residual = input
    assert res is x and out.shape == (t, h)
    res2 = torch.empty(t, h, dtype=torch.bfloat16, **meta)
    out, res = fwd(layer, pos, x, res2)
    assert res is res2 and out.shape == (t, h)
    widths = [(a[1], sa, n) for a, sa, n in mms]
    assert widths == [(h // 2, (128, h // 16), q + 2 * kv), (h // 2, (128, h // 16), 2 * inter),
                      (inter // 2, (128, inter // 16), h)] * 2
    mlp.down_proj.tp_size = 2                                # tensor parallel: vLLM's path
    assert fwd(layer, pos, x, res2) == "vllm"
    assert vllm_e2e.DECODER_CALLS == {"fused": 2, "fallback": 1}


def test_gemm_dispatch_rule_and_shapes(monkeypatch):
    vllm_e2e.register_dispatch_ops()
    monkeypatch.setattr(vllm_e2e, "OURS_M_RANGES", {(4096, 28672): ((1, 64), (384, 512))})
    assert vllm_e2e._ours_for(64, 28672, 4096)
    assert not vllm_e2e._ours_for(65, 28672, 4096)       # between the measured ranges
    assert vllm_e2e._ours_for(384, 28672, 4096) and vllm_e2e._ours_for(512, 28672, 4096)
    assert not vllm_e2e._ours_for(513, 28672, 4096)
    assert not vllm_e2e._ours_for(16, 6144, 4096)        # shape not listed: vLLM's GEMM
    monkeypatch.setattr(vllm_e2e, "OURS_M_RANGES", {(4000, 28672): ((1, 64),)})
    assert not vllm_e2e._ours_for(16, 28672, 4000)       # K the GEMM does not take
    meta = dict(device="meta")
    a = torch.empty(16, 2048, dtype=torch.uint8, **meta)
    b = torch.empty(28672, 2048, dtype=torch.uint8, **meta)
    sa = torch.empty(128, 256, dtype=torch.float8_e4m3fn, **meta)
    sb = torch.empty(28672, 256, dtype=torch.float8_e4m3fn, **meta)
    alpha = torch.empty(1, **meta)
    out = torch.ops.scalesweep_b200.nvfp4_mm_dispatch(a, b, sa, sb, alpha)
    assert out.shape == (16, 28672) and out.dtype == torch.bfloat16
    x = torch.empty(16, 4096, dtype=torch.bfloat16, **meta)
    out = torch.ops.scalesweep_b200.scalesweep_nvfp4_linear_dispatch(x, alpha, b, sb, alpha)
    assert out.shape == (16, 28672) and out.dtype == torch.bfloat16


def test_linear_hook_with_dispatch_calls_the_dispatch_op(monkeypatch):
    monkeypatch.setattr(vllm_cutlass.CutlassNvFp4LinearKernel, "apply_weights",
                        lambda self, layer, x, bias=None: "vllm")
    vllm_e2e.install_linear_hook(dispatch=True)
    apply = vllm_cutlass.CutlassNvFp4LinearKernel.apply_weights
    x = torch.empty(3, 4096, dtype=torch.bfloat16, device="meta")
    out = apply(None, _layer(n=4096), x)
    assert out.shape == (3, 4096)


def test_gemm_hook_rebinds_the_module_local_name(monkeypatch):
    import vllm._custom_ops as vllm_ops
    seen = []

    def original(a, b, sa, sb, alpha, out_dtype):
        seen.append(out_dtype)
        return "vllm"

    monkeypatch.setattr(vllm_ops, "cutlass_scaled_fp4_mm", original)
    monkeypatch.setattr(vllm_cutlass, "cutlass_scaled_fp4_mm", original)
    assert vllm_e2e.install_gemm_hook() >= 1
    hooked = vllm_cutlass.cutlass_scaled_fp4_mm
    assert hooked is not original
    # vLLM's own module keeps its GEMM, which the dispatch op calls for the
    # token counts it leaves to vLLM (rebinding it would recurse)
    assert vllm_ops.cutlass_scaled_fp4_mm is original
    meta = dict(device="meta")
    a = torch.empty(16, 2048, dtype=torch.uint8, **meta)
    b = torch.empty(4096, 2048, dtype=torch.uint8, **meta)
    sa = torch.empty(128, 256, dtype=torch.float8_e4m3fn, **meta)
    sb = torch.empty(4096, 256, dtype=torch.float8_e4m3fn, **meta)
    alpha = torch.empty(1, **meta)
    out = hooked(a, b, sa, sb, alpha, torch.bfloat16)     # through the dispatch op
    assert out.shape == (16, 4096) and out.dtype == torch.bfloat16
    assert hooked(a, b, sa, sb, alpha, torch.float16) == "vllm" and seen == [torch.float16]
