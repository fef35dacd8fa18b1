"""CPU tests of the NVFP4 checkpoint writer: which weights are quantized and
grouped, the format written, and the argument checks.  The GPU quantizer is
replaced by the oracle here (quantizing itself needs a CUDA device)."""
import json
import os

import numpy as np
import pytest
import torch

import oracle
from test_speed_scalesweep_b200 import checkpoint

NAMES = ["model.embed_tokens.weight", "model.norm.weight", "lm_head.weight",
         "model.layers.0.input_layernorm.weight",
         "model.layers.0.self_attn.q_proj.weight", "model.layers.0.self_attn.k_proj.weight",
         "model.layers.0.self_attn.v_proj.weight", "model.layers.0.self_attn.o_proj.weight",
         "model.layers.0.mlp.gate_proj.weight", "model.layers.0.mlp.up_proj.weight",
         "model.layers.0.mlp.down_proj.weight"]


def test_groups_follow_vllm_fused_layers_and_skip_lm_head():
    groups = checkpoint.fused_groups(NAMES)
    flat = sorted(n for g in groups for n in g)
    assert "lm_head.weight" not in flat and "model.embed_tokens.weight" not in flat
    assert len(flat) == 7
    as_sets = {frozenset(g) for g in groups}
    p = "model.layers.0."
    assert frozenset({p + "self_attn.q_proj.weight", p + "self_attn.k_proj.weight",
                      p + "self_attn.v_proj.weight"}) in as_sets
    assert frozenset({p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight"}) in as_sets
    assert frozenset({p + "mlp.down_proj.weight"}) in as_sets


def test_config_is_compressed_tensors_nvfp4():
    q = checkpoint.quantization_config()
    assert q["quant_method"] == "compressed-tensors" and q["format"] == "nvfp4-pack-quantized"
    assert q["ignore"] == ["lm_head"]
    g = q["config_groups"]["group_0"]
    assert g["weights"]["group_size"] == 16 and g["weights"]["num_bits"] == 4


def _write_tiny(path, h=64, inter=128, vocab=96, seed=0):
    from safetensors.torch import save_file
    g = torch.Generator().manual_seed(seed)
    shapes = {"model.embed_tokens.weight": (vocab, h), "model.norm.weight": (h,),
              "lm_head.weight": (vocab, h), "model.layers.0.input_layernorm.weight": (h,),
              "model.layers.0.self_attn.q_proj.weight": (h, h),
              "model.layers.0.self_attn.k_proj.weight": (h // 2, h),
              "model.layers.0.self_attn.v_proj.weight": (h // 2, h),
              "model.layers.0.self_attn.o_proj.weight": (h, h),
              "model.layers.0.mlp.gate_proj.weight": (inter, h),
              "model.layers.0.mlp.up_proj.weight": (inter, h),
              "model.layers.0.mlp.down_proj.weight": (h, inter)}
    t = {k: (torch.randn(*s, generator=g) * 0.05).to(torch.bfloat16) for k, s in shapes.items()}
    t["model.layers.0.self_attn.k_proj.weight"][3, 5] = 1.5   # k's amax sets q/k/v's scale
    os.makedirs(path, exist_ok=True)
    save_file(t, os.path.join(path, "model.safetensors"))
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump({"model_type": "llama", "hidden_size": h}, f)
    with open(os.path.join(path, "tokenizer.json"), "w") as f:
        f.write("{}")
    return t


def _bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def test_writer_format_with_the_oracle_as_quantizer(tmp_path, monkeypatch):
    """The whole writer with the device kernels swapped for the oracle."""
    src = _write_tiny(str(tmp_path / "src"))

    def absmax(w):
        return torch.tensor([oracle.absmax(_bits(w))], dtype=torch.float32)

    def scale_from_amax(amax, fp8_max):
        return torch.tensor([oracle.global_scale_inv(float(amax.item()), fp8_max)],
                            dtype=torch.float32)

    def quant(w, gsi, swizzled):
        c, s = oracle.quantize(_bits(w), float(gsi.item()), mode="rtn", swizzled=swizzled)
        return torch.from_numpy(c), torch.from_numpy(s).view(torch.float8_e4m3fn)

    monkeypatch.setattr(checkpoint, "_quantizers", lambda wq: (absmax, scale_from_amax, quant))
    monkeypatch.setattr(checkpoint, "activation_scale", lambda amax, device: torch.tensor(
        [oracle.global_scale_inv(amax, 448.0)], dtype=torch.float32))
    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    monkeypatch.setattr(torch.Tensor, "to", lambda self, *a, **k: self if "device" in k
                        else torch.Tensor.__dict__["to"](self, *a, **k), raising=False)
    dst = str(tmp_path / "dst")
    summary = checkpoint.quantize_checkpoint(str(tmp_path / "src"), dst, act_amax=8.0)
    assert summary["quantized_linears"] == 7 and summary["fused_groups"] == 2
    from safetensors import safe_open
    with safe_open(os.path.join(dst, "model.safetensors"), framework="pt") as h:
        out = {k: h.get_tensor(k) for k in h.keys()}
    p = "model.layers.0."
    gs = [out[p + f"self_attn.{m}_proj.weight_global_scale"] for m in "qkv"]
    assert all(torch.equal(g, gs[0]) for g in gs)
    assert gs[0].item() == np.float32(oracle.global_scale_inv(1.5, 448.0))
    assert out[p + "self_attn.q_proj.weight_packed"].shape == (64, 32)
    assert out[p + "self_attn.q_proj.weight_packed"].dtype == torch.uint8
    assert out[p + "mlp.down_proj.weight_scale"].shape == (64, 8)
    assert out[p + "mlp.down_proj.weight_scale"].dtype == torch.float8_e4m3fn
    assert out[p + "mlp.down_proj.input_global_scale"].item() == np.float32(448.0 * 6 / 8.0)
    assert torch.equal(out["lm_head.weight"], src["lm_head.weight"])
    assert p + "self_attn.q_proj.weight" not in out
    cfg = json.load(open(os.path.join(dst, "config.json")))
    assert cfg["quantization_config"]["format"] == "nvfp4-pack-quantized"
    assert os.path.exists(os.path.join(dst, "tokenizer.json"))


def test_writer_refuses_without_a_gpu_and_checks_directories(tmp_path):
    _write_tiny(str(tmp_path / "src"))
    with pytest.raises(FileNotFoundError):
        checkpoint.quantize_checkpoint(str(tmp_path / "none"), str(tmp_path / "d"))
    busy = tmp_path / "busy"
    busy.mkdir()
    (busy / "x").write_text("x")
    with pytest.raises(FileExistsError):
        checkpoint.quantize_checkpoint(str(tmp_path / "src"), str(busy))
    if not torch.cuda.is_available():
        with pytest.raises(ValueError, match="CUDA"):
            checkpoint.quantize_checkpoint(str(tmp_path / "src"), str(tmp_path / "d2"))


def test_calibration_refuses_without_a_gpu(tmp_path):
    if torch.cuda.is_available():
        pytest.skip("checks the no-GPU refusal")
    with pytest.raises(ValueError, match="CUDA"):
        checkpoint.calibrate(str(tmp_path), [[[1, 2, 3]]])


def test_weight_global_scale_follows_the_quantizers_fp8_range(monkeypatch):
    """RTN weights use fp8_max 448; scale-sweep weights 256, the reference's
    convention for scale-sweep backends (headroom for the candidates above
    the base scale)."""
    assert checkpoint.weight_fp8_max("rtn") == 448.0
    assert checkpoint.weight_fp8_max("scalesweep_mse") == 256.0
    with pytest.raises(ValueError):
        checkpoint.weight_fp8_max("cutlass")
    seen = []

    def absmax(w):
        return torch.tensor([oracle.absmax(_bits(w))], dtype=torch.float32)

    def scale_from_amax(amax, fp8_max):
        seen.append(fp8_max)
        return torch.tensor([oracle.global_scale_inv(float(amax.item()), fp8_max)],
                            dtype=torch.float32)

    monkeypatch.setattr(checkpoint, "_quantizers",
                        lambda wq: (absmax, scale_from_amax, lambda w, g, s: (w, g)))
    w = torch.full((16, 32), 2.0, dtype=torch.bfloat16)
    for quantizer, fp8_max in (("rtn", 448.0), ("scalesweep_mse", 256.0)):
        gsi, _ = checkpoint.quantize_group([w], quantizer)
        assert seen[-1] == fp8_max
        assert gsi.item() == np.float32(oracle.global_scale_inv(2.0, fp8_max))


@pytest.mark.parametrize("amax", [0.0, float("inf"), float("nan"), -1.0])
def test_activation_amax_must_give_a_finite_scale(amax):
    with pytest.raises(ValueError, match="activation amax"):
        checkpoint.check_activation_amax("model.layers.0.mlp.down_proj", amax)
    assert checkpoint.check_activation_amax("x", 3.5) == 3.5
