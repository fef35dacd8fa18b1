"""GPU test of the NVFP4 checkpoint writer: a tiny Llama is written to
safetensors, converted on the device, compared with the oracle's RTN codes
and scales, and loaded by vLLM (in a subprocess) to check that vLLM reads
the codes and global scales as written and generates from them.  It starts
a vLLM engine and a transformers model, so it is named to run after the
kernel parity files."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

TINY = dict(architectures=["LlamaForCausalLM"], model_type="llama", hidden_size=256,
            intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
            num_key_value_heads=2, head_dim=64, vocab_size=512, max_position_embeddings=512,
            rms_norm_eps=1e-5, rope_theta=10000.0, hidden_act="silu", attention_bias=False,
            mlp_bias=False, tie_word_embeddings=False, torch_dtype="bfloat16")


def _tiny_checkpoint(path, seed=0):
    from safetensors.torch import save_file
    c = TINY
    h, i, v = c["hidden_size"], c["intermediate_size"], c["vocab_size"]
    q, kv = c["num_attention_heads"] * c["head_dim"], c["num_key_value_heads"] * c["head_dim"]
    g = torch.Generator().manual_seed(seed)
    t = {"model.embed_tokens.weight": torch.randn(v, h, generator=g),
         "model.norm.weight": torch.ones(h), "lm_head.weight": torch.randn(v, h, generator=g)}
    for layer in range(c["num_hidden_layers"]):
        p = f"model.layers.{layer}."
        t[p + "input_layernorm.weight"] = torch.ones(h)
        t[p + "post_attention_layernorm.weight"] = torch.ones(h)
        for name, shape in (("self_attn.q_proj", (q, h)), ("self_attn.k_proj", (kv, h)),
                            ("self_attn.v_proj", (kv, h)), ("self_attn.o_proj", (h, q)),
                            ("mlp.gate_proj", (i, h)), ("mlp.up_proj", (i, h)),
                            ("mlp.down_proj", (h, i))):
            t[p + name + ".weight"] = torch.randn(*shape, generator=g) * 0.05
    t = {k: x.to(torch.bfloat16).contiguous() for k, x in t.items()}
    os.makedirs(path, exist_ok=True)
    save_file(t, os.path.join(path, "model.safetensors"))
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(c, f)
    return t


def _bits(x):
    return x.contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.fixture(scope="module")
def converted(tmp_path_factory, built_library):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from test_speed_scalesweep_b200 import checkpoint
    root = tmp_path_factory.mktemp("ckpt")
    src = _tiny_checkpoint(str(root / "src"))
    dst = str(root / "dst")
    summary = checkpoint.quantize_checkpoint(str(root / "src"), dst, act_amax=16.0)
    from safetensors import safe_open
    with safe_open(os.path.join(dst, "model.safetensors"), framework="pt") as h:
        out = {k: h.get_tensor(k) for k in h.keys()}
    return src, dst, out, summary


def test_codes_scales_and_shared_global_scale_match_the_oracle(converted):
    src, _, out, summary = converted
    assert summary["quantized_linears"] == 14 and summary["fused_groups"] == 4
    p = "model.layers.1.self_attn."
    ws = [src[p + f"{m}_proj.weight"] for m in "qkv"]
    amax = max(oracle.absmax(_bits(w)) for w in ws)
    gsi = np.float32(oracle.global_scale_inv(amax, 448.0))
    for m, w in zip("qkv", ws):
        assert out[p + f"{m}_proj.weight_global_scale"].item() == gsi
        c, s = oracle.quantize(_bits(w), float(gsi), mode="rtn", swizzled=False)
        assert np.array_equal(out[p + f"{m}_proj.weight_packed"].numpy(), c)
        assert np.array_equal(out[p + f"{m}_proj.weight_scale"].view(torch.uint8).numpy(), s)
        assert out[p + f"{m}_proj.input_global_scale"].item() == np.float32(448.0 * 6 / 16.0)
    d = "model.layers.0.mlp.down_proj."
    gd = np.float32(oracle.global_scale_inv(oracle.absmax(_bits(src[d + "weight"])), 448.0))
    assert out[d + "weight_global_scale"].item() == gd
    assert torch.equal(out["lm_head.weight"], src["lm_head.weight"])


VLLM_SCRIPT = r"""
import json, os, sys
os.environ["VLLM_ENABLE_V1_MULTIPROCESSING"] = "0"
import torch
from vllm import LLM, SamplingParams
from vllm.inputs import TokensPrompt
llm = LLM(model=sys.argv[1], skip_tokenizer_init=True, dtype="bfloat16", max_model_len=256,
          max_num_seqs=4, gpu_memory_utilization=0.2, enforce_eager=True, seed=0,
          kernel_config={"linear_backend": "cutlass"})
def probe(m):
    qkv = m.model.layers[1].self_attn.qkv_proj
    n, k2 = qkv.output_size_per_partition, qkv.input_size_per_partition // 2
    return {"gsi_in": qkv.input_global_scale_inv.item(), "alpha": qkv.alpha.item(),
            "weight": qkv.weight.data[:n, :k2].cpu().numpy().tolist()}
info = llm.apply_model(probe)[0]
outs = llm.generate([TokensPrompt(prompt_token_ids=[1, 2, 3, 4, 5])],
                    SamplingParams(max_tokens=4, temperature=0.0, detokenize=False))
info["tokens"] = list(outs[0].outputs[0].token_ids)
print("RESULT " + json.dumps(info), flush=True)
"""


def test_vllm_loads_the_checkpoint(converted, tmp_path):
    pytest.importorskip("vllm._custom_ops")
    _, dst, out, _ = converted
    script = tmp_path / "load.py"
    script.write_text(VLLM_SCRIPT)
    r = subprocess.run([sys.executable, str(script), dst], capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    line = next(x for x in r.stdout.splitlines() if x.startswith("RESULT "))
    info = json.loads(line[len("RESULT "):])
    p = "model.layers.1.self_attn."
    codes = torch.cat([out[p + f"{m}_proj.weight_packed"] for m in "qkv"]).numpy()
    assert np.array_equal(np.array(info["weight"], dtype=np.uint8), codes)
    gsi_in = out[p + "q_proj.input_global_scale"].item()
    gsi_w = out[p + "q_proj.weight_global_scale"].item()
    assert info["gsi_in"] == gsi_in
    assert np.isclose(info["alpha"], (1.0 / gsi_in) * (1.0 / gsi_w), rtol=1e-6)
    assert len(info["tokens"]) == 4


def test_calibration_measures_each_linears_input_amax(converted, tmp_path):
    """calibrate() against torch hooks on the same model and tokens: the
    amax of every target Linear's input, bit for bit (max is exact)."""
    from transformers import AutoModelForCausalLM
    from test_speed_scalesweep_b200 import checkpoint
    src_dir = os.path.join(os.path.dirname(converted[1]), "src")
    g = torch.Generator().manual_seed(7)
    batches = [torch.randint(0, TINY["vocab_size"], (2, 24), generator=g).tolist()
               for _ in range(3)]
    amax = checkpoint.calibrate(src_dir, batches)
    assert len(amax) == 14
    model = AutoModelForCausalLM.from_pretrained(src_dir, dtype=torch.bfloat16).cuda().eval()
    seen = {}
    hooks = [m.register_forward_pre_hook(
        lambda mod, args, n=n: seen.__setitem__(n, max(seen.get(n, 0.0),
                                                       args[0].abs().max().float().item())))
        for n, m in model.named_modules() if n in amax]
    with torch.no_grad():
        for b in batches:
            model(input_ids=torch.tensor(b, device="cuda"))
    for h in hooks:
        h.remove()
    assert seen.keys() == amax.keys()
    for n in amax:
        assert amax[n] == seen[n], n
    p = "model.layers.0.self_attn."
    assert amax[p + "q_proj"] == amax[p + "k_proj"] == amax[p + "v_proj"]  # one input
    dst = str(tmp_path / "calibrated")
    checkpoint.quantize_checkpoint(src_dir, dst, act_amax=amax)
    from safetensors import safe_open
    with safe_open(os.path.join(dst, "model.safetensors"), framework="pt") as h:
        got = h.get_tensor(p + "o_proj.input_global_scale").item()
    assert got == np.float32(oracle.global_scale_inv(amax[p + "o_proj"], 448.0))
