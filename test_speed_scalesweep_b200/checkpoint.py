"""Offline NVFP4 checkpoint writer on this package's kernels.

The reference makes its W4A4 checkpoint with llmcompressor
(``quant_model_nvfp4.py:57-87``): ``oneshot`` with a
``QuantizationModifier(targets="Linear", scheme="NVFP4", ignore=["lm_head"])``
writes a compressed-tensors ``nvfp4-pack-quantized`` checkpoint, which vLLM
loads with ``CompressedTensorsW4A4Fp4``.  This module writes the same format
from a bf16 safetensors checkpoint, quantizing on the GPU:

- per Linear ``<name>``: ``weight_packed`` uint8 [N, K/2] (two E2M1 codes a
  byte, even element in the low nibble), ``weight_scale`` float8_e4m3fn
  [N, K/16] (row-major, not swizzled; vLLM swizzles it when loading),
  ``weight_global_scale`` and ``input_global_scale`` float32 [1].  The global
  scales are stored as the quantizer's multiplier ``fp8_max * 6 / amax``;
  vLLM takes the reciprocal (vllm 0.22
  ``compressed_tensors/schemes/compressed_tensors_w4a4_nvfp4.py:105-121``);
- layers vLLM fuses (q/k/v, gate/up) share one weight global scale, the one
  of their joint amax, since vLLM keeps a single one per fused layer
  (``:93-113``);
- everything else (embeddings, norms, ``lm_head``) is copied unchanged.

Weights are quantized with this package's RTN kernel (the rounding of
vLLM's ``scaled_fp4_quant``), or with the scale-sweep MSE kernel.  The
activation global scales come from an activation amax: one value, one per
layer, or measured by ``calibrate`` (the role of llmcompressor's
calibration pass in ``oneshot``), which runs the bf16 model over
calibration token ids and keeps the running max |input| of every target
Linear on the device.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import re
import shutil
import warnings

import torch

FP8_MAX = 448.0
# Linear weights of Llama-family checkpoints; lm_head is left in bf16 as the
# reference's recipe ignores it.
DEFAULT_TARGETS = r".*\.(q|k|v|o|gate|up|down)_proj\.weight$"
FUSED_GROUPS = (("q_proj", "k_proj", "v_proj"), ("gate_proj", "up_proj"))


def fused_groups(names, targets: str = DEFAULT_TARGETS):
    """Group target weight names that vLLM loads into one fused layer:
    returns a list of lists of names (singletons for unfused layers)."""
    pat = re.compile(targets)
    chosen = sorted(n for n in names if pat.match(n))
    groups, seen = [], set()
    for name in chosen:
        if name in seen:
            continue
        parent, leaf = name.rsplit(".", 2)[0], name.rsplit(".", 2)[1]
        group = [name]
        for members in FUSED_GROUPS:
            if leaf in members:
                group = [f"{parent}.{m}.weight" for m in members
                         if f"{parent}.{m}.weight" in chosen]
                break
        seen.update(group)
        groups.append(group)
    return groups


def _quantizers(weight_quantizer: str):
    from . import global_scale
    from .scalesweep_mse_nvfp4_utils import rtn_nvfp4_quant_impl, scalesweep_mse_nvfp4_quant_impl
    quant = {"rtn": rtn_nvfp4_quant_impl,
             "scalesweep_mse": scalesweep_mse_nvfp4_quant_impl}[weight_quantizer]
    return global_scale.absmax, global_scale.global_scale_from_amax, quant


def quantize_group(weights: list[torch.Tensor], weight_quantizer: str = "rtn"):
    """Quantize the bf16 [N_i, K] weights of one fused group on their (CUDA)
    device with one shared global scale.  Returns (global scale float32 [1],
    [(codes uint8 [N_i, K/2], scales float8_e4m3fn [N_i, K/16]), ...])."""
    absmax, scale_from_amax, quant = _quantizers(weight_quantizer)
    for w in weights:
        if w.dim() != 2 or w.shape[1] % 16:
            raise ValueError(f"a weight must be 2-D with K % 16 == 0, got {tuple(w.shape)}")
    amax = torch.stack([absmax(w).reshape(()) for w in weights]).max().reshape(1)
    gsi = scale_from_amax(amax, weight_fp8_max(weight_quantizer))
    return gsi, [quant(w, gsi, False) for w in weights]


def weight_fp8_max(weight_quantizer: str) -> float:
    """FP8 range behind a weight group's global scale: 448 for RTN, 256 for
    the scale sweep, whose candidates above the base scale need E4M3 headroom
    (the reference's convention for scale-sweep backends,
    bench_kernel/test_kernel_latency.py:73-75)."""
    from . import global_scale
    if weight_quantizer not in ("rtn", "scalesweep_mse"):
        raise ValueError(f"unknown weight quantizer {weight_quantizer!r}")
    return global_scale.fp8_scale_max(weight_quantizer)


def check_activation_amax(name: str, amax: float) -> float:
    """An activation amax that gives a finite, nonzero input global scale."""
    if not math.isfinite(amax) or amax <= 0.0:
        raise ValueError(f"activation amax of {name} is {amax}: the input global scale "
                         f"fp8_max*6/amax would not be finite and positive (a layer that saw "
                         f"no calibration input, or inf/NaN activations)")
    return amax


def activation_scale(amax: float, device) -> torch.Tensor:
    """The activation global scale ``fp8_max * 6 / amax`` as float32 [1],
    evaluated as torch evaluates the reference's expression."""
    from . import global_scale
    return global_scale.global_scale_from_amax(
        torch.tensor([amax], dtype=torch.float32, device=device), FP8_MAX)


def quantization_config() -> dict:
    from .vllm_e2e import NVFP4_QUANT_CONFIG
    return json.loads(json.dumps(NVFP4_QUANT_CONFIG))


def _load_tensors(source: str) -> dict[str, torch.Tensor]:
    from safetensors import safe_open
    files = sorted(f for f in os.listdir(source) if f.endswith(".safetensors"))
    if not files:
        raise FileNotFoundError(f"No safetensors checkpoint found in: {source}")
    out = {}
    for f in files:
        with safe_open(os.path.join(source, f), framework="pt") as h:
            for k in h.keys():
                out[k] = h.get_tensor(k)
    return out


def calibrate(source: str, token_batches, *, targets: str = DEFAULT_TARGETS,
              device: str = "cuda") -> dict[str, float]:
    """Activation amax of every target Linear of the bf16 model in
    ``source``, over forward passes on ``token_batches`` (lists of token-id
    lists).  Returns {layer prefix: amax}, the ``act_amax`` mapping of
    ``quantize_checkpoint``.  The model runs under transformers in bf16; a
    forward pre-hook on each target Linear folds max |input| (this package's
    absmax kernel) into a running maximum on the device."""
    from transformers import AutoModelForCausalLM
    from . import global_scale
    if not torch.device(device).type == "cuda" or not torch.cuda.is_available():
        raise ValueError("calibration needs a CUDA device (there is no CPU implementation)")
    model = AutoModelForCausalLM.from_pretrained(source, dtype=torch.bfloat16).to(device)
    model.eval()
    pat = re.compile(targets)
    running: dict[str, torch.Tensor] = {}
    handles = []
    for name, mod in model.named_modules():
        if isinstance(mod, torch.nn.Linear) and pat.match(name + ".weight"):
            running[name] = torch.zeros(1, dtype=torch.float32, device=device)

            def hook(module, args, name=name):
                x = args[0]
                if x.numel() == 0:  # an empty batch carries no amax
                    return
                torch.maximum(running[name], global_scale.absmax(x.contiguous()),
                              out=running[name])
            handles.append(mod.register_forward_pre_hook(hook))
    try:
        with torch.no_grad():
            for batch in token_batches:
                ids = torch.tensor(batch, dtype=torch.long, device=device)
                model(input_ids=ids)
    finally:
        for h in handles:
            h.remove()
    torch.cuda.synchronize()
    result = {name: float(v.item()) for name, v in running.items()}
    unseen = [n for n, v in result.items() if v == 0.0]
    if unseen:
        warnings.warn(f"{len(unseen)} target layers saw no nonzero calibration input "
                      f"(amax 0), e.g. {unseen[0]}; quantize_checkpoint will reject them")
    return result


def quantize_checkpoint(source: str, destination: str, *, act_amax: float | dict = 16.0,
                        weight_quantizer: str = "rtn", targets: str = DEFAULT_TARGETS,
                        device: str = "cuda") -> dict:
    """Write the NVFP4 checkpoint of ``source`` (a directory with config.json
    and bf16 safetensors) to ``destination``.  ``act_amax``: the activation
    amax of every layer, or a {weight name prefix: amax} mapping (missing
    layers raise).  Returns a summary."""
    from safetensors.torch import save_file
    if not os.path.isdir(source):
        raise FileNotFoundError(f"Source model is not a directory: {source}")
    if os.path.exists(destination) and os.listdir(destination):
        raise FileExistsError(f"Output directory is not empty: {destination}")
    if not torch.device(device).type == "cuda" or not torch.cuda.is_available():
        raise ValueError("quantizing needs a CUDA device (there is no CPU implementation)")
    tensors = _load_tensors(source)
    groups = fused_groups(tensors.keys(), targets)
    out: dict[str, torch.Tensor] = {}
    quantized = set()
    for group in groups:
        ws = [tensors[n].to(device=device, dtype=torch.bfloat16).contiguous() for n in group]
        gsi, results = quantize_group(ws, weight_quantizer)
        for name, (codes, scales) in zip(group, results):
            prefix = name[: -len(".weight")]
            amax = check_activation_amax(
                prefix, float(act_amax[prefix] if isinstance(act_amax, dict) else act_amax))
            out[prefix + ".weight_packed"] = codes.cpu()
            out[prefix + ".weight_scale"] = scales.cpu()
            out[prefix + ".weight_global_scale"] = gsi.cpu().clone()  # one tensor per name
            out[prefix + ".input_global_scale"] = activation_scale(float(amax), device).cpu()
            quantized.add(name)
        del ws, results
    for name, t in tensors.items():
        if name not in quantized:
            out[name] = t
    os.makedirs(destination, exist_ok=True)
    save_file(out, os.path.join(destination, "model.safetensors"), metadata={"format": "pt"})
    with open(os.path.join(source, "config.json")) as f:
        cfg = json.load(f)
    cfg["quantization_config"] = quantization_config()
    with open(os.path.join(destination, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    for f in os.listdir(source):  # tokenizer and generation files travel as they are
        if not f.endswith(".safetensors") and f not in ("config.json",
                                                        "model.safetensors.index.json"):
            p = os.path.join(source, f)
            if os.path.isfile(p):
                shutil.copy(p, os.path.join(destination, f))
    return {"quantized_linears": len(quantized), "fused_groups": sum(len(g) > 1 for g in groups),
            "weight_quantizer": weight_quantizer, "tensors_written": len(out)}


def main() -> None:
    ap = argparse.ArgumentParser(description="Write an NVFP4 (compressed-tensors "
                                             "nvfp4-pack-quantized) checkpoint on a B200.")
    ap.add_argument("source")
    ap.add_argument("destination")
    ap.add_argument("--act-amax", default="16.0",
                    help="activation amax of every layer, or a JSON file {layer prefix: amax}")
    ap.add_argument("--weight-quantizer", choices=["rtn", "scalesweep_mse"], default="rtn")
    ap.add_argument("--calibration-tokens", default=None,
                    help="JSON file of token-id batches ([[ids, ...], ...] per batch); the "
                         "activation amax is then measured (overrides --act-amax)")
    args = ap.parse_args()
    if args.calibration_tokens:
        with open(args.calibration_tokens) as f:
            act = calibrate(args.source, json.load(f))
    elif os.path.isfile(args.act_amax):
        with open(args.act_amax) as f:
            act = {k: float(v) for k, v in json.load(f).items()}
    else:
        act = float(args.act_amax)
    print(json.dumps(quantize_checkpoint(args.source, args.destination, act_amax=act,
                                         weight_quantizer=args.weight_quantizer)))


if __name__ == "__main__":
    main()
