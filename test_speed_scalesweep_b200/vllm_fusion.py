"""vLLM compile-pass routing of the fused scale-sweep quantizers.

vLLM fuses a producer into the NVFP4 activation quantizer with post-grad
pattern-matcher passes.  With ``fuse_act_quant``, ``SiluMulNvfp4QuantPattern``
(vllm 0.22 ``compilation/passes/fusion/act_quant_fusion.py:124-168``) rewrites
SiLU-and-mul followed by ``torch.ops._C.scaled_fp4_quant.out`` into
``_C.silu_and_mul_nvfp4_quant``.  Those patterns name vLLM's own RTN
quantizer.  Once ``vllm_e2e.install_act_quant_hook`` routes the W4A4 linear
layers through this package, the graph holds
``torch.ops.scalesweep_b200.scalesweep_mse_nvfp4_quant`` instead, so they never
match.  vLLM 0.22 also has no RMSNorm + NVFP4 pattern at all
(``rms_quant_fusion.py:103-128`` lists FP8 keys only).

``ScaleSweepQuantFusionPass`` supplies the patterns for this quantizer:

- ``vllm_ir.rms_norm`` -> quant becomes ``rms_norm_scalesweep_mse_nvfp4_quant``;
- ``vllm_ir.fused_add_rms_norm`` -> quant becomes
  ``fused_add_rms_norm_nvfp4_quant``, with the residual updated in place as
  the IR op returns it;
- SiLU-and-mul -> quant becomes ``silu_and_mul_scalesweep_mse_nvfp4_quant``.
  This covers both forms vLLM may trace: the native
  ``F.silu(x[..., :d]) * x[..., d:]`` and its ``_C.silu_and_mul`` custom op.

The fused kernels compute the producer as vLLM's CUDA kernels do
(``_C.rms_norm``, ``_C.fused_add_rms_norm``, ``_C.silu_and_mul``).  Where
Inductor would have compiled the native form instead, the fused result can
differ from the unfused compiled graph in the last bits of the producer's
bf16 output.  vLLM's own fusion passes make the same substitution.

``install_fusion_pass()`` appends the pass to vLLM's ``PostGradPassManager``,
after vLLM's own passes and before IR lowering.  It then applies to any model
whose compiled graph holds these producer -> quantizer pairs, not only to
Llama's modules.  ``MATCHES`` counts, per pattern kind, the matches its
check accepted (Inductor compiles each distinct graph piece once, so
identical decoder layers count once).
"""
from __future__ import annotations

import torch

QUANT_FUNCTIONAL = "scalesweep_mse_nvfp4_quant"
EPSILONS = (1e-5, 1e-6)
MATCHES = {"rms_norm": 0, "fused_add_rms_norm": 0, "silu_and_mul": 0}


def _quant():
    return getattr(torch.ops.scalesweep_b200, QUANT_FUNCTIONAL).default


def _round_up(x, m):
    return (x + m - 1) // m * m


def _meta(match, name):
    node = match.kwargs.get(name)
    return getattr(node, "meta", {}).get("val") if node is not None else None


def _norm_supported(match) -> bool:
    """The fused norm front end is bf16 only, with a row width the quantizer
    takes (a multiple of 16) and a weight of that width."""
    x, w = _meta(match, "input"), _meta(match, "weight")
    if x is None or w is None:
        return False
    return (x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and x.dim() == 2
            and w.dim() == 1 and x.shape[-1] == w.shape[0] and x.shape[-1] % 16 == 0)


def _silu_supported(match) -> bool:
    """bf16 or f16 gate_up rows of 2n values, n a multiple of 16."""
    x = _meta(match, "input")
    if x is None:
        return False
    return (x.dtype in (torch.bfloat16, torch.float16) and x.dim() == 2
            and x.shape[-1] % 32 == 0)


def _example(*shape, dtype=torch.bfloat16):
    return torch.empty(*shape, dtype=dtype, device="cuda")


def _norm_eps_is(eps):
    """Inductor's pattern matcher treats float literals as wildcards, so a
    pattern traced with one epsilon also matches norms with another.  Each
    epsilon's pattern therefore accepts only a matched norm node that
    carries its own epsilon, and the replacement passes that value on."""
    targets = {"vllm_ir.rms_norm.default", "vllm_ir.fused_add_rms_norm.default"}

    def check(match) -> bool:
        for node in match.nodes:
            if str(node.target) in targets:
                floats = [a for a in node.args if isinstance(a, float)]
                return bool(floats) and floats[-1] == eps
        return False
    return check


def _all(*checks):
    return lambda match: all(c(match) for c in checks)


def _counted(kind, check):
    def extra_check(match) -> bool:
        ok = check(match)
        if ok:
            MATCHES[kind] += 1
        return ok
    return extra_check


def register_patterns(pm_pass) -> None:
    """Register every pattern into ``pm_pass`` (an Inductor PatternMatcherPass).
    Runs under fake mode: the example inputs only fix ranks and dtypes."""
    import torch._inductor.pattern_matcher as pm
    import vllm.ir.ops
    from torch._higher_order_ops.auto_functionalize import auto_functionalized

    from . import ops as _ops  # noqa: F401  (registers torch.ops.scalesweep_b200.*)

    quant = _quant()
    ops = torch.ops.scalesweep_b200

    def norm_patterns(eps):
        # the pattern functions' arguments are exactly the graph inputs, so
        # the epsilon is closed over rather than passed
        def add_pattern(input, weight, residual, scale):
            normed, res = vllm.ir.ops.fused_add_rms_norm(input, residual, weight, eps)
            q = quant(normed, scale, True, None)
            return q[0], q[1], res

        def add_replacement(input, weight, residual, scale):
            m, n = input.shape
            codes = torch.empty((m, n // 2), dtype=torch.uint8, device=input.device)
            scales = torch.empty((_round_up(m, 128), _round_up(n // 16, 4)),
                                 dtype=torch.float8_e4m3fn, device=input.device)
            at = auto_functionalized(ops.fused_add_rms_norm_nvfp4_quant.default, result=codes,
                                     result_block_scale=scales, input=input, residual=residual,
                                     weight=weight, input_global_scale=scale, epsilon=eps)
            return at[1], at[2], at[3]

        def norm_pattern(input, weight, scale):
            q = quant(vllm.ir.ops.rms_norm(input, weight, eps), scale, True, None)
            return q[0], q[1]

        def norm_replacement(input, weight, scale):
            q = ops.rms_norm_scalesweep_mse_nvfp4_quant.default(input, weight, eps, scale, True)
            return q[0], q[1]

        return add_pattern, add_replacement, norm_pattern, norm_replacement

    for eps in EPSILONS:
        add_p, add_r, norm_p, norm_r = norm_patterns(eps)
        # fused_add_rms_norm first: plain rms_norm is a subgraph of its native form
        pm.register_replacement(add_p, add_r,
                                [_example(5, 32), _example(32), _example(5, 32),
                                 _example(1, dtype=torch.float32)],
                                pm.fwd_only, pm_pass,
                                extra_check=_counted("fused_add_rms_norm",
                                                     _all(_norm_eps_is(eps), _norm_supported)))
        pm.register_replacement(norm_p, norm_r,
                                [_example(5, 32), _example(32), _example(1, dtype=torch.float32)],
                                pm.fwd_only, pm_pass,
                                extra_check=_counted("rms_norm",
                                                     _all(_norm_eps_is(eps), _norm_supported)))

    def silu_replacement(input, scale):
        q = ops.silu_and_mul_scalesweep_mse_nvfp4_quant.default(input, scale, True)
        return q[0], q[1]

    def silu_native_pattern(input, scale):
        d = input.shape[-1] // 2
        h = torch.nn.functional.silu(input[..., :d]) * input[..., d:]
        q = quant(h, scale, True, None)
        return q[0], q[1]

    silu_inputs = [_example(5, 64), _example(1, dtype=torch.float32)]
    pm.register_replacement(silu_native_pattern, silu_replacement, silu_inputs, pm.fwd_only,
                            pm_pass, extra_check=_counted("silu_and_mul", _silu_supported))

    silu_op = getattr(getattr(torch.ops, "_C", None), "silu_and_mul", None)
    if silu_op is not None:
        def silu_custom_pattern(input, scale):
            d = input.shape[-1] // 2
            out = torch.empty(input.shape[:-1] + (d,), dtype=input.dtype, device=input.device)
            h = auto_functionalized(silu_op.default, result=out, input=input)[1]
            q = quant(h, scale, True, None)
            return q[0], q[1]

        pm.register_replacement(silu_custom_pattern, silu_replacement, silu_inputs, pm.fwd_only,
                                pm_pass, extra_check=_counted("silu_and_mul", _silu_supported))


def make_pass_class():
    """The pass as a subclass of vLLM's ``VllmPatternMatcherPass`` (built on
    first use, so importing this module does not import vLLM)."""
    from torch._inductor.pattern_matcher import PatternMatcherPass
    from vllm.compilation.passes.inductor_pass import enable_fake_mode
    from vllm.compilation.passes.vllm_inductor_pass import (VllmInductorPass,
                                                            VllmPatternMatcherPass)

    from . import ops  # noqa: F401  (registers torch.ops.scalesweep_b200.*)

    class ScaleSweepQuantFusionPass(VllmPatternMatcherPass):
        """RMSNorm / fused-add RMSNorm / SiLU-and-mul fused into this package's
        scale-sweep NVFP4 quantizer (module docstring)."""

        @enable_fake_mode
        def __init__(self, config) -> None:
            super().__init__(config)
            self.patterns = PatternMatcherPass(pass_name="scalesweep_quant_fusion_pass")
            register_patterns(self.patterns)

        @VllmInductorPass.time_and_log
        def __call__(self, graph: torch.fx.Graph) -> None:
            self.matched_count = self.patterns.apply(graph)

        def uuid(self) -> str:
            return self.hash_source(self, register_patterns, _norm_supported, _silu_supported,
                                    _norm_eps_is)

    return ScaleSweepQuantFusionPass


_PASS_CLASS = None


def fusion_pass_class():
    global _PASS_CLASS
    if _PASS_CLASS is None:
        _PASS_CLASS = make_pass_class()
    return _PASS_CLASS


def install_fusion_pass() -> None:
    """Append ``ScaleSweepQuantFusionPass`` to every vLLM post-grad pass
    manager configured from now on (idempotent)."""
    from vllm.compilation.passes.pass_manager import PostGradPassManager
    from vllm.config import set_current_vllm_config

    original = PostGradPassManager.configure
    if getattr(original, "_scalesweep_b200", False):
        return
    cls = fusion_pass_class()

    def configure(self, config):
        original(self, config)
        with set_current_vllm_config(config, check_compile=False):
            self.passes.append(cls(config))

    configure._scalesweep_b200 = True
    PostGradPassManager.configure = configure
