"""CPU test of the vLLM compile-pass routing (vllm_fusion.py): the pattern
pass rewrites each producer -> scale-sweep quantizer pair of a traced graph
into this package's fused op, and leaves unsupported pairs alone.  The graph
is traced in fake mode with the same decompositions vLLM's pattern passes use
(``torch._inductor.pattern_matcher.fwd_only``), so nothing runs on a device."""
import pytest
import torch

vllm_ir = pytest.importorskip("vllm.ir.ops")

from test_speed_scalesweep_b200 import ops as _ops  # noqa: E402,F401
from test_speed_scalesweep_b200 import vllm_fusion  # noqa: E402


def _fused_eps(gm):
    """The epsilon each fused norm op received, by op name."""
    out = {}
    for n in gm.graph.nodes:
        if n.op != "call_function":
            continue
        if "rms_norm_scalesweep_mse_nvfp4_quant" in str(n.target):
            out["rms_norm"] = n.args[2]
        if "auto_functionalized" in str(n.target) and "fused_add_rms_norm_nvfp4" in str(n.args[0]):
            out["fused_add_rms_norm"] = n.kwargs["epsilon"]
    return out


def _trace_and_fuse(fn, inputs):
    import torch._inductor.pattern_matcher as pm
    from torch._inductor.pattern_matcher import PatternMatcherPass
    from torch._subclasses.fake_tensor import FakeTensorMode
    with torch._guards.tracing(None), FakeTensorMode():
        fake = [torch.empty(*shape, dtype=dt, device="cuda") for shape, dt in inputs]
        gm = pm.fwd_only(fn, fake)
        pm_pass = PatternMatcherPass(pass_name="test_scalesweep_fusion")
        vllm_fusion.register_patterns(pm_pass)
        for k in vllm_fusion.MATCHES:
            vllm_fusion.MATCHES[k] = 0
        count = pm_pass.apply(gm.graph)
    gm.graph.lint()
    _trace_and_fuse.last_eps = _fused_eps(gm)
    # an auto_functionalized node names the in-place op it wraps as its first argument
    targets = [str(n.args[0]) if "auto_functionalized" in str(n.target) else str(n.target)
               for n in gm.graph.nodes if n.op == "call_function"]
    return count, targets


def _decoder_like(x, w, r, gsi, gu):
    quant = torch.ops.scalesweep_b200.scalesweep_mse_nvfp4_quant
    normed, res = vllm_ir.fused_add_rms_norm(x, r, w, 1e-5)
    c1, s1 = quant(normed, gsi, True, None)
    c2, s2 = quant(vllm_ir.rms_norm(x, w, 1e-6), gsi, True, None)
    d = gu.shape[-1] // 2
    h = torch.nn.functional.silu(gu[..., :d]) * gu[..., d:]
    c3, s3 = quant(h, gsi, True, None)
    return c1, s1, res, c2, s2, c3, s3


BF16, F32 = torch.bfloat16, torch.float32


def test_pass_fuses_norms_and_silu_into_the_quantizer():
    count, targets = _trace_and_fuse(
        _decoder_like, [((8, 64), BF16), ((64,), BF16), ((8, 64), BF16), ((1,), F32),
                        ((8, 256), BF16)])
    assert count == 3
    assert vllm_fusion.MATCHES == {"rms_norm": 1, "fused_add_rms_norm": 1, "silu_and_mul": 1}
    joined = " ".join(targets)
    assert "scalesweep_b200.scalesweep_mse_nvfp4_quant" not in joined
    assert "scalesweep_b200.rms_norm_scalesweep_mse_nvfp4_quant" in joined
    assert "scalesweep_b200.fused_add_rms_norm_nvfp4_quant" in joined
    assert "scalesweep_b200.silu_and_mul_scalesweep_mse_nvfp4_quant" in joined
    assert "vllm_ir.rms_norm" not in joined and "vllm_ir.fused_add_rms_norm" not in joined
    # each fused op carries its own norm's epsilon (1e-5 for the fused add, 1e-6 for the plain)
    assert _trace_and_fuse.last_eps == {"fused_add_rms_norm": 1e-5, "rms_norm": 1e-6}


def _norm_then_quant_and_reuse(x, w, gsi):
    quant = torch.ops.scalesweep_b200.scalesweep_mse_nvfp4_quant
    normed = vllm_ir.rms_norm(x, w, 1e-5)
    c, s = quant(normed, gsi, True, None)
    return c, s, normed * 2  # the norm output has a second user: no fusion


def test_pass_leaves_a_shared_producer_alone():
    count, targets = _trace_and_fuse(_norm_then_quant_and_reuse,
                                     [((8, 64), BF16), ((64,), BF16), ((1,), F32)])
    assert count == 0
    assert any("scalesweep_b200.scalesweep_mse_nvfp4_quant" in t for t in targets)


def _f16_norm(x, w, gsi):
    quant = torch.ops.scalesweep_b200.scalesweep_mse_nvfp4_quant
    c, s = quant(vllm_ir.rms_norm(x, w, 1e-5), gsi, True, None)
    return c, s


def test_pass_skips_inputs_the_fused_kernel_does_not_take():
    # the norm front end is bf16 only: an f16 RMSNorm keeps the unfused pair
    count, _ = _trace_and_fuse(_f16_norm, [((8, 64), torch.float16), ((64,), torch.float16),
                                           ((1,), F32)])
    assert count == 0


def test_install_appends_the_pass_after_vllms_own(monkeypatch):
    pm_mod = pytest.importorskip("vllm.compilation.passes.pass_manager")
    cls = pm_mod.PostGradPassManager
    calls = []

    def stub_configure(self, config):  # stands in for vLLM's own pass list
        self.passes = ["vllm-pass"]
        calls.append(config)

    monkeypatch.setattr(cls, "configure", stub_configure)
    made = []

    class FakePass:
        def __init__(self, config):
            made.append(config)

    monkeypatch.setattr(vllm_fusion, "_PASS_CLASS", FakePass)
    import vllm.config as vcfg
    monkeypatch.setattr(vcfg, "set_current_vllm_config",
                        lambda config, check_compile=False: __import__("contextlib").nullcontext())
    vllm_fusion.install_fusion_pass()
    vllm_fusion.install_fusion_pass()  # idempotent: one wrapper
    mgr = cls.__new__(cls)
    cls.configure(mgr, "cfg")
    assert calls == ["cfg"] and made == ["cfg"]
    assert mgr.passes[0] == "vllm-pass" and isinstance(mgr.passes[1], FakePass)
    assert len(mgr.passes) == 2
