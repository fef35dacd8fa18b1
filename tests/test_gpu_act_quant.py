"""GPU parity of SiLU-and-mul and the fused SiLU-and-mul quantizer (through
the C ABI): against the CPU oracle bit for bit, against vLLM's silu_and_mul
when its compiled ops are importable, and the fused op against the unfused
composition (silu_and_mul, then scalesweep_mse) at a full Llama-3.1-8B MLP
width."""
import ctypes

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

SENTINEL = 0xA5
TORCH_DT = {"bf16": torch.bfloat16, "f16": torch.float16}


@pytest.fixture(scope="module")
def lib(built_library):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from test_speed_scalesweep_b200 import _lib
    return _lib.lib()


def bits_of(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def nan_equal(a, b, dtype):
    ta = torch.from_numpy(a.view(np.int16)).view(TORCH_DT[dtype]).float()
    tb = torch.from_numpy(b.view(np.int16)).view(TORCH_DT[dtype]).float()
    return bool(((torch.from_numpy(a.view(np.int16)) == torch.from_numpy(b.view(np.int16)))
                 | (torch.isnan(ta) & torch.isnan(tb))).all())


def make_input(m, n, dtype, seed, specials=True):
    """[m, 2n]: gate N(0, 3) with 0.5% outlier channels x20, up N(0, 1);
    with specials, a few gates/ups at +-inf, NaN, -100 (silu -> -0) and tiny."""
    g = torch.Generator().manual_seed(seed)
    gate = torch.randn(m, n, generator=g) * 3.0
    cols = torch.randperm(n, generator=g)[: max(1, n // 200)]
    gate[:, cols] *= 20.0
    up = torch.randn(m, n, generator=g)
    if specials and m * n >= 64:
        flat_g, flat_u = gate.view(-1), up.view(-1)
        idx = torch.randperm(m * n, generator=g)[:12]
        vals = [float("inf"), float("-inf"), float("nan"), -100.0, 1e-30, -88.5]
        for i, j in enumerate(idx[:6].tolist()):
            flat_g[j] = vals[i]
        for i, j in enumerate(idx[6:].tolist()):
            flat_u[j] = vals[i]
    x = torch.cat([gate, up], dim=1).to(TORCH_DT[dtype])
    return x.cuda()


def c_silu_mul(lib, x):
    m, n2 = x.shape
    out = torch.empty(m, n2 // 2, dtype=x.dtype, device="cuda")
    st = lib.ssw_silu_and_mul(ctypes.c_void_p(x.data_ptr()), 0 if x.dtype == torch.bfloat16 else 1,
                              m, n2 // 2, ctypes.c_void_p(out.data_ptr()),
                              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0, lib.ssw_last_error()
    torch.cuda.synchronize()
    return out


def c_fused(lib, x, gsi, swizzled=True):
    m, n2 = x.shape
    n = n2 // 2
    codes = torch.full((m, n // 2), SENTINEL, dtype=torch.uint8, device="cuda")
    scales = torch.full(oracle.scale_shape(m, n, swizzled), SENTINEL, dtype=torch.uint8,
                        device="cuda")
    g = torch.tensor([gsi], dtype=torch.float32, device="cuda")
    st = lib.ssw_silu_and_mul_scalesweep_mse_nvfp4_quant_out(
        ctypes.c_void_p(x.data_ptr()), 0 if x.dtype == torch.bfloat16 else 1, m, n,
        ctypes.c_void_p(g.data_ptr()), ctypes.c_void_p(codes.data_ptr()),
        ctypes.c_void_p(scales.data_ptr()), int(swizzled),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0, lib.ssw_last_error()
    torch.cuda.synchronize()
    return codes.cpu().numpy(), scales.cpu().numpy()


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_silu_and_mul_matches_oracle_on_every_gate_value(lib, dtype):
    gate = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(TORCH_DT[dtype])
    up = torch.randn(65536, generator=torch.Generator().manual_seed(7)).to(TORCH_DT[dtype])
    x = torch.cat([gate, up]).view(1, -1).cuda()
    got = bits_of(c_silu_mul(lib, x))
    want = oracle.silu_mul(bits_of(x), dtype)
    assert nan_equal(got, want, dtype)


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_silu_and_mul_matches_vllm(lib, dtype):
    pytest.importorskip("vllm._custom_ops")
    if not hasattr(torch.ops._C, "silu_and_mul"):
        pytest.skip("vLLM compiled silu_and_mul not available")
    x = make_input(257, 1024, dtype, seed=11)
    ref = torch.empty(257, 1024, dtype=x.dtype, device="cuda")
    torch.ops._C.silu_and_mul(ref, x)
    got = c_silu_mul(lib, x)
    assert nan_equal(bits_of(got), bits_of(ref), dtype)


# (m, n): lane sharing by 4 and 2 at decode sizes, one lane per block, a
# partial 128-row scale tile, the Llama-3.1-8B intermediate width (14336)
@pytest.mark.parametrize("m,n", [(1, 64), (4, 14336), (16, 14336), (200, 2048), (1000, 512)])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("swizzled", [True, False])
def test_fused_matches_oracle(lib, m, n, dtype, swizzled):
    x = make_input(m, n, dtype, seed=m * 7 + n)
    gsi = 448.0 * 6.0 / 40.0
    codes, scales = c_fused(lib, x, gsi, swizzled)
    want_codes, want_scales = oracle.silu_mul_quantize(bits_of(x), gsi, dtype=dtype,
                                                       swizzled=swizzled)
    np.testing.assert_array_equal(codes, want_codes)
    np.testing.assert_array_equal(scales, want_scales)  # padding keeps the sentinel


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_fused_equals_unfused_composition_at_full_width(lib, dtype):
    from test_speed_scalesweep_b200 import act_quant
    from test_speed_scalesweep_b200.scalesweep_mse_nvfp4_utils import (
        scalesweep_mse_nvfp4_quant_impl)
    x = make_input(4096, 14336, dtype, seed=5)
    gsi = torch.tensor([448.0 * 6.0 / 40.0], dtype=torch.float32, device="cuda")
    fused_c, fused_s = act_quant.silu_and_mul_scalesweep_mse_nvfp4_quant(x, gsi)
    h = act_quant.silu_and_mul(x)
    c, s = scalesweep_mse_nvfp4_quant_impl(h, gsi, True)
    torch.cuda.synchronize()
    assert torch.equal(fused_c, c)
    assert torch.equal(fused_s.view(torch.uint8), s.view(torch.uint8))


def test_vllm_signature_op_writes_caller_buffers(lib):
    from test_speed_scalesweep_b200 import act_quant, ops  # noqa: F401
    x = make_input(130, 256, "bf16", seed=9)
    gsi = torch.tensor([448.0 * 6.0 / 40.0], dtype=torch.float32, device="cuda")
    result = torch.zeros(130, 128, dtype=torch.uint8, device="cuda")
    block_scale = torch.zeros(256, 4, dtype=torch.int32, device="cuda")  # 256 x 16 bytes
    torch.ops.scalesweep_b200.silu_and_mul_nvfp4_quant(result, block_scale, x, gsi)
    codes = torch.zeros(130, 128, dtype=torch.uint8, device="cuda")
    scales = torch.zeros(256, 16, dtype=torch.uint8, device="cuda")
    act_quant.silu_and_mul_scalesweep_mse_nvfp4_quant_out(x, gsi, True, output=codes,
                                                          output_scale=scales)
    torch.cuda.synchronize()
    assert torch.equal(result, codes)
    assert torch.equal(block_scale.view(torch.uint8).view(256, 16), scales)
