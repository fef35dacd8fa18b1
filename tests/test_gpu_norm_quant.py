"""GPU parity of RMSNorm fused into the scalesweep_mse quantizer (through the
C ABI): against the CPU oracle (vLLM's reduction order restated; the
device's rsqrtf bounded, then every byte compared), and against vLLM's own
rms_norm / fused_add_rms_norm composed with the unfused quantizer, bit for
bit, at Llama-3.1-8B widths on both sides of vLLM's 256-row block-size
switch."""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

SENTINEL = 0xA5
EPS = 1e-5


@pytest.fixture(scope="module")
def mods(built_library):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from test_speed_scalesweep_b200 import custom, norm_quant, ops  # noqa: F401
    return custom, norm_quant


def bits_of(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def make_case(m, n, seed):
    """x with row magnitudes spread over four decades and 0.5% outlier
    channels x20; weight 1 + 0.3 N(0,1); residual 4 N(0,1); all bf16."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, n, generator=g) * torch.logspace(-2, 2, max(m, 1))[:m, None]
    cols = torch.randperm(n, generator=g)[: max(1, n // 200)]
    x[:, cols] *= 20.0
    w = 1.0 + 0.3 * torch.randn(n, generator=g)
    res = 4.0 * torch.randn(m, n, generator=g)
    return (x.to(torch.bfloat16).cuda(), w.to(torch.bfloat16).cuda(),
            res.to(torch.bfloat16).cuda())


def sentinel_outputs(m, n, swizzled):
    codes = torch.full((m, n // 2), SENTINEL, dtype=torch.uint8, device="cuda")
    scales = torch.full(oracle.scale_shape(m, n, swizzled), SENTINEL, dtype=torch.uint8,
                        device="cuda")
    return codes, scales


def ulp_distance(a, b):
    """|a - b| in float32 units in the last place of b (both positive)."""
    ulp = np.spacing(b.astype(np.float32)).astype(np.float64)
    return np.abs(a.astype(np.float64) - b.astype(np.float64)) / ulp


@pytest.mark.parametrize("m,n", [(1, 2048), (7, 4096), (255, 1024), (256, 1024), (300, 2048)])
@pytest.mark.parametrize("add", [False, True])
@pytest.mark.parametrize("swizzled", [True, False])
def test_matches_oracle(mods, m, n, add, swizzled):
    _, nq = mods
    x, w, res = make_case(m, n, seed=m * 7 + n + add)
    xb, wb, rb = bits_of(x), bits_of(w), bits_of(res)
    gsi = 448.0 * 6.0 / 60.0
    codes, scales = sentinel_outputs(m, n, swizzled)
    rstd = torch.empty(m, dtype=torch.float32, device="cuda")
    nq.rms_norm_scalesweep_mse_nvfp4_quant_out(
        x, w, EPS, torch.tensor([gsi], dtype=torch.float32, device="cuda"), swizzled,
        output=codes, output_scale=scales,
        residual=res if add else None, rstd=rstd)
    torch.cuda.synchronize()
    acc, res_ref = oracle.rms_sumsq(xb, rb if add else None)
    r_dev = rstd.cpu().numpy()
    # rsqrtf is CUDA's; its stated error bound is 2 ulp
    assert ulp_distance(r_dev, oracle.rms_rsqrt_bound(acc, n, EPS)).max() <= 2.0
    if add:
        assert np.array_equal(bits_of(res), res_ref), "residual write-back"
    normed = oracle.rms_apply(res_ref if add else xb, wb, r_dev)
    oc, os_ = oracle.quantize(normed, gsi, swizzled=swizzled)
    assert np.array_equal(codes.cpu().numpy(), oc)
    assert np.array_equal(scales.cpu().numpy(), os_)


VLLM_CASES = ([(m, n) for m in (1, 100, 255, 256, 1000) for n in (4096, 14336)]
              # widths below vLLM's block size (it launches min(n, 1024 or 256)
              # threads) and the 70B hidden size
              + [(3, 128), (300, 128), (5, 512), (260, 512), (3, 8192), (300, 8192)])


@pytest.mark.parametrize("m,n", VLLM_CASES)
@pytest.mark.parametrize("add", [False, True])
def test_matches_vllm_then_quantize(mods, m, n, add):
    """The fused op against vLLM's RMSNorm followed by the unfused
    scalesweep_mse quantizer: codes, scales and the residual bit for bit."""
    pytest.importorskip("vllm._custom_ops")
    _, nq = mods
    x, w, res = make_case(m, n, seed=3 * m + n + add)
    if add:
        xa, ra = x.clone(), res.clone()
        torch.ops._C.fused_add_rms_norm(xa, ra, w, EPS)
        normed = xa
    else:
        normed = torch.empty_like(x)
        torch.ops._C.rms_norm(normed, x, w, EPS)
    from test_speed_scalesweep_b200 import global_scale
    from test_speed_scalesweep_b200 import scalesweep_mse_nvfp4_utils as mse
    gsi = global_scale.global_scale_inv_from_max(normed, 448.0)
    # sentinel-filled outputs: the swizzled layout's padding is written by neither
    ref_codes, ref_scales = sentinel_outputs(m, n, True)
    mse.scalesweep_mse_nvfp4_quant_out(normed, gsi, True, output=ref_codes,
                                       output_scale=ref_scales.view(torch.float8_e4m3fn))
    res_f = res.clone()
    codes, scales = sentinel_outputs(m, n, True)
    nq.rms_norm_scalesweep_mse_nvfp4_quant_out(x, w, EPS, gsi, True, output=codes,
                                               output_scale=scales,
                                               residual=res_f if add else None)
    torch.cuda.synchronize()
    if add:
        assert torch.equal(res_f.view(torch.int16), ra.view(torch.int16)), "residual"
    assert torch.equal(codes, ref_codes)
    assert torch.equal(scales, ref_scales)


def test_vllm_style_ops_and_empty_input(mods):
    _, nq = mods
    m, n = 128, 4096  # whole 128-row tiles: no swizzle padding left unwritten
    x, w, res = make_case(m, n, seed=11)
    gsi = torch.tensor([448.0 * 6.0 / 50.0], dtype=torch.float32, device="cuda")
    c1, s1 = nq.rms_norm_scalesweep_mse_nvfp4_quant(x, w, EPS, gsi)
    c2, s2 = nq.alloc_outputs(x)
    torch.ops.scalesweep_b200.rms_norm_nvfp4_quant(c2, s2, x, w, gsi, EPS)
    assert torch.equal(c1, c2) and torch.equal(s1.view(torch.uint8), s2.view(torch.uint8))
    c3, s3 = torch.ops.scalesweep_b200.rms_norm_scalesweep_mse_nvfp4_quant(x, w, EPS, gsi)
    assert torch.equal(c1, c3) and torch.equal(s1.view(torch.uint8), s3.view(torch.uint8))
    r1, r2 = res.clone(), res.clone()
    c4, s4 = nq.rms_norm_scalesweep_mse_nvfp4_quant(x, w, EPS, gsi, residual=r1)
    c5, s5 = nq.alloc_outputs(x)
    torch.ops.scalesweep_b200.fused_add_rms_norm_nvfp4_quant(c5, s5, x, r2, w, gsi, EPS)
    assert torch.equal(r1.view(torch.int16), r2.view(torch.int16))
    assert torch.equal(c4, c5) and torch.equal(s4.view(torch.uint8), s5.view(torch.uint8))
    # zero rows: nothing launched, nothing written
    e = x[:0]
    ce, se = nq.rms_norm_scalesweep_mse_nvfp4_quant(e, w, EPS, gsi)
    torch.cuda.synchronize()
    assert ce.shape == (0, n // 2)
