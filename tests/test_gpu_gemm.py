"""NVFP4 GEMM (tcgen05) against the CPU dequantize-matmul oracle and, when vLLM's
compiled ops are present, against vLLM's CUTLASS NVFP4 GEMM.  Bar: relative
Frobenius error <= 1e-2 (bf16 output rounding alone is ~2e-3)."""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

TOL = 1e-2


@pytest.fixture(scope="module")
def lib(built_library):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from test_speed_scalesweep_b200 import _lib
    return _lib.lib()


def _quantized(rows, k, seed, std, backend):
    from test_speed_scalesweep_b200 import custom, global_scale
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = (torch.randn(rows, k, generator=g, device="cuda") * std).to(torch.bfloat16)
    gsi = global_scale.global_scale_inv_from_max(x, 448.0)
    codes, scales = custom.nvfp4_quant(x, gsi, True, backend)
    return x, gsi, codes, scales


def _rel_fro(got, ref):
    got = np.asarray(got, np.float64)
    return float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))


# Persistent 256x256 CTA-pair tiles (more tiles than resident pairs):
# (2000, 2560, 512) last pair's upper CTA partial; (1793, 2560, 512) its upper
# CTA wholly past M (A scales from the last slab); (1970, 2560, 2048) upper CTA
# 50 rows, K wraps the 5-stage ring; (1400, 4608, 768) three K blocks per tile
# and two tiles for some pairs, so the ring wraps across tiles.
# One-CTA 128x256 tiles: (1281, 2560, 512), (1458, 2560, 2048).
# (64, 4096, 1024): 128x64 tiles, upper-half scale columns.
# (16, 192, 512), (200, 320, 1024): N % 128 == 64, the last 64-wide tile in
# the first half of a padded scale slab (one and two M tiles).
@pytest.mark.parametrize("m,n,k", [(128, 128, 256), (16, 256, 512), (200, 384, 1024),
                                   (1, 128, 4096), (1024, 512, 4096), (2000, 2560, 512),
                                   (1793, 2560, 512), (1970, 2560, 2048), (1400, 4608, 768),
                                   (1281, 2560, 512), (1458, 2560, 2048), (64, 4096, 1024),
                                   (16, 192, 512), (200, 320, 1024)])
def test_gemm_matches_dequant_matmul_oracle(lib, m, n, k):
    from test_speed_scalesweep_b200.gemm import cutlass_scaled_fp4_mm
    _, gsi_a, qa, sa = _quantized(m, k, 1 + m, 1.0, "scalesweep_mse")
    _, gsi_b, qb, sb = _quantized(n, k, 2 + n, 0.02, "rtn")
    alpha = (1.0 / (gsi_a * gsi_b)).reshape(1).float()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = cutlass_scaled_fp4_mm(qa, qb, sa, sb, alpha, torch.bfloat16, status=status)
    torch.cuda.synchronize()
    assert status.item() == 0
    ref = oracle.gemm(qa.cpu().numpy(), sa.view(torch.uint8).cpu().numpy(), qb.cpu().numpy(),
                      sb.view(torch.uint8).cpu().numpy(), m, n, k, alpha.item())
    err = _rel_fro(out.float().cpu().numpy(), ref)
    assert err <= TOL, err


# The tile choices between one and four M tiles: 64-wide tiles over two M
# tiles (256 and 160 rows at N=4096), 128 x 256 tiles for one M tile of any
# rows (full and trimmed A boxes at N=28672, down to 16 rows), 4 or 2
# cluster splits over two and four M tiles at K=14336, and 4 splits of a
# 1-row tile at N=6144.
@pytest.mark.parametrize("m,n,k", [(16, 6144, 4096), (128, 4096, 4096), (1024, 4096, 14336),
                                   (8192, 4096, 4096), (256, 4096, 4096), (160, 4096, 4096),
                                   (128, 28672, 4096), (96, 28672, 4096), (256, 4096, 14336),
                                   (512, 4096, 14336), (16, 28672, 4096), (1, 6144, 4096)])
def test_gemm_matches_vllm_cutlass_fp4_gemm(lib, m, n, k):
    vops = pytest.importorskip("vllm._custom_ops")
    if not hasattr(torch.ops, "_C") or not hasattr(torch.ops._C, "cutlass_scaled_fp4_mm"):
        pytest.skip("vLLM compiled CUTLASS FP4 GEMM not available")
    from test_speed_scalesweep_b200.gemm import cutlass_scaled_fp4_mm
    _, gsi_a, qa, sa = _quantized(m, k, 11, 1.0, "scalesweep_mse")
    _, gsi_b, qb, sb = _quantized(n, k, 12, 0.02, "rtn")
    alpha = (1.0 / (gsi_a * gsi_b)).reshape(1).float()
    ours = cutlass_scaled_fp4_mm(qa, qb, sa, sb, alpha, torch.bfloat16)
    ref = vops.cutlass_scaled_fp4_mm(qa, qb, sa, sb, alpha, torch.bfloat16)
    torch.cuda.synchronize()
    err = _rel_fro(ours.float().cpu().numpy(), ref.float().cpu().numpy().astype(np.float64))
    assert err <= TOL, err


# cluster split-K (partials reduced in distributed shared memory): 4 splits,
# 8 splits of one tile, 8 splits over two M tiles (the second 72 rows), 4
# splits of a full 128-row tile; global-memory split-K: 10 splits at K=20480
@pytest.mark.parametrize("m,n,k", [(16, 4096, 14336), (1, 128, 8192), (200, 384, 14336),
                                   (128, 4096, 14336), (16, 1024, 20480)])
def test_split_k_agrees_with_single_pass(lib, m, n, k):
    from test_speed_scalesweep_b200.gemm import cutlass_scaled_fp4_mm
    assert lib.ssw_nvfp4_gemm_workspace_bytes(m, n, k) > 0  # these shapes are split
    _, gsi_a, qa, sa = _quantized(m, k, 21, 1.0, "scalesweep_mse")
    _, gsi_b, qb, sb = _quantized(n, k, 22, 0.02, "rtn")
    alpha = (1.0 / (gsi_a * gsi_b)).reshape(1).float()
    split = cutlass_scaled_fp4_mm(qa, qb, sa, sb, alpha, split_k=True)
    split2 = cutlass_scaled_fp4_mm(qa, qb, sa, sb, alpha, split_k=True)
    single = cutlass_scaled_fp4_mm(qa, qb, sa, sb, alpha, split_k=False)
    torch.cuda.synchronize()
    assert torch.equal(split, split2)  # the split reduction order is fixed
    err = _rel_fro(split.float().cpu().numpy(), single.float().cpu().numpy().astype(np.float64))
    assert err <= TOL, err


# One-call quantize + GEMM (programmatic dependent launch): unsplit 64-wide
# decode tiles, cluster split-K, 128-wide tiles over two M tiles, the CTA-pair
# kernel, and the global-memory split (launched without the dependency).
@pytest.mark.parametrize("m,n,k", [(1, 4096, 4096), (16, 6144, 4096), (16, 4096, 14336),
                                   (200, 384, 1024), (2000, 2560, 512), (16, 1024, 20480)])
def test_quant_gemm_linear_equals_quantize_then_gemm(lib, m, n, k):
    from test_speed_scalesweep_b200.gemm import cutlass_scaled_fp4_mm, scalesweep_nvfp4_linear
    x, gsi_a, qa, sa = _quantized(m, k, 31 + m, 1.0, "scalesweep_mse")
    _, gsi_b, qb, sb = _quantized(n, k, 32 + n, 0.02, "rtn")
    alpha = (1.0 / (gsi_a * gsi_b)).reshape(1).float()
    scale_a = gsi_a.reshape(1).float()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ref = cutlass_scaled_fp4_mm(qa, qb, sa, sb, alpha)
    got = scalesweep_nvfp4_linear(x, scale_a, qb, sb, alpha, status=status)
    # back to back, so each dependent GEMM follows its own quantizer
    again = [scalesweep_nvfp4_linear(x, scale_a, qb, sb, alpha) for _ in range(3)]
    torch.cuda.synchronize()
    # the registered op (what the vLLM linear hook calls)
    from test_speed_scalesweep_b200 import ops  # noqa: F401
    via_op = torch.ops.scalesweep_b200.scalesweep_nvfp4_linear(x, scale_a, qb, sb, alpha)
    torch.cuda.synchronize()
    assert status.item() == 0
    assert torch.equal(got, ref)
    assert torch.equal(via_op, ref)
    for g in again:
        assert torch.equal(g, ref)


# The GEMM as a programmatic dependent of the kernel before it on the stream:
# right after the quantizer that writes A (unsplit 64-wide and wide tiles,
# cluster split-K), and after a kernel that does not signal early (a torch
# copy); the global-memory split launches without the dependency.
@pytest.mark.parametrize("m,n,k", [(16, 6144, 4096), (16, 28672, 4096), (16, 4096, 14336),
                                   (1, 128, 8192), (256, 4096, 4096), (16, 1024, 20480)])
def test_dependent_gemm_equals_plain_gemm(lib, m, n, k):
    from test_speed_scalesweep_b200 import custom
    from test_speed_scalesweep_b200.gemm import cutlass_scaled_fp4_mm
    x, gsi_a, qa, sa = _quantized(m, k, 51 + m, 1.0, "scalesweep_mse")
    _, gsi_b, qb, sb = _quantized(n, k, 52 + n, 0.02, "rtn")
    alpha = (1.0 / (gsi_a * gsi_b)).reshape(1).float()
    ref = cutlass_scaled_fp4_mm(qa, qb, sa, sb, alpha)
    outs = []
    for _ in range(3):
        ca, csa = custom.nvfp4_quant(x, gsi_a, True, "scalesweep_mse")
        outs.append(cutlass_scaled_fp4_mm(ca, qb, csa, sb, alpha, dependent_launch=True))
    a_copy = qa.clone()
    outs.append(cutlass_scaled_fp4_mm(a_copy, qb, sa, sb, alpha, dependent_launch=True))
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o, ref)


def test_mma_rate_probe_reports_every_sm(lib):
    """The dense FP4 rate probe (the measured peak GEMM fractions use): every
    SM's CTA finishes its MMAs within the bounded wait, at a per-cycle rate
    near the tensor pipe's 32768 FP4 FLOPs per SM cycle."""
    import ctypes
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    cycles = torch.zeros(sms, dtype=torch.int64, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for bn in (128, 256):
        st = lib.ssw_nvfp4_mma_rate_probe(bn, 256, ctypes.c_void_p(cycles.data_ptr()),
                                          ctypes.c_void_p(status.data_ptr()), None)
        assert st == 0
        torch.cuda.synchronize()
        assert status.item() == 0 and int(cycles.min().item()) > 0
        per_cycle = 2.0 * 128 * bn * 64 * 4 * 256 / float(cycles.median().item())
        assert 8000 < per_cycle < 70000, per_cycle
    assert lib.ssw_nvfp4_mma_rate_probe(64, 256, ctypes.c_void_p(cycles.data_ptr()), None,
                                        None) != 0
