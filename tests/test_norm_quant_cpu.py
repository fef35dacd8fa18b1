"""CPU tests of the RMSNorm-fused quantizer: the oracle's restatement of
vLLM's RMSNorm reduction, and the argument checks of the C ABI and the
Python API (no GPU needed; nothing is launched)."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from test_speed_scalesweep_b200 import _lib, norm_quant


def bf16_bits(a):
    return (np.asarray(a, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def bf16_vals(bits):
    return (bits.astype(np.uint32) << 16).view(np.float32)


@pytest.mark.parametrize("m", [3, 256])
def test_oracle_sum_of_squares_is_close_to_exact(m):
    rng = np.random.default_rng(m)
    bits = bf16_bits(rng.standard_normal((m, 1024)) * 5)
    acc, res = oracle.rms_sumsq(bits)
    assert res is None
    exact = (bf16_vals(bits).astype(np.float64) ** 2).sum(1)
    assert np.allclose(acc, exact, rtol=1e-5)


def test_oracle_order_depends_on_the_block_size_switch():
    """vLLM's block is 1024 threads below 256 rows and 256 from there; the
    same row summed in the two orders differs in the last bits for some rows
    and the oracle follows the row count."""
    rng = np.random.default_rng(5)
    row = bf16_bits(rng.standard_normal((1, 14336)) * np.logspace(-3, 3, 14336))
    small, _ = oracle.rms_sumsq(np.repeat(row, 255, axis=0))
    large, _ = oracle.rms_sumsq(np.repeat(row, 256, axis=0))
    assert len(set(small.tolist())) == 1 and len(set(large.tolist())) == 1
    assert np.isclose(small[0], large[0], rtol=1e-5)


def test_oracle_fused_add_rounds_the_sum_to_bf16_and_returns_it():
    rng = np.random.default_rng(9)
    x = bf16_bits(rng.standard_normal((4, 512)))
    r = bf16_bits(rng.standard_normal((4, 512)) * 3)
    acc, res = oracle.rms_sumsq(x, r)
    z = bf16_vals(x) + bf16_vals(r)  # binary32 sums
    zb = bf16_bits(torch.from_numpy(z).to(torch.bfloat16).float().numpy())
    assert np.array_equal(res, zb)
    plain, _ = oracle.rms_sumsq(res)
    assert np.allclose(acc, plain, rtol=1e-6)


def test_oracle_apply_rounds_each_product():
    x = bf16_bits([[1.5, -3.0, 0.0, 7.0] * 4])
    w = bf16_bits([0.5, 2.0, 1.0, -1.0] * 4)
    out = oracle.rms_apply(x, w, np.array([0.25], np.float32))
    assert np.array_equal(bf16_vals(out)[0, :4], np.float32([0.1875, -1.5, 0.0, -1.75]))


def test_rsqrt_bound_is_the_float64_reciprocal_root():
    acc = np.float32([4096.0, 1e-30])
    b = oracle.rms_rsqrt_bound(acc, 4096, 1e-5)
    assert np.isclose(b[0], 1.0 / np.sqrt(np.float64(np.float32(1.0) + np.float32(1e-5))))
    assert np.isclose(b[1], 1.0 / np.sqrt(np.float64(np.float32(1e-5))))


def _p(v):
    return ctypes.c_void_p(v) if v else None  # never dereferenced


@pytest.mark.parametrize("kwargs,needle", [
    (dict(n=40), "multiple of 16"),
    (dict(m=-1), "bad sizes"),
    (dict(w=0), "null"),
    (dict(ws=0), "null"),
    (dict(inp=0x1010), "aligned"),
    (dict(res=0x2008), "aligned"),
    (dict(m=1 << 31), "below 2^31"),
    (dict(m=1 << 20, n=1 << 16), "blocks below 2^32"),
])
def test_abi_rejects_bad_arguments_before_any_launch(built_library, kwargs, needle):
    h = _lib.lib()
    a = dict(inp=0x1000, res=0, w=0x3000, m=4, n=64, scale=0x4000, out=0x5000, osc=0x6000,
             ws=0x7000)
    a.update(kwargs)
    st = h.ssw_rms_norm_scalesweep_mse_nvfp4_quant_out(
        _p(a["inp"]), _p(a["res"]), _p(a["w"]), 1e-5, a["m"], a["n"], _p(a["scale"]),
        _p(a["out"]), _p(a["osc"]), 1, _p(a["ws"]), None)
    assert st == _lib.SSW_ERR_INVALID_ARGUMENT
    assert needle in h.ssw_last_error().decode()


def test_abi_zero_rows_is_a_no_op(built_library):
    h = _lib.lib()
    assert h.ssw_rms_norm_scalesweep_mse_nvfp4_quant_out(
        None, None, None, 1e-5, 0, 64, None, None, None, 1, None, None) == _lib.SSW_OK


def test_python_api_checks_arguments_before_any_launch():
    x = torch.zeros(4, 64, dtype=torch.bfloat16)
    w = torch.ones(64, dtype=torch.bfloat16)
    gsi = torch.ones(1)
    with pytest.raises(ValueError, match="CUDA"):
        norm_quant.rms_norm_scalesweep_mse_nvfp4_quant(x, w, 1e-5, gsi)
    with pytest.raises(ValueError, match="bf16"):
        norm_quant.rms_norm_scalesweep_mse_nvfp4_quant(x.half(), w, 1e-5, gsi)
    with pytest.raises(ValueError, match="multiple of 16"):
        norm_quant.rms_norm_scalesweep_mse_nvfp4_quant(torch.zeros(4, 40, dtype=torch.bfloat16),
                                                       w[:40], 1e-5, gsi)
    with pytest.raises(ValueError, match="weight"):
        norm_quant.rms_norm_scalesweep_mse_nvfp4_quant(x, w[:32], 1e-5, gsi)
    with pytest.raises(ValueError, match="residual"):
        norm_quant.rms_norm_scalesweep_mse_nvfp4_quant(x, w, 1e-5, gsi, residual=x[:2])
    codes, scales = norm_quant.alloc_outputs(torch.empty(3, 80, dtype=torch.bfloat16,
                                                         device="meta"))
    assert codes.shape == (3, 40) and scales.shape == (128, 8)


def test_ops_are_registered():
    from test_speed_scalesweep_b200 import ops  # noqa: F401
    for name in ("rms_norm_scalesweep_mse_nvfp4_quant", "rms_norm_nvfp4_quant",
                 "fused_add_rms_norm_nvfp4_quant"):
        assert hasattr(torch.ops.scalesweep_b200, name)
