"""Host-side behaviour of the Python API that needs no GPU: dispatcher errors,
shape functions, allocation shapes, op registration."""
import pytest
import torch

from test_speed_scalesweep_b200 import custom, ops  # noqa: F401
from test_speed_scalesweep_b200 import scalesweep_mse_nvfp4_utils as mse
from test_speed_scalesweep_b200 import scalesweep_mse_reference_nvfp4_utils as mse_ref


def test_dispatcher_errors_match_reference():
    s = torch.ones(1)
    with pytest.raises(ValueError, match="at least one dimension"):
        custom.nvfp4_quant(torch.tensor(1.0), s)
    with pytest.raises(ValueError, match="multiple of 16"):
        custom.nvfp4_quant(torch.zeros(2, 24, dtype=torch.bfloat16), s)
    with pytest.raises(ValueError, match="Unsupported backend"):
        custom.nvfp4_quant(torch.zeros(2, 32, dtype=torch.bfloat16), s, backend="nope")


def test_cpu_tensors_are_rejected_not_emulated():
    x = torch.zeros(2, 32, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        custom.nvfp4_quant(x, torch.ones(1))


def test_reference_variant_rejects_padded_n():
    x = torch.zeros(2, 32, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="padded_n"):
        mse_ref.scalesweep_mse_nvfp4_quant_impl(x, torch.ones(1), True, padded_n=64)
    with pytest.raises(ValueError, match="padded_n"):
        mse_ref._scalesweep_mse_reference_nvfp4_quant_fake(x, torch.ones(1), True, 64)


@pytest.mark.parametrize("m,n,padded,swz", [(1, 64, None, True), (129, 80, None, True),
                                             (33, 64, 96, True), (5, 32, None, False)])
def test_allocation_shapes(m, n, padded, swz):
    out, sc = custom.create_fp4_output_tensors(m, n, torch.device("cpu"), swz, padded_n=padded)
    pn = padded or n
    assert out.shape == (m, pn // 2) and out.dtype == torch.uint8
    if swz:
        assert sc.shape == ((m + 127) // 128 * 128, ((pn // 16 + 3) // 4 * 4) // 4)
        assert sc.dtype == torch.int32
    else:
        assert sc.shape == (m, pn // 16) and sc.dtype == torch.uint8
    fo, fs = mse._scalesweep_mse_nvfp4_quant_fake(torch.empty(m, n, dtype=torch.bfloat16),
                                                  torch.ones(1), swz, padded)
    assert fo.shape == out.shape and fs.dtype == torch.float8_e4m3fn
    assert fs.numel() == sc.numel() * sc.element_size()


def test_vllm_allocation_helper_agrees():
    vops = pytest.importorskip("vllm._custom_ops")
    for m, n, pn, swz in [(7, 64, None, True), (200, 4096, None, True), (3, 64, 96, False)]:
        a = custom.create_fp4_output_tensors(m, n, torch.device("cpu"), swz, padded_n=pn)
        b = vops.create_fp4_output_tensors(m, n, torch.device("cpu"), swz, padded_n=pn)
        for x, y in zip(a, b):
            assert x.shape == y.shape and x.dtype == y.dtype


def test_ops_registered_with_fake_shapes():
    x = torch.empty(300, 4096, dtype=torch.bfloat16, device="meta")
    s = torch.empty(1, dtype=torch.float32, device="meta")
    for name in ("scalesweep_mse_nvfp4_quant", "scalesweep_mse128_nvfp4_quant",
                 "scalesweep_mse_reference_nvfp4_quant", "rtn_nvfp4_quant",
                 "scalesweep_nvfp4_quant", "scalesweep128_nvfp4_quant"):
        op = getattr(torch.ops.scalesweep_b200, name)
        c, sc = op(x, s, True)
        assert c.shape == (300, 2048) and sc.shape == (384, 256)
        assert sc.dtype == torch.float8_e4m3fn
        assert hasattr(op, "out")


def test_reference_constants():
    assert (mse.BLOCK_SIZE, mse.LOWER_BOUND, mse.UPPER_BOUND) == (16, -3, 7)
    assert (mse.FP4_E2M1_MAX, mse.REF_MAX_SCALE_RAW) == (6.0, 126)
