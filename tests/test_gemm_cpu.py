"""The NVFP4 GEMM entry points without a GPU: the C ABI rejects bad shapes,
null and misaligned pointers before any device call, and the Python
wrappers reject tensors they cannot hand to the kernels."""
import ctypes

import pytest
import torch

from test_speed_scalesweep_b200 import _lib
from test_speed_scalesweep_b200.gemm import cutlass_scaled_fp4_mm, scalesweep_nvfp4_linear


def _p(v):
    return ctypes.c_void_p(v) if v else None  # never dereferenced


def _gemm(h, m=16, n=128, k=256, a=0x1000, out=0x1000, ws=None):
    return h.ssw_nvfp4_gemm(_p(a), _p(0x1000), _p(0x1000), _p(0x1000), _p(0x1000), _p(out),
                            m, n, k, _p(ws), 0, None, None)


def _quant_gemm(h, m=16, n=128, k=256, x=0x1000, dtype=0):
    return h.ssw_nvfp4_quant_gemm(_p(x), dtype, _p(0x1000), _p(0x1000), _p(0x1000),
                                  _p(0x1000), _p(0x1000), m, n, k, _p(0x1000), 1 << 20, None,
                                  None)


@pytest.mark.parametrize("kwargs,status,needle", [
    (dict(k=300), _lib.SSW_ERR_UNSUPPORTED, "multiple of 256"),
    (dict(n=100), _lib.SSW_ERR_UNSUPPORTED, "multiple of 64"),
    (dict(m=-1), _lib.SSW_ERR_INVALID_ARGUMENT, "bad sizes"),
    (dict(m=1 << 31), _lib.SSW_ERR_INVALID_ARGUMENT, "below 2^31"),
    (dict(a=0), _lib.SSW_ERR_INVALID_ARGUMENT, "null"),
    (dict(out=0x1008), _lib.SSW_ERR_INVALID_ARGUMENT, "16-byte aligned"),
])
def test_gemm_rejects_bad_arguments_without_a_gpu(built_library, kwargs, status, needle):
    h = _lib.lib()
    assert _gemm(h, **kwargs) == status
    assert needle in h.ssw_last_error().decode()


@pytest.mark.parametrize("kwargs,status,needle", [
    (dict(k=300), _lib.SSW_ERR_UNSUPPORTED, "multiple of 256"),
    (dict(n=100), _lib.SSW_ERR_UNSUPPORTED, "multiple of 64"),
    (dict(m=-1), _lib.SSW_ERR_INVALID_ARGUMENT, "bad sizes"),
])
def test_quant_gemm_rejects_bad_shapes_without_a_gpu(built_library, kwargs, status, needle):
    h = _lib.lib()
    assert _quant_gemm(h, **kwargs) == status
    assert "nvfp4_quant_gemm" in h.ssw_last_error().decode()
    assert needle in h.ssw_last_error().decode()


def test_empty_m_is_a_no_op(built_library):
    h = _lib.lib()
    assert _gemm(h, m=0) == _lib.SSW_OK
    assert _quant_gemm(h, m=0) == _lib.SSW_OK


def test_workspace_query_is_zero_for_unsupported_shapes(built_library):
    h = _lib.lib()
    assert h.ssw_nvfp4_gemm_workspace_bytes(16, 100, 256) == 0
    assert h.ssw_nvfp4_quant_gemm_workspace_bytes(16, 128, 300) == 0


def test_python_wrappers_reject_cpu_tensors_and_other_outputs():
    a = torch.zeros(16, 128, dtype=torch.uint8)
    b = torch.zeros(128, 128, dtype=torch.uint8)
    s = torch.zeros(128, 16, dtype=torch.uint8)
    alpha = torch.ones(1)
    with pytest.raises(ValueError, match="CUDA"):
        cutlass_scaled_fp4_mm(a, b, s, s, alpha)
    with pytest.raises(ValueError, match="bf16"):
        cutlass_scaled_fp4_mm(a, b, s, s, alpha, out_dtype=torch.float16)
    x = torch.zeros(16, 256, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        scalesweep_nvfp4_linear(x, torch.ones(1), b, s, alpha)
    with pytest.raises(ValueError, match="bf16 or f16"):
        scalesweep_nvfp4_linear(x.float(), torch.ones(1), b, s, alpha)


def test_linear_op_traces_with_its_fake_shape():
    from test_speed_scalesweep_b200 import ops  # noqa: F401
    x = torch.empty(3, 5, 4096, dtype=torch.bfloat16, device="meta")
    w = torch.empty(6144, 2048, dtype=torch.uint8, device="meta")
    ws = torch.empty(6144, 256, dtype=torch.float8_e4m3fn, device="meta")
    one = torch.empty(1, device="meta")
    out = torch.ops.scalesweep_b200.scalesweep_nvfp4_linear(x, one, w, ws, one)
    assert out.shape == (3, 5, 6144) and out.dtype == torch.bfloat16
