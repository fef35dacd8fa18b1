"""SiLU-and-mul and the fused SiLU-and-mul quantizer, without a GPU: the
oracle's SiLU pinned to vLLM's silu_and_mul on every bf16 and f16 gate value
(tests/golden/silu_golden.npz, made by tests/golden/make_silu_golden.py), and
argument checks of the C ABI and the Python API."""
import ctypes
import os

import numpy as np
import pytest
import torch

import oracle
from test_speed_scalesweep_b200 import _lib, act_quant

HERE = os.path.dirname(os.path.abspath(__file__))
ONE = {"bf16": 0x3F80, "f16": 0x3C00}


def _is_nan(bits, dtype):
    if dtype == "bf16":
        return ((bits & 0x7F80) == 0x7F80) & ((bits & 0x7F) != 0)
    return ((bits & 0x7C00) == 0x7C00) & ((bits & 0x3FF) != 0)


@pytest.fixture(scope="module")
def silu_golden():
    return np.load(os.path.join(HERE, "golden", "silu_golden.npz"))


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_oracle_silu_matches_vllm_on_every_gate_value(silu_golden, dtype):
    gate = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    x = np.concatenate([gate.reshape(1, -1), np.full((1, 65536), ONE[dtype], np.uint16)], axis=1)
    got = oracle.silu_mul(x, dtype).reshape(-1)
    want = silu_golden[dtype]
    same = (got == want) | (_is_nan(got, dtype) & _is_nan(want, dtype))
    assert same.all(), np.nonzero(~same)[0][:8]
    assert bool(silu_golden["torch_equals_vllm"].all())


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_oracle_product_is_rounded_once(dtype):
    # bf16(1.5) * bf16(1.5) = 2.25 exactly; the f16 pair 1.0009765625^2 needs a
    # rounding of the exact product (1 + 2^-9 + 2^-20 -> 1 + 2^-9)
    t = {"bf16": torch.bfloat16, "f16": torch.float16}[dtype]
    gate = torch.tensor([40.0, 40.0], dtype=t)        # silu(40) rounds to 40
    up = torch.tensor([1.5, 1.0009765625], dtype=t)
    x = torch.cat([gate, up]).view(torch.int16).numpy().view(np.uint16).reshape(1, 4)
    got = oracle.silu_mul(x, dtype).view({"bf16": np.uint16, "f16": np.float16}[dtype])
    want = (torch.tensor([40.0, 40.0], dtype=torch.float64) * up.double()).to(t)
    assert np.array_equal(got.reshape(-1).view(np.uint16),
                          want.view(torch.int16).numpy().view(np.uint16))


def test_oracle_fused_is_quantize_of_silu_mul():
    rng = np.random.default_rng(3)
    x = torch.from_numpy(rng.standard_normal((5, 128)).astype(np.float32)).to(torch.bfloat16)
    bits = x.view(torch.int16).numpy().view(np.uint16)
    c1, s1 = oracle.silu_mul_quantize(bits, 448.0 * 6 / 4.0)
    c2, s2 = oracle.quantize(oracle.silu_mul(bits), 448.0 * 6 / 4.0)
    assert np.array_equal(c1, c2) and np.array_equal(s1, s2)


def _ptr(v):
    return ctypes.c_void_p(0x1000 * v) if v else None  # never dereferenced


@pytest.mark.parametrize("kwargs,needle", [
    (dict(dtype=5), "dtype"),
    (dict(n=40), "multiple of 16"),
    (dict(m=-1), "negative"),
    (dict(out=0), "null"),
    (dict(inp=3), "aligned"),
])
def test_silu_and_mul_rejects_bad_arguments_without_a_gpu(built_library, kwargs, needle):
    h = _lib.lib()
    a = dict(dtype=0, m=4, n=64, inp=32, out=32)
    a.update(kwargs)
    inp = ctypes.c_void_p(a["inp"]) if a["inp"] else None
    st = h.ssw_silu_and_mul(inp, a["dtype"], a["m"], a["n"], _ptr(a["out"]), None)
    assert st == _lib.SSW_ERR_INVALID_ARGUMENT
    assert needle in h.ssw_last_error().decode()


@pytest.mark.parametrize("kwargs,needle", [
    (dict(dtype=5), "dtype"),
    (dict(n=40), "multiple of 16"),
    (dict(scale=0), "null"),
    (dict(inp=3), "aligned"),
])
def test_fused_quant_rejects_bad_arguments_without_a_gpu(built_library, kwargs, needle):
    h = _lib.lib()
    a = dict(dtype=0, m=4, n=64, inp=32, scale=1, out=1, osc=1)
    a.update(kwargs)
    inp = ctypes.c_void_p(a["inp"]) if a["inp"] else None
    st = h.ssw_silu_and_mul_scalesweep_mse_nvfp4_quant_out(inp, a["dtype"], a["m"], a["n"],
                                                           _ptr(a["scale"]), _ptr(a["out"]),
                                                           _ptr(a["osc"]), 1, None)
    assert st == _lib.SSW_ERR_INVALID_ARGUMENT
    assert needle in h.ssw_last_error().decode()


def test_python_api_checks_arguments_before_any_launch():
    x = torch.zeros(4, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        act_quant.silu_and_mul(x)
    with pytest.raises(ValueError, match="multiple of 16"):
        act_quant.silu_and_mul(torch.zeros(4, 40, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="bf16 or f16"):
        act_quant.silu_and_mul(torch.zeros(4, 64, dtype=torch.float32))
    codes, scales = act_quant.alloc_outputs(torch.empty(3, 2 * 80, dtype=torch.bfloat16,
                                                        device="meta"))
    assert codes.shape == (3, 40) and scales.shape == (128, 8)
