"""GPU parity against the reference's own Triton kernels, run on the same GPU.

The reference's quantizer modules (bench_kernel/scalesweep_mse_nvfp4_utils.py,
bench_kernel/scalesweep_mse_reference_nvfp4_utils.py and
bench_kernel/scalesweep_nvfp4_utils.py) are installed unmodified under
baseline/_ref by baseline/install_ref.py.  Each test runs a reference kernel
through its public ``*_quant_out`` function and the matching CUDA entry point
through the C ABI on identical seeded inputs, both into sentinel-filled
buffers, and compares every byte: codes, written scale bytes, and the padding
neither kernel may touch.

  K1  scalesweep_mse_nvfp4_quant_out            (:462-477)  <->  mse
  K1  scalesweep_mse128_nvfp4_quant_out         (:480-495)  <->  mse128
  K2  reference scalesweep_mse_nvfp4_quant_out  (:412-445)  <->  reference
  K3  scalesweep_nvfp4_quant_out / 128 variant              <->  weighted / weighted128

Skipped when baseline/_ref is absent (it is not part of the repository).
"""
import ctypes
import os
import sys

import numpy as np
import pytest
import torch

import golden_inputs as gi
import oracle

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.path.join(ROOT, "baseline", "_ref")
SENTINEL = 0xA5

ENTRY = {"mse": "ssw_scalesweep_mse_nvfp4_quant_out",
         "mse128": "ssw_scalesweep_mse128_nvfp4_quant_out",
         "reference": "ssw_scalesweep_mse_reference_nvfp4_quant_out",
         "weighted": "ssw_scalesweep_nvfp4_quant_out",
         "weighted128": "ssw_scalesweep128_nvfp4_quant_out"}


@pytest.fixture(scope="module")
def ref():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    if not os.path.isdir(os.path.join(REF_DIR, "bench_kernel")):
        pytest.skip("the reference is not installed under baseline/_ref "
                    "(python baseline/install_ref.py)")
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    from bench_kernel import scalesweep_mse_nvfp4_utils as k1
    from bench_kernel import scalesweep_mse_reference_nvfp4_utils as k2
    from bench_kernel import scalesweep_nvfp4_utils as k3
    return {"mse": k1.scalesweep_mse_nvfp4_quant_out,
            "mse128": k1.scalesweep_mse128_nvfp4_quant_out,
            "reference": k2.scalesweep_mse_nvfp4_quant_out,
            "weighted": k3.scalesweep_nvfp4_quant_out,
            "weighted128": k3.scalesweep128_nvfp4_quant_out}


@pytest.fixture(scope="module")
def lib(built_library):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from test_speed_scalesweep_b200 import _lib
    return _lib.lib()


def _buffers(m, pn, swizzled):
    codes = torch.full((m, pn // 2), SENTINEL, dtype=torch.uint8, device="cuda")
    scales = torch.full(oracle.scale_shape(m, pn, swizzled), SENTINEL, dtype=torch.uint8,
                        device="cuda")
    return codes, scales


def run_ref(ref, kind, x, gsi, pn, swizzled):
    m = x.shape[0]
    codes, scales = _buffers(m, pn, swizzled)
    ref[kind](x, gsi, swizzled, output=codes, output_scale=scales)
    torch.cuda.synchronize()
    return codes.cpu().numpy(), scales.cpu().numpy()


def run_ours(lib, kind, x, gsi, pn, swizzled):
    m, n = x.shape
    codes, scales = _buffers(m, pn, swizzled)
    st = getattr(lib, ENTRY[kind])(
        ctypes.c_void_p(x.data_ptr()), 0 if x.dtype == torch.bfloat16 else 1, m, n, pn,
        ctypes.c_void_p(gsi.data_ptr()), ctypes.c_void_p(codes.data_ptr()),
        ctypes.c_void_p(scales.data_ptr()), int(swizzled),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0, lib.ssw_last_error()
    torch.cuda.synchronize()
    return codes.cpu().numpy(), scales.cpu().numpy()


def to_device(bits, dtype="bf16"):
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).cuda()
    return t.view(torch.bfloat16 if dtype == "bf16" else torch.float16)


def check(ref, lib, kind, bits, gsi, *, dtype="bf16", padded_n=None, swizzled=True):
    x = to_device(bits, dtype)
    g = torch.tensor([gsi], dtype=torch.float32, device="cuda")
    pn = padded_n or x.shape[1]
    rc, rs = run_ref(ref, kind, x, g, pn, swizzled)
    oc, os_ = run_ours(lib, kind, x, g, pn, swizzled)
    bad = np.flatnonzero(rc.ravel() != oc.ravel())
    assert bad.size == 0, f"{kind}: {bad.size} code bytes differ, first at {bad[:4]}"
    bad = np.flatnonzero(rs.ravel() != os_.ravel())
    assert bad.size == 0, f"{kind}: {bad.size} scale bytes differ, first at {bad[:4]}"


def test_config1_both_conventions(ref, lib):
    """Config 1: bf16 [128, 4096], 0.5% outlier columns, gsi from 448 and 256."""
    bits = gi.outlier_activations(128, 4096, seed=1)
    for fp8_max in (448.0, 256.0):
        gsi = gi.torch_style_gsi(bits, fp8_max)
        for kind in ("mse", "reference", "mse128", "weighted", "weighted128"):
            check(ref, lib, kind, bits, gsi)


CONFIG2 = [(m, k) for k in (4096, 8192, 14336) for m in (1, 16, 64, 256, 1024)]


@pytest.mark.parametrize("m,k", CONFIG2)
@pytest.mark.parametrize("kind", ["mse", "reference"])
def test_config2_shapes(ref, lib, kind, m, k):
    bits = gi.outlier_activations(m, k, seed=2000 + m + k)
    check(ref, lib, kind, bits, gi.torch_style_gsi(bits, 448.0))


@pytest.mark.parametrize("case", gi.CASES, ids=lambda c: c["name"])
def test_golden_edge_cases(ref, lib, case):
    """The golden-vector cases (ragged, padded_n, fp16, ties, NaN/Inf,
    saturation, wide-range) on every variant each case lists."""
    bits = gi.make_input(case)
    gsi = gi.make_gsi(case, bits)
    dtype = case.get("dtype", "bf16")
    for variant in case["variants"]:
        kind, layout = variant.rsplit("_", 1)
        check(ref, lib, kind, bits, gsi, dtype=dtype, padded_n=case.get("padded_n"),
              swizzled=(layout == "swz"))


def test_wide_range_and_unaligned_rows(ref, lib):
    """Per-row magnitudes e^[-8, 8] (both window ends and the E4M3 subnormal
    scales), rows that end mid-scale-word, and the linear scale layout."""
    bits = gi.wide_range_activations(300, 16 * 37, seed=77)
    gsi = gi.torch_style_gsi(bits, 448.0)
    for kind in ("mse", "reference", "weighted"):
        for swz in (True, False):
            check(ref, lib, kind, bits, gsi, swizzled=swz)
