"""GPU parity: the sm_100a kernels (through the C ABI) against the golden
vectors of the reference's own kernels and against the CPU oracle.  Integer /
byte outputs, so the bar is bit-exact everywhere."""
import ctypes
import hashlib

import numpy as np
import pytest
import torch

import golden_inputs as gi
import oracle

pytestmark = pytest.mark.gpu

SENTINEL = 0xA5


@pytest.fixture(scope="module")
def lib(built_library):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from test_speed_scalesweep_b200 import _lib
    return _lib.lib()


ENTRY = {"mse": "ssw_scalesweep_mse_nvfp4_quant_out",
         "mse128": "ssw_scalesweep_mse128_nvfp4_quant_out",
         "reference": "ssw_scalesweep_mse_reference_nvfp4_quant_out",
         "rtn": "ssw_rtn_nvfp4_quant_out",
         "weighted": "ssw_scalesweep_nvfp4_quant_out",
         "weighted128": "ssw_scalesweep128_nvfp4_quant_out"}


def to_device(bits, dtype="bf16"):
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).cuda()
    return t.view(torch.bfloat16 if dtype == "bf16" else torch.float16)


def c_quant(lib, kind, x, gsi, *, padded_n=None, swizzled=True, input_offset_elems=0):
    """Call the C ABI directly with sentinel-filled output buffers."""
    m, n = x.shape
    pn = padded_n or n
    if input_offset_elems:
        buf = torch.empty(m * n + input_offset_elems, dtype=x.dtype, device=x.device)
        view = buf[input_offset_elems:].view(m, n)
        view.copy_(x)
        x = view
    codes = torch.full((m, pn // 2), SENTINEL, dtype=torch.uint8, device="cuda")
    shape = oracle.scale_shape(m, pn, swizzled)
    scales = torch.full(shape, SENTINEL, dtype=torch.uint8, device="cuda")
    g = torch.tensor([gsi], dtype=torch.float32, device="cuda")
    fn = getattr(lib, ENTRY[kind])
    st = fn(ctypes.c_void_p(x.data_ptr()), 0 if x.dtype == torch.bfloat16 else 1, m, n, pn,
            ctypes.c_void_p(g.data_ptr()), ctypes.c_void_p(codes.data_ptr()),
            ctypes.c_void_p(scales.data_ptr()), int(swizzled),
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0, lib.ssw_last_error()
    torch.cuda.synchronize()
    return codes.cpu().numpy(), scales.cpu().numpy()


def _kind(variant):
    kind, layout = variant.rsplit("_", 1)
    return kind, layout == "swz"


GOLDEN_CASES = [(c["name"], v) for c in gi.CASES for v in c["variants"]]


@pytest.mark.parametrize("name,variant", GOLDEN_CASES)
def test_kernel_matches_reference_golden(lib, golden, name, variant):
    case = next(c for c in gi.CASES if c["name"] == name)
    dtype = case.get("dtype", "bf16")
    x = to_device(golden[f"{name}/input"], dtype)
    gsi = float(golden[f"{name}/gsi"][0])
    kind, swz = _kind(variant)
    codes, scales = c_quant(lib, kind, x, gsi, padded_n=case.get("padded_n"), swizzled=swz)
    np.testing.assert_array_equal(codes, golden[f"{name}/{variant}/codes"])
    # written scale bytes match; padding the kernel must not touch keeps the sentinel
    np.testing.assert_array_equal(scales, golden[f"{name}/{variant}/scales"])


@pytest.mark.parametrize("case", gi.CHECKSUM_CASES, ids=lambda c: c["name"])
def test_kernel_full_config1_checksums(lib, golden, case):
    x = gi.make_input(case)
    gsi = gi.make_gsi(case, x)
    xd = to_device(x)
    for variant in case["variants"]:
        kind, _ = _kind(variant)
        codes, scales = c_quant(lib, kind, xd, gsi)
        h = hashlib.sha256(codes.tobytes() + scales.tobytes()).digest()
        assert h == golden[f"{case['name']}/{variant}/sha256"].tobytes(), variant


SWEEP = [(m, k) for k in (4096, 8192, 14336) for m in (1, 16, 64, 256, 1024)]


@pytest.mark.parametrize("m,k", SWEEP)
@pytest.mark.parametrize("kind", ["mse", "reference", "rtn", "weighted"])
def test_kernel_matches_oracle_config2_shapes(lib, m, k, kind):
    x = gi.outlier_activations(m, k, seed=1000 + m + k)
    gsi = gi.torch_style_gsi(x, 448.0 if kind != "mse" else 256.0)
    codes, scales = c_quant(lib, kind, to_device(x), gsi)
    var = kind if kind in ("reference", "weighted") else "mse"
    mode = "rtn" if kind == "rtn" else "window"
    oc, os_ = oracle.quantize(x, gsi, variant=var, mode=mode)
    np.testing.assert_array_equal(codes, oc)
    np.testing.assert_array_equal(scales, os_)


def _lane_sharing_shapes():
    """(m, k) pairs whose block count sits on each side of the 4-lane and 2-lane
    thresholds (blocks x lanes <= SMs x 256 threads), with k = 16 x 37 so rows
    end mid-scale-word (byte scale stores)."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count if \
        torch.cuda.is_available() else 148
    bpc = 37
    limit4, limit2 = sms * 256 // 4, sms * 256 // 2
    return [(limit4 // bpc, 16 * bpc), (limit4 // bpc + 1, 16 * bpc),
            (limit2 // bpc, 16 * bpc), (limit2 // bpc + 1, 16 * bpc), (3, 4096)]


@pytest.mark.parametrize("m,k", _lane_sharing_shapes())
@pytest.mark.parametrize("kind", ["mse", "reference", "weighted"])
@pytest.mark.parametrize("swz", [True, False])
def test_lane_shared_blocks_match_oracle(lib, m, k, kind, swz):
    # decode-sized inputs give each block 2 or 4 lanes that sweep disjoint
    # candidate subsets; wide-range values make exact ties and variant
    # differences likely
    x = gi.wide_range_activations(m, k, m + k)
    gsi = gi.torch_style_gsi(x, 448.0)
    codes, scales = c_quant(lib, kind, to_device(x), gsi, swizzled=swz)
    oc, os_ = oracle.quantize(x, gsi, variant=kind, swizzled=swz)
    np.testing.assert_array_equal(codes, oc)
    np.testing.assert_array_equal(scales, os_)


@pytest.mark.parametrize("m,k,seed", [(300, 1024, 1), (64, 2048, 2), (1, 64, 3)])
@pytest.mark.parametrize("kind", ["mse128", "weighted128"])
def test_full_range_mode_matches_oracle(lib, m, k, seed, kind):
    x = gi.wide_range_activations(m, k, seed)
    gsi = gi.torch_style_gsi(x, 448.0)
    codes, scales = c_quant(lib, kind, to_device(x), gsi)
    oc, os_ = oracle.quantize(x, gsi, mode="full_range",
                              variant="weighted" if kind == "weighted128" else "mse")
    np.testing.assert_array_equal(codes, oc)
    np.testing.assert_array_equal(scales, os_)


@pytest.mark.parametrize("kind", ["mse", "reference", "weighted"])
def test_wide_range_inputs_where_variants_differ(lib, kind):
    x = gi.wide_range_activations(512, 2048, 77)
    gsi = gi.torch_style_gsi(x, 448.0)
    codes, scales = c_quant(lib, kind, to_device(x), gsi, swizzled=False)
    oc, os_ = oracle.quantize(x, gsi, variant=kind, swizzled=False)
    np.testing.assert_array_equal(codes, oc)
    np.testing.assert_array_equal(scales, os_)


@pytest.mark.parametrize("m,n,pn,swz", [(129, 80, 80, True), (3, 48, 48, False), (130, 64, 112, True),
                                        (257, 32, 32, True), (7, 16, 64, False)])
def test_ragged_and_unaligned_shapes(lib, m, n, pn, swz):
    x = gi.outlier_activations(m, n, seed=m * 7 + n)
    gsi = gi.torch_style_gsi(x, 448.0)
    codes, scales = c_quant(lib, "mse", to_device(x), gsi, padded_n=pn, swizzled=swz)
    oc, os_ = oracle.quantize(x, gsi, padded_n=pn, swizzled=swz)
    np.testing.assert_array_equal(codes, oc)
    np.testing.assert_array_equal(scales, os_)


@pytest.mark.parametrize("offset", [1, 8])
def test_misaligned_input_pointer_uses_the_scalar_path(lib, offset):
    x = gi.outlier_activations(33, 256, seed=5)
    gsi = gi.torch_style_gsi(x, 448.0)
    codes, scales = c_quant(lib, "mse", to_device(x), gsi, input_offset_elems=offset)
    oc, os_ = oracle.quantize(x, gsi)
    np.testing.assert_array_equal(codes, oc)
    np.testing.assert_array_equal(scales, os_)


def test_fp16_input(lib):
    x = gi.outlier_activations(100, 1024, seed=11, dtype="f16")
    gsi = gi.torch_style_gsi(x, 448.0, "f16")
    for kind in ("mse", "reference"):
        codes, scales = c_quant(lib, kind, to_device(x, "f16"), gsi)
        oc, os_ = oracle.quantize(x, gsi, dtype="f16", variant=kind)
        np.testing.assert_array_equal(codes, oc)
        np.testing.assert_array_equal(scales, os_)


def test_large_shape_sampled_rows_and_determinism(lib):
    """Full config-2 maximum (16384 x 14336): rows are independent given the
    global scale, so a seeded sample of rows is checked against the oracle,
    and two launches must agree byte for byte."""
    from test_speed_scalesweep_b200 import scalesweep_mse_nvfp4_utils as mse
    m, k = 16384, 14336
    g = torch.Generator(device="cuda").manual_seed(123)
    x = torch.randn(m, k, generator=g, device="cuda", dtype=torch.float32).to(torch.bfloat16)
    x[:, ::211] *= 20
    gsi = (448.0 * 6.0) / x.abs().max().to(torch.float32)
    c1, s1 = mse.scalesweep_mse_nvfp4_quant_impl(x, gsi, False)
    c2, s2 = mse.scalesweep_mse_nvfp4_quant_impl(x, gsi, False)
    assert torch.equal(c1, c2) and torch.equal(s1.view(torch.uint8), s2.view(torch.uint8))
    rows = torch.from_numpy(np.sort(np.random.default_rng(0).choice(m, 48, replace=False))).cuda()
    bits = x[rows].view(torch.int16).cpu().numpy().view(np.uint16)
    oc, os_ = oracle.quantize(bits, gsi.item(), swizzled=False)
    np.testing.assert_array_equal(c1[rows].cpu().numpy(), oc)
    np.testing.assert_array_equal(s1.view(torch.uint8)[rows].cpu().numpy(), os_)


# ---- global amax / scale -------------------------------------------------------------


@pytest.mark.parametrize("shape,dtype", [((128, 4096), torch.bfloat16), ((1, 16), torch.bfloat16),
                                         ((333, 80), torch.float16), ((4096, 14336), torch.bfloat16),
                                         ((7, 24), torch.bfloat16)])
@pytest.mark.parametrize("fp8_max", [448.0, 256.0])
def test_global_scale_matches_torch_bit_exact(lib, shape, dtype, fp8_max):
    from test_speed_scalesweep_b200 import global_scale
    g = torch.Generator(device="cuda").manual_seed(sum(shape))
    x = (torch.randn(shape, generator=g, device="cuda") * 3).to(dtype)
    ref = (fp8_max * 6.0) / x.abs().max().to(torch.float32)
    amax = torch.empty(1, device="cuda")
    got = global_scale.global_scale_inv_from_max(x, fp8_max, amax_out=amax)
    assert got.view(torch.int32).item() == ref.view(torch.int32).item()
    assert amax.item() == x.abs().max().float().item()
    two_step = global_scale.global_scale_from_amax(global_scale.absmax(x), fp8_max)
    assert two_step.view(torch.int32).item() == ref.view(torch.int32).item()


def test_absmax_propagates_nan_like_torch(lib):
    from test_speed_scalesweep_b200 import global_scale
    x = torch.randn(64, 64, device="cuda").to(torch.bfloat16)
    x[3, 5] = float("nan")
    assert torch.isnan(global_scale.absmax(x)).item()
    assert torch.isnan(x.abs().max()).item()


def test_global_scale_oracle_agrees(lib):
    from test_speed_scalesweep_b200 import global_scale
    x = gi.outlier_activations(64, 1024, seed=9)
    got = global_scale.global_scale_inv_from_max(to_device(x), 448.0).item()
    assert np.float32(got) == np.float32(oracle.global_scale_inv(oracle.absmax(x), 448.0))


# ---- Python API --------------------------------------------------------------------


def test_python_api_and_dispatcher(lib):
    from test_speed_scalesweep_b200 import custom, scalesweep_mse_nvfp4_utils as mse
    x = gi.outlier_activations(130, 512, seed=13)
    xd = to_device(x)
    gsi = torch.tensor([gi.torch_style_gsi(x, 256.0)], device="cuda")
    codes, scales = mse.scalesweep_mse_nvfp4_quant_impl(xd, gsi, True)
    assert scales.dtype == torch.float8_e4m3fn and scales.shape == (256, 32)
    oc, os_ = oracle.quantize(x, gsi.item())
    mask = gi.written_scale_mask(dict(m=130, k=512), "mse", True, os_.shape)
    np.testing.assert_array_equal(codes.cpu().numpy(), oc)
    np.testing.assert_array_equal(scales.view(torch.uint8).cpu().numpy()[mask], os_[mask])
    # N-D input through the dispatcher flattens to [-1, K]
    c3, s3 = custom.nvfp4_quant(xd.view(13, 10, 512), gsi, True, "scalesweep_mse")
    assert torch.equal(c3, codes)
    assert torch.equal(s3.view(torch.uint8)[torch.from_numpy(mask).cuda()],
                       scales.view(torch.uint8)[torch.from_numpy(mask).cuda()])


def test_registered_ops_and_cuda_graph_capture(lib):
    import test_speed_scalesweep_b200.ops  # noqa: F401
    x = to_device(gi.outlier_activations(256, 4096, seed=17))
    gsi = torch.tensor([gi.torch_style_gsi(x.view(torch.int16).cpu().numpy().view(np.uint16), 448.0)],
                       device="cuda")
    op = torch.ops.scalesweep_b200.scalesweep_mse_nvfp4_quant
    c_eager, s_eager = op(x, gsi, True)
    out = torch.empty_like(c_eager)
    osc = torch.empty_like(s_eager)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        op.out(x, gsi, True, output=out, output_scale=osc)  # warm-up on the side stream
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    out.zero_()
    with torch.cuda.graph(graph):
        op.out(x, gsi, True, output=out, output_scale=osc)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, c_eager)
    assert torch.equal(osc.view(torch.uint8), s_eager.view(torch.uint8))


def _random_case(i):
    """Seeded random configuration: shape (ragged K, padded_n, misaligned
    rows), dtype, variant, layout and input distribution, with NaN / inf /
    zero / denormal specials sprinkled in some cases."""
    rng = np.random.default_rng(9000 + i)
    kind = ["mse", "reference", "weighted", "rtn", "mse", "reference"][i % 6]
    if i % 8 == 7:
        kind = "mse128" if i % 16 == 7 else "weighted128"
    small = kind in ("mse128", "weighted128")
    m = int(rng.integers(1, 64 if small else 700))
    k = 16 * int(rng.integers(1, 32 if small else 400))
    pn = k + 16 * int(rng.integers(0, 5)) if rng.random() < 0.3 else k
    dtype = "f16" if rng.random() < 0.25 else "bf16"
    swz = bool(rng.random() < 0.7)
    if rng.random() < 0.5:
        x = gi.wide_range_activations(m, k, 100 + i, dtype)
    else:
        x = gi.outlier_activations(m, k, 100 + i, dtype)
    if rng.random() < 0.3:
        specials = np.array([0x7FC0, 0x7F80, 0xFF80, 0x0000, 0x8000, 0x0001, 0x8003]
                            if dtype == "bf16" else
                            [0x7E00, 0x7C00, 0xFC00, 0x0000, 0x8000, 0x0001, 0x8003], np.uint16)
        flat = x.reshape(-1)
        idx = rng.choice(flat.size, size=min(flat.size, 1 + flat.size // 97), replace=False)
        flat[idx] = rng.choice(specials, size=idx.size)
    return kind, m, k, pn, dtype, swz, x


@pytest.mark.parametrize("i", range(48))
def test_random_configurations_match_oracle(lib, i):
    kind, m, k, pn, dtype, swz, x = _random_case(i)
    if kind == "reference" and pn != k:
        pn = k  # the reference variant has no padded_n (it raises)
    finite = gi.bits_to_f32(x, dtype)
    finite = finite[np.isfinite(finite)]
    amax = float(np.abs(finite).max()) if finite.size else 1.0
    gsi = float(np.float32(2688.0) / np.float32(amax if amax > 0 else 1.0))
    codes, scales = c_quant(lib, kind, to_device(x, dtype), gsi, padded_n=pn if pn != k else None,
                            swizzled=swz)
    variant = {"mse": "mse", "reference": "reference", "weighted": "weighted", "rtn": "mse",
               "mse128": "mse", "weighted128": "weighted"}[kind]
    mode = {"rtn": "rtn", "mse128": "full_range", "weighted128": "full_range"}.get(kind, "window")
    oc, os_ = oracle.quantize(x, gsi, dtype=dtype, padded_n=pn if pn != k else None,
                              swizzled=swz, variant=variant, mode=mode)
    np.testing.assert_array_equal(codes, oc)
    np.testing.assert_array_equal(scales, os_)
