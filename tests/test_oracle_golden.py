"""The CPU oracle against the golden vectors produced by the reference's own
Triton kernels (tests/golden/make_golden.py), plus unit checks of the
conversions the oracle restates."""
import hashlib

import numpy as np
import pytest

import golden_inputs as gi
import oracle


def _kind(variant):
    kind, layout = variant.rsplit("_", 1)
    var = {"reference": "reference", "weighted": "weighted", "weighted128": "weighted"}.get(kind,
                                                                                            "mse")
    mode = "full_range" if kind in ("mse128", "weighted128") else "window"
    return var, mode, layout == "swz"


CASES = [(c["name"], v) for c in gi.CASES for v in c["variants"]]


@pytest.mark.parametrize("name,variant", CASES)
def test_oracle_matches_reference_golden(golden, name, variant):
    case = next(c for c in gi.CASES if c["name"] == name)
    x = golden[f"{name}/input"]
    gsi = float(golden[f"{name}/gsi"][0])
    # the seeded generator still reproduces the stored inputs
    assert np.array_equal(x, gi.make_input(case))
    assert np.float32(gsi) == np.float32(gi.make_gsi(case, x))
    var, mode, swz = _kind(variant)
    codes, scales = oracle.quantize(x, gsi, dtype=case.get("dtype", "bf16"),
                                    padded_n=case.get("padded_n"), swizzled=swz, variant=var,
                                    mode=mode)
    assert np.array_equal(codes, golden[f"{name}/{variant}/codes"])
    # written bytes equal; unwritten padding untouched (both hold the sentinel)
    assert np.array_equal(scales, golden[f"{name}/{variant}/scales"])


@pytest.mark.parametrize("case", gi.CHECKSUM_CASES, ids=lambda c: c["name"])
def test_oracle_full_config1_checksums(golden, case):
    name = case["name"]
    x = gi.make_input(case)
    assert hashlib.sha256(x.tobytes()).digest() == golden[f"{name}/input_sha256"].tobytes()
    gsi = gi.make_gsi(case, x)
    assert np.float32(gsi) == golden[f"{name}/gsi"][0]
    for variant in case["variants"]:
        var = "reference" if variant.startswith("reference") else "mse"
        codes, scales = oracle.quantize(x, gsi, variant=var)
        h = hashlib.sha256(codes.tobytes() + scales.tobytes()).digest()
        assert h == golden[f"{name}/{variant}/sha256"].tobytes(), variant


def test_variants_differ_on_wide_range_golden(golden):
    a = golden["wide/mse_swz/scales"]
    b = golden["wide/reference_swz/scales"]
    c = golden["wide/weighted_swz/scales"]
    assert np.sum(a != b) > 0
    assert np.sum(a != c) > 0


def test_e2m1_encode_thresholds():
    # nearest-even on the E2M1 grid; the torch RTN thresholds of
    # benchmark_nvfp4_tokens.py:162-183 give the same magnitudes
    cases = {0.0: 0, 0.25: 0, 0.2500001: 1, 0.75: 2, 0.7499999: 1, 1.25: 2, 1.2500001: 3,
             1.75: 4, 2.5: 4, 2.5000002: 5, 3.5: 6, 5.0: 6, 5.0000005: 7, 6.0: 7, 1e30: 7,
             float("inf"): 7}
    for x, code in cases.items():
        assert oracle.e2m1_encode(x) == code, x
        assert oracle.e2m1_encode(-x) == code | 8, -x
    assert oracle.e2m1_encode(float("nan")) == 7
    assert oracle.e2m1_encode(-float("nan")) == 7


def test_e4m3_encode_matches_torch_in_range():
    import torch
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.uniform(0, 448, 20000), np.exp(rng.uniform(-12, 6, 20000)),
                         np.arange(0, 448.0, 0.125)]).astype(np.float32)
    ref = torch.from_numpy(xs).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    got = np.array([oracle.e4m3_encode(float(v)) for v in xs], np.uint8)
    assert np.array_equal(got, ref)
    # saturation and NaN (torch's CPU cast is not saturating; hardware is)
    assert oracle.e4m3_encode(449.0) == 0x7E
    assert oracle.e4m3_encode(1e9) == 0x7E
    assert oracle.e4m3_encode(float("inf")) == 0x7E
    assert oracle.e4m3_encode(-float("inf")) == 0xFE
    assert oracle.e4m3_encode(float("nan")) == 0x7F
    assert oracle.e4m3_encode(-float("nan")) == 0x7F
    for raw in range(127):
        assert oracle.e4m3_encode(oracle.e4m3_decode(raw)) == raw


def test_swizzle_is_a_bijection_on_the_padded_tile_grid():
    for m, bpc in [(128, 4), (256, 12), (129, 5), (1, 1)]:
        rp = -(-m // 128) * 128
        bp = -(-bpc // 4) * 4
        rows, cols = np.meshgrid(np.arange(rp), np.arange(bp), indexing="ij")
        off = gi.swizzled_offset(rows, cols, bp).ravel()
        assert np.array_equal(np.sort(off), np.arange(rp * bp))
        for r, c in [(0, 0), (min(m, 100) - 1, bpc - 1)]:
            assert oracle.lib().orc_swizzled_offset(r, c, bp) == gi.swizzled_offset(r, c, bp)


def test_rtn_mode_is_the_base_code():
    x = gi.outlier_activations(8, 256, 3)
    gsi = gi.torch_style_gsi(x, 448.0)
    c_rtn, s_rtn = oracle.quantize(x, gsi, mode="rtn", swizzled=False)
    v = gi.bits_to_f32(x).reshape(8, 16, 16) * np.float32(gsi)
    amax = np.abs(v).max(-1)
    expect = np.array([oracle.e4m3_encode(float(np.float32(a) * np.float32(1.0 / 6.0)))
                       for a in amax.ravel()])
    assert np.array_equal(s_rtn.ravel(), np.clip(expect, 1, 126))


def test_sweep_beats_rtn_mse():
    x = gi.outlier_activations(64, 1024, 4)
    gsi = gi.torch_style_gsi(x, 256.0)
    xf = gi.bits_to_f32(x)
    errs = {}
    for mode in ("window", "rtn"):
        c, s = oracle.quantize(x, gsi, mode=mode)
        deq = oracle.dequantize(c, s, 64, 1024) / np.float32(gsi)
        errs[mode] = float(np.mean((deq - xf) ** 2))
    assert errs["window"] < errs["rtn"]
