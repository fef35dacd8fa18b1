"""Seeded inputs for the golden vectors and the parity tests.

Activations follow the workload description of the scale-sweep benchmarks:
bf16 N(0, 1) with ceil(0.5% * K) seeded columns multiplied by 20 (outlier
channels); the global-scale multiplier handed to the kernel is
``fp8_max * 6 / amax`` evaluated the way torch evaluates
``(fp8_max * 6.0) / x.abs().max().float()`` (``Tensor.__rdiv__`` =
``reciprocal() * scalar``), see ``bench_kernel/test_kernel_latency.py:65-75``.
"""
from __future__ import annotations

import numpy as np

BLOCK = 16


def _to_bits(x32: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 to bf16/f16 (nearest-even) and return the raw uint16 bits."""
    x32 = np.ascontiguousarray(x32, np.float32)
    if dtype == "f16":
        return x32.astype(np.float16).view(np.uint16)
    u = x32.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x32)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FC0
    return r


def outlier_activations(m: int, k: int, seed: int, dtype: str = "bf16") -> np.ndarray:
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k), dtype=np.float32)
    n_out = -(-5 * k // 1000)  # ceil(0.005 * k)
    cols = rng.choice(k, size=n_out, replace=False)
    x[:, cols] *= np.float32(20.0)
    return _to_bits(x, dtype)


def wide_range_activations(m: int, k: int, seed: int, dtype: str = "bf16") -> np.ndarray:
    """Uniform(-1, 1) values with a per-row magnitude spread of e^[-8, 8]:
    exercises every region of the E4M3 scale range and the window edges,
    where the two reference variants (round-to-nearest vs round-down base
    code, chain vs tree SSE) choose different scales."""
    rng = np.random.default_rng(seed)
    x = rng.uniform(-1.0, 1.0, (m, k)).astype(np.float32)
    x *= np.exp(rng.uniform(-8.0, 8.0, (m, 1))).astype(np.float32)
    return _to_bits(x, dtype)


def bits_to_f32(bits: np.ndarray, dtype: str = "bf16") -> np.ndarray:
    if dtype == "f16":
        return bits.view(np.float16).astype(np.float32)
    return (bits.astype(np.uint32) << 16).view(np.float32)


def torch_style_gsi(bits: np.ndarray, fp8_max: float, dtype: str = "bf16") -> float:
    amax = np.float32(np.max(np.abs(bits_to_f32(bits, dtype)))) if bits.size else np.float32(0)
    with np.errstate(divide="ignore"):
        rec = np.float32(1.0) / amax
    return float(np.float32(rec * np.float32(fp8_max * 6.0)))


def _edge_rows() -> np.ndarray:
    """Hand-built blocks: zeros, lone values, ties, tiny and saturating blocks."""
    k = 256
    rows = []
    r = np.zeros(k, np.float32)
    rows.append(r.copy())                                    # all-zero row
    r = np.zeros(k, np.float32); r[::17] = 1.0               # lone values
    rows.append(r)
    ties = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0,
                     -0.25, -0.75, -1.25, -1.75, -2.5, -3.5, -5.0, -6.0], np.float32)
    rows.append(np.tile(ties, k // 16))                      # e2m1 midpoints
    rows.append(np.tile(ties * np.float32(1.0 / 64), k // 16))
    tiny = np.linspace(-3e-3, 3e-3, k).astype(np.float32)   # subnormal e4m3 scales
    rows.append(tiny)
    rows.append(np.linspace(-9000.0, 9000.0, k).astype(np.float32))  # base > 448
    neg0 = np.full(k, -0.0, np.float32); neg0[5::16] = -1e-3
    rows.append(neg0)
    const = np.full(k, 3.0, np.float32); const[1::2] = -3.0
    rows.append(const)
    return np.stack(rows)


CASES = [
    dict(name="cfg1_slice", m=16, k=4096, seed=1, fp8_max=448.0,
         variants=["mse_swz", "reference_swz", "mse128_swz", "mse_lin", "weighted_swz",
                   "weighted128_swz"]),
    dict(name="conv256", m=7, k=2048, seed=2, fp8_max=256.0,
         variants=["mse_swz", "reference_swz"]),
    dict(name="ragged", m=129, k=80, seed=3, fp8_max=448.0,
         variants=["mse_swz", "reference_swz", "mse_lin", "reference_lin"]),
    dict(name="padded", m=33, k=64, seed=4, fp8_max=448.0, padded_n=96,
         variants=["mse_swz", "mse_lin", "mse128_swz", "weighted_swz"]),
    dict(name="single_row", m=1, k=512, seed=5, fp8_max=448.0,
         variants=["mse_swz", "reference_swz"]),
    dict(name="one_block", m=5, k=16, seed=6, fp8_max=448.0,
         variants=["mse_swz", "reference_swz", "mse128_swz"]),
    dict(name="fp16", m=9, k=256, seed=7, fp8_max=448.0, dtype="f16",
         variants=["mse_swz", "reference_swz"]),
    dict(name="edge", m=8, k=256, gsi=1.0, rows="edge",
         variants=["mse_swz", "reference_swz", "mse128_swz", "mse_lin", "weighted_swz",
                   "weighted128_swz"]),
    dict(name="special", m=2, k=256, gsi=1.0, rows="special",
         variants=["mse_swz", "reference_swz", "mse128_swz", "weighted_swz"]),
    dict(name="huge_gsi", m=3, k=64, seed=8, gsi=1e30,
         variants=["mse_swz", "reference_swz"]),
    dict(name="wide", m=48, k=1024, seed=10, fp8_max=448.0, rows="wide",
         variants=["mse_swz", "reference_swz", "weighted_swz", "weighted_lin"]),
]

# Full-size pins (config-1 shape): the golden file stores SHA-256 digests of the
# reference's outputs instead of the outputs themselves.
CHECKSUM_CASES = [
    dict(name="cfg1_full", m=128, k=4096, seed=1001, fp8_max=448.0,
         variants=["mse_swz", "reference_swz"]),
    dict(name="cfg1_full_conv256", m=128, k=4096, seed=1002, fp8_max=256.0,
         variants=["mse_swz", "reference_swz"]),
]


def _special_rows() -> np.ndarray:
    """NaN / Inf blocks (bf16 bit patterns); NaN of both signs."""
    rng = np.random.default_rng(99)
    x = _to_bits(rng.standard_normal((2, 256), dtype=np.float32), "bf16")
    x[0, 3] = 0x7FC0                # one NaN in block 0
    x[0, 16 + 5] = 0x7F80           # +inf in block 1
    x[0, 32 + 9] = 0xFF80           # -inf in block 2
    x[0, 48:64] = 0xFFC0            # block 3 all (negative) NaN
    x[0, 64:80] = 0                 # block 4 zeros with one NaN
    x[0, 64 + 7] = 0x7FC0
    x[1, 0:16] = 0x7F80             # block of +inf
    x[1, 16:32] = 0x0001            # bf16 subnormals
    x[1, 32:48] = 0x8000            # -0.0
    return x


def make_input(case: dict) -> np.ndarray:
    dtype = case.get("dtype", "bf16")
    if case.get("rows") == "edge":
        return _to_bits(_edge_rows(), dtype)
    if case.get("rows") == "special":
        return _special_rows()
    if case.get("rows") == "wide":
        return wide_range_activations(case["m"], case["k"], case["seed"], dtype)
    return outlier_activations(case["m"], case["k"], case["seed"], dtype)


def make_gsi(case: dict, bits: np.ndarray) -> float:
    if "gsi" in case:
        return float(np.float32(case["gsi"]))
    return torch_style_gsi(bits, case["fp8_max"], case.get("dtype", "bf16"))


def swizzled_offset(row, col, bpc_pad):
    """CUTLASS 128x4 scale-factor layout (bench_kernel/scalesweep_mse_nvfp4_utils.py:23-43)."""
    return ((row >> 7) * (bpc_pad * 128) + (col >> 2) * 512 + (row & 31) * 16
            + ((row & 127) >> 5) * 4 + (col & 3))


def written_scale_mask(case: dict, kind: str, swizzled: bool, shape) -> np.ndarray:
    m = case["m"]
    n_phys = case.get("padded_n") or case["k"]
    bpc = n_phys // BLOCK
    mask = np.zeros(int(np.prod(shape)), bool)
    if not swizzled:
        mask[: m * bpc] = True
        return mask.reshape(shape)
    bpc_pad = -(-bpc // 4) * 4
    rows, cols = np.meshgrid(np.arange(m), np.arange(bpc), indexing="ij")
    mask[swizzled_offset(rows, cols, bpc_pad).ravel()] = True
    return mask.reshape(shape)
