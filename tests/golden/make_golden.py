"""Generate the golden vectors in ``tests/golden/golden.npz`` by running the
reference's OWN Triton kernels (``bench_kernel/scalesweep_mse_nvfp4_utils.py``
and ``bench_kernel/scalesweep_mse_reference_nvfp4_utils.py``) unmodified under
Triton's CPU interpreter (``TRITON_INTERPRET=1``).

The interpreter cannot execute inline PTX, and its software float8 / bfloat16
casts are approximate, so this script replaces exactly those builder hooks
with exact numpy emulation of the hardware instructions:

* ``cvt.rn.satfinite.e2m1x2.f32``  round-to-nearest-even onto
  {0, 0.5, 1, 1.5, 2, 3, 4, 6}, saturating at 6, sign kept (-0 included);
* ``cvt.rn.f16x2.e2m1x2`` + ``cvt.f32.f16``  exact decode;
* ``sub.rn.f32`` / ``mul.rn.f32`` / ``fma.rn.f32``  IEEE binary32 (fma via
  round-to-odd in binary64, Boldo & Melquiond 2008);
* ``fp32 -> float8e4nv``  round-to-nearest-even, saturating finite (>448 -> 448,
  NaN -> 0x7F), which is what ``cvt.rn.satfinite.e4m3x2.f32`` does;
* ``float8e4nv -> fp32`` and ``bf16/f16 -> fp32``  exact.

Everything else -- candidate windows, clamps, division, tie-break, swizzle,
nibble packing, masking -- is the reference's own kernel code.  Run here
(needs the reference checkout; the GPU machine does not have it):

    python tests/golden/make_golden.py /path/to/reference
"""
from __future__ import annotations

import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import golden_inputs  # noqa: E402


def _fma_f32(a, b, c):
    """Correctly rounded binary32 fma(a, b, c) via round-to-odd in binary64."""
    a = np.asarray(a, np.float32).astype(np.float64)
    b = np.asarray(b, np.float32).astype(np.float64)
    c = np.asarray(c, np.float32).astype(np.float64)
    p = a * b  # exact: 48 significant bits
    with np.errstate(invalid="ignore", over="ignore"):
        s = p + c
        bb = s - p
        e = (p - (s - bb)) + (c - bb)
        bits = s.view(np.uint64)
        adjust = (e != 0) & ((bits & 1) == 0) & np.isfinite(s)
        toward = np.where(e > 0, np.inf, -np.inf)
        s = np.where(adjust, np.nextafter(s, toward), s)
        return s.astype(np.float32)


_E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], np.float32)


def e2m1_encode(x):
    x = np.asarray(x, np.float32)
    a = np.abs(x)
    code = np.select(
        [a <= 0.25, a < 0.75, a <= 1.25, a < 1.75, a <= 2.5, a < 3.5, a <= 5.0],
        [0, 1, 2, 3, 4, 5, 6], 7).astype(np.uint8)
    code = np.where(np.isnan(x), NAN_E2M1_NIBBLE & 7, code).astype(np.uint8)
    sign = np.where(np.isnan(x), NAN_E2M1_NIBBLE >> 3, np.signbit(x)).astype(np.uint8)
    return code | (sign << 3)


# Nibble produced by cvt.rn.satfinite.e2m1x2.f32 for a NaN input of either
# sign: +6.0 (measured on B200).
NAN_E2M1_NIBBLE = 0x7


def e2m1_decode(nib):
    nib = np.asarray(nib, np.uint8)
    v = _E2M1_VALUES[nib & 7]
    return np.where((nib & 8) != 0, -v, v).astype(np.float32)


def e4m3_encode(x):
    x = np.asarray(x, np.float32)
    a = np.abs(x).astype(np.float64)
    out = np.zeros(x.shape, np.uint8)
    fin = np.isfinite(a)
    sub = fin & (a < 2.0 ** -6)
    out[sub] = np.rint(a[sub] * 512.0).astype(np.uint8)
    nm = fin & ~sub
    if np.any(nm):
        an = a[nm]
        e = np.floor(np.log2(an)).astype(np.int64)
        e = np.where(np.ldexp(1.0, e) > an, e - 1, e)
        e = np.where(np.ldexp(1.0, e + 1) <= an, e + 1, e)
        m = np.rint((an / np.ldexp(1.0, e) - 1.0) * 8.0).astype(np.int64)
        e = np.where(m == 8, e + 1, e)
        m = np.where(m == 8, 0, m)
        out[nm] = np.minimum((e + 7) * 8 + m, 0x7E).astype(np.uint8)
    out[np.isinf(a)] = 0x7E
    out = out | (np.signbit(x).astype(np.uint8) << 7)
    # NaN of either sign becomes the positive NaN code 0x7F (measured on B200).
    out[np.isnan(a)] = 0x7F
    return out


def e4m3_decode(raw):
    raw = np.asarray(raw, np.uint8)
    e = (raw >> 3) & 0xF
    m = (raw & 7).astype(np.float64)
    mag = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * np.ldexp(1.0, e.astype(np.int64) - 7))
    mag = np.where((raw & 0x7F) == 0x7F, np.nan, mag)
    return np.where((raw & 0x80) != 0, -mag, mag).astype(np.float32)


def _pair_sq_err(x0, x1, acc=None):
    q0 = e2m1_decode(e2m1_encode(x0))
    q1 = e2m1_decode(e2m1_encode(x1))
    with np.errstate(invalid="ignore", over="ignore"):
        d0 = (q0 - np.asarray(x0, np.float32)).astype(np.float32)
        d1 = (q1 - np.asarray(x1, np.float32)).astype(np.float32)
        if acc is None:
            d0 = (d0 * d0).astype(np.float32)
        else:
            d0 = _fma_f32(d0, d0, acc)
    return _fma_f32(d1, d1, d0)


def _pair_weighted(x0, x1, w0, w1, acc=None):
    """scalesweep_nvfp4_utils.py:40-111: d^2 rounded, times weight, fma-accumulated."""
    q0 = e2m1_decode(e2m1_encode(x0))
    q1 = e2m1_decode(e2m1_encode(x1))
    with np.errstate(invalid="ignore", over="ignore"):
        d0 = (q0 - np.asarray(x0, np.float32)).astype(np.float32)
        d1 = (q1 - np.asarray(x1, np.float32)).astype(np.float32)
        d0 = (d0 * d0).astype(np.float32)
        d1 = (d1 * d1).astype(np.float32)
        if acc is None:
            d0 = (d0 * np.asarray(w0, np.float32)).astype(np.float32)
        else:
            d0 = _fma_f32(d0, w0, acc)
    return _fma_f32(d1, w1, d0)


def _pack16(xs):
    nib = [e2m1_encode(x).astype(np.uint32) for x in xs]
    words = []
    for w in range(2):
        word = np.zeros(nib[0].shape, np.uint32)
        for byte in range(4):
            k = 4 * w + byte
            b = nib[2 * k] | (nib[2 * k + 1] << 4)
            word |= b << (8 * byte)
        words.append(word)
    return words


class _Call:
    def __init__(self, results):
        self._results = results

    def get_result(self, i):
        return self._results[i]


def install_shims():
    import triton.language as tl
    from triton.runtime import interpreter as interp

    TensorHandle = interp.TensorHandle

    pair_plain = ["cvt.rn.satfinite.e2m1x2.f32 b, $2, $1;", "cvt.rn.f16x2.e2m1x2 h, b;",
                  "sub.rn.f32 d0, q0, $1;", "sub.rn.f32 d1, q1, $2;",
                  "mul.rn.f32 d0, d0, d0;", "fma.rn.f32 $0, d1, d1, d0;"]
    pair_acc = ["cvt.rn.satfinite.e2m1x2.f32 b, $2, $1;", "cvt.rn.f16x2.e2m1x2 h, b;",
                "sub.rn.f32 d0, q0, $1;", "sub.rn.f32 d1, q1, $2;",
                "fma.rn.f32 d0, d0, d0, $3;", "fma.rn.f32 $0, d1, d1, d0;"]
    w_plain = ["cvt.rn.satfinite.e2m1x2.f32 b, $2, $1;", "sub.rn.f32 d0, q0, $1;",
               "mul.rn.f32 d0, d0, d0;", "mul.rn.f32 d1, d1, d1;", "mul.rn.f32 d0, d0, $3;",
               "fma.rn.f32 $0, d1, $4, d0;"]
    w_acc = ["cvt.rn.satfinite.e2m1x2.f32 b, $2, $1;", "sub.rn.f32 d0, q0, $1;",
             "mul.rn.f32 d0, d0, d0;", "mul.rn.f32 d1, d1, d1;", "fma.rn.f32 d0, d0, $3, $5;",
             "fma.rn.f32 $0, d1, $4, d0;"]
    pack = ["cvt.rn.satfinite.e2m1x2.f32 b0,  $3,  $2;", "cvt.rn.satfinite.e2m1x2.f32 b7,  $17, $16;",
            "mov.b32 $0, {b0, b1, b2, b3};", "mov.b32 $1, {b4, b5, b6, b7};"]

    def create_inline_asm(self, inlineAsm, constraints, values, type, isPure, pack_n):
        assert pack_n == 1
        data = [np.asarray(v.data) for v in values]
        text = " ".join(inlineAsm.split())
        if all(" ".join(s.split()) in text for s in pack):
            assert constraints == "=r,=r," + ",".join(["f"] * 16) and len(data) == 16
            lo, hi = _pack16([d.astype(np.float32) for d in data])
            return _Call([TensorHandle(lo, tl.uint32), TensorHandle(hi, tl.uint32)])
        if all(s in text for s in w_acc):
            assert constraints == "=f,f,f,f,f,f" and len(data) == 5
            return _Call([TensorHandle(_pair_weighted(data[0], data[1], data[2], data[3], data[4]),
                                       tl.float32)])
        if all(s in text for s in w_plain):
            assert constraints == "=f,f,f,f,f" and len(data) == 4
            return _Call([TensorHandle(_pair_weighted(data[0], data[1], data[2], data[3]),
                                       tl.float32)])
        if all(s in text for s in pair_acc):
            assert constraints == "=f,f,f,f" and len(data) == 3
            return _Call([TensorHandle(_pair_sq_err(data[0], data[1], data[2]), tl.float32)])
        if all(s in text for s in pair_plain):
            assert constraints == "=f,f,f" and len(data) == 2
            return _Call([TensorHandle(_pair_sq_err(data[0], data[1]), tl.float32)])
        raise AssertionError("unrecognised inline asm block:\n" + inlineAsm)

    orig_fp_to_fp = interp.InterpreterBuilder.create_fp_to_fp
    orig_cast_impl = interp.InterpreterBuilder.cast_impl

    def create_fp_to_fp(self, src, dst_type, rounding_mode):
        s = src.dtype.scalar
        d = dst_type.scalar
        if s == tl.float32 and d == tl.float8e4nv:
            return TensorHandle(e4m3_encode(src.data.astype(np.float32)), tl.float8e4nv)
        if s == tl.float8e4nv and d == tl.float32:
            return TensorHandle(e4m3_decode(src.data.astype(np.uint8)), tl.float32)
        return orig_fp_to_fp(self, src, dst_type, rounding_mode)

    def cast_impl(self, src, dst_type):
        s = src.dtype.scalar
        d = dst_type.scalar
        if s == tl.bfloat16 and d == tl.float32:
            u = src.data.view(np.uint16).astype(np.uint32) << 16
            return TensorHandle(u.view(np.float32), tl.float32)
        if s == tl.float16 and d == tl.float32:
            return TensorHandle(src.data.view(np.float16).astype(np.float32), tl.float32)
        return orig_cast_impl(self, src, dst_type)

    interp.InterpreterBuilder.create_inline_asm = create_inline_asm
    interp.InterpreterBuilder.create_fp_to_fp = create_fp_to_fp
    interp.InterpreterBuilder.cast_impl = cast_impl
    interp.InterpreterBuilder.create_fp_ext = lambda self, src, dst_type: cast_impl(self, src, dst_type)


def load_reference(ref_root):
    import triton

    sys.path.insert(0, os.path.join(ref_root, "bench_kernel"))
    import scalesweep_mse_nvfp4_utils as mse
    import scalesweep_mse_reference_nvfp4_utils as mse_ref

    # The autotuner would time several configs (needs a GPU); every config
    # gives identical per-block numerics, so pin one.
    mse._scalesweep_mse_nvfp4_quant_kernel.configs = [
        triton.Config({"BLOCKS_PER_PROGRAM": 512}, num_warps=16)]
    mse_ref.scalesweep_quantize_kernel.configs = [
        triton.Config({"BLOCKS_PER_PROGRAM": 512, "NUM_STAGES": 2}, num_warps=16)]
    import scalesweep_nvfp4_utils as weighted
    weighted._scalesweep_nvfp4_quant_kernel.configs = [
        triton.Config({"BLOCKS_PER_PROGRAM": 512}, num_warps=16)]

    # Output buffers come from torch.empty; pre-fill them with a sentinel so
    # the bytes the kernel leaves untouched are deterministic in the fixture.
    def filled(create):
        def wrapper(*args, **kwargs):
            out, scale = create(*args, **kwargs)
            out.view(torch.uint8).fill_(SENTINEL)
            scale.view(torch.uint8).fill_(SENTINEL)
            return out, scale
        return wrapper

    import torch
    mse.create_fp4_output_tensors = filled(mse.create_fp4_output_tensors)
    mse_ref.create_fp4_output_tensors = filled(mse_ref.create_fp4_output_tensors)
    weighted.create_fp4_output_tensors = filled(weighted.create_fp4_output_tensors)
    return mse, mse_ref, weighted


SENTINEL = 0xA5


def main(ref_root):
    import torch

    install_shims()
    mse, mse_ref, weighted = load_reference(ref_root)
    out = {}
    for case in golden_inputs.CASES:
        name = case["name"]
        x = golden_inputs.make_input(case)
        gsi = golden_inputs.make_gsi(case, x)
        xt = torch.from_numpy(x.view(np.int16)).view(
            torch.bfloat16 if case.get("dtype", "bf16") == "bf16" else torch.float16)
        gt = torch.tensor([gsi], dtype=torch.float32)
        out[f"{name}/input"] = x
        out[f"{name}/gsi"] = np.array([gsi], np.float32)
        for variant in case["variants"]:
            swz = variant.endswith("_swz")
            kind = variant.rsplit("_", 1)[0]
            padded_n = case.get("padded_n")
            if kind == "mse":
                codes, scales = mse.scalesweep_mse_nvfp4_quant_impl(xt, gt, swz, padded_n)
            elif kind == "mse128":
                codes, scales = mse.scalesweep_mse128_nvfp4_quant_impl(xt, gt, swz, padded_n)
            elif kind == "reference":
                codes, scales = mse_ref.scalesweep_mse_nvfp4_quant_impl(xt, gt, swz, padded_n)
            elif kind == "weighted":
                codes, scales = weighted.scalesweep_nvfp4_quant_impl(xt, gt, swz, padded_n)
            elif kind == "weighted128":
                codes, scales = weighted.scalesweep128_nvfp4_quant_impl(xt, gt, swz, padded_n)
            else:
                raise ValueError(variant)
            out[f"{name}/{variant}/codes"] = codes.numpy().copy()
            # Scale rows >= M (and columns past the blocks) are never written by
            # the kernel; record which bytes are meaningful.
            sc = scales.view(torch.uint8).numpy().copy()
            out[f"{name}/{variant}/scales"] = sc
            out[f"{name}/{variant}/scale_mask"] = golden_inputs.written_scale_mask(
                case, kind, swz, sc.shape)
        print(name, "done", flush=True)
    import hashlib
    for case in golden_inputs.CHECKSUM_CASES:
        name = case["name"]
        x = golden_inputs.make_input(case)
        gsi = golden_inputs.make_gsi(case, x)
        xt = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16)
        gt = torch.tensor([gsi], dtype=torch.float32)
        out[f"{name}/input_sha256"] = np.frombuffer(hashlib.sha256(x.tobytes()).digest(), np.uint8)
        out[f"{name}/gsi"] = np.array([gsi], np.float32)
        for variant in case["variants"]:
            kind = variant.rsplit("_", 1)[0]
            impl = mse if kind == "mse" else mse_ref
            codes, scales = impl.scalesweep_mse_nvfp4_quant_impl(xt, gt, True, None)
            h = hashlib.sha256(codes.numpy().tobytes() + scales.view(torch.uint8).numpy().tobytes())
            out[f"{name}/{variant}/sha256"] = np.frombuffer(h.digest(), np.uint8)
        print(name, "done", flush=True)
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz")
    np.savez_compressed(dst, **out)
    print("wrote", dst, os.path.getsize(dst), "bytes")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
