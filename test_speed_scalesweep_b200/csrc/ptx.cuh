// sm_100a PTX helpers for the NVFP4 scale-sweep kernels.
//
// Every arithmetic step whose rounding is part of the quantizer's result is
// written as explicit PTX with an explicit rounding mode, so neither nvcc's
// fma contraction nor any other rewrite can change a bit.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace ssw {

// ---- packed f32x2 (sm_100) -------------------------------------------------
__device__ __forceinline__ uint64_t pack2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpack2(uint64_t r, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(r));
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// ---- scalar binary32 with explicit rounding --------------------------------
__device__ __forceinline__ float mul_rn(float a, float b) {
  float r;
  asm("mul.rn.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float fma_rn(float a, float b, float c) {
  float r;
  asm("fma.rn.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ float add_rn(float a, float b) {
  float r;
  asm("add.rn.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// ---- E2M1 -----------------------------------------------------------------
// Round-trip delta of a pair: d_i = e2m1(x_i) - x_i, computed as
//   cvt.rn.satfinite.e2m1x2.f32 (x1 -> high nibble, x0 -> low nibble),
//   cvt.rn.f16x2.e2m1x2 (exact), and the mixed-precision subtract
//   sub.rn.f32.f16, which widens the f16 operand exactly and rounds once --
//   the same value as cvt.f32.f16 followed by sub.rn.f32.
__device__ __forceinline__ void e2m1_delta2(float x0, float x1, float& d0, float& d1) {
  asm("{\n\t.reg .b8 b;\n\t.reg .b32 h;\n\t.reg .b16 lo, hi;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b, %3, %2;\n\t"
      "cvt.rn.f16x2.e2m1x2 h, b;\n\t"
      "mov.b32 {lo, hi}, h;\n\t"
      "sub.rn.f32.f16 %0, lo, %2;\n\t"
      "sub.rn.f32.f16 %1, hi, %3;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(x0), "f"(x1));
}

// Same value through the two-step path (cvt.f32.f16 then sub.rn.f32).
__device__ __forceinline__ void e2m1_delta2_cvt(float x0, float x1, float& d0, float& d1) {
  asm("{\n\t.reg .b8 b;\n\t.reg .b32 h;\n\t.reg .b16 lo, hi;\n\t.reg .f32 q0, q1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b, %3, %2;\n\t"
      "cvt.rn.f16x2.e2m1x2 h, b;\n\t"
      "mov.b32 {lo, hi}, h;\n\t"
      "cvt.f32.f16 q0, lo;\n\t"
      "cvt.f32.f16 q1, hi;\n\t"
      "sub.rn.f32 %0, q0, %2;\n\t"
      "sub.rn.f32 %1, q1, %3;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(x0), "f"(x1));
}

// Eight values -> four packed code bytes, element 2j in the low nibble.
__device__ __forceinline__ uint32_t e2m1x8(float x0, float x1, float x2, float x3, float x4,
                                           float x5, float x6, float x7) {
  uint32_t r;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(r)
      : "f"(x0), "f"(x1), "f"(x2), "f"(x3), "f"(x4), "f"(x5), "f"(x6), "f"(x7));
  return r;
}

// ---- E4M3 -----------------------------------------------------------------
// fp32 -> E4M3 code, nearest-even, saturating finite; NaN -> 0x7F.
__device__ __forceinline__ uint32_t e4m3_code(float x) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.0f), "f"(x));
  return (uint32_t)(r & 0xFF);
}

// Exact E4M3 -> fp32 for codes 0..127 (sign bit clear); 0x7F -> NaN.
__device__ __forceinline__ float e4m3_value(uint32_t raw) {
  uint32_t e = (raw >> 3) & 0xF, m = raw & 7;
  if (raw == 0x7F) return __uint_as_float(0x7FC00000u);
  if (e == 0) return mul_rn((float)m, 0.001953125f);  // m * 2^-9, exact
  return __uint_as_float(((e + 120u) << 23) | (m << 20));
}

// ---- loads / stores ---------------------------------------------------------
// One 16-element block of 16-bit values (32 bytes, 32-byte aligned), streamed.
__device__ __forceinline__ void ld_block_v8(const void* p, uint32_t (&w)[8]) {
  asm volatile(
      "ld.global.nc.L1::no_allocate.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
      : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]), "=r"(w[4]), "=r"(w[5]), "=r"(w[6]),
        "=r"(w[7])
      : "l"(p));
}

__device__ __forceinline__ void st_v2(void* p, uint32_t a, uint32_t b) {
  asm volatile("st.global.v2.b32 [%0], {%1, %2};" ::"l"(p), "r"(a), "r"(b) : "memory");
}

}  // namespace ssw
