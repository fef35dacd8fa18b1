// Fused scale-sweep NVFP4 block quantizer for sm_100a.
//
// One thread owns one 16-element block (32 bytes of bf16/f16 input, 8 bytes
// of codes, 1 scale byte).  A warp covers 32 consecutive blocks, so its input
// load is one 1 KiB contiguous 256-bit-per-lane transaction and its code store
// one 256 B contiguous transaction; each lane stores its block's scale byte
// in the swizzled (or linear) scale layout.
//
// The candidate sweep is the hot loop.  Two candidates are evaluated side by
// side so that the normalisation multiply and the squared-error FMA run as
// packed f32x2 instructions (one issue slot for two lanes of work) and the
// E2M1 round trip's decode+subtract is a single mixed-precision
// sub.rn.f32.f16.  Summation order and rounding are exactly the reference's:
//   "mse"       : acc = d0*d0; acc = fma(d1,d1,acc); ... fma(d15,d15,acc)
//                 (bench_kernel/scalesweep_mse_nvfp4_utils.py:92-176)
//   "reference" : s_k = fma(d_{2k+1}, d_{2k+1}, d_{2k}*d_{2k}),
//                 ((s0+s1)+(s2+s3))+((s4+s5)+(s6+s7))
//                 (bench_kernel/scalesweep_mse_reference_nvfp4_utils.py:91-143)
//   "weighted"  : acc = d1^2 + d0^2, then acc = d^2 + acc per element, every
//                 square and sum rounded (importance weights of 1;
//                 bench_kernel/scalesweep_nvfp4_utils.py:40-149, :314)
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "ptx.cuh"
#include "quant.cuh"

namespace ssw {

namespace {

constexpr int kThreads = 256;  // the shared tables below rely on 256 threads
constexpr int kLower = -3;       // bench_kernel/scalesweep_mse_nvfp4_utils.py:17
constexpr int kWindow = 11;      // UPPER_BOUND - LOWER_BOUND + 1 (:17-18, :452-454)
constexpr int kMaxRaw = 126;     // REF_MAX_SCALE_RAW (:20)
constexpr int kWindowTab = 128 + kWindow;  // window positions j = code + 3, code in [-3, 134]
#ifndef SSW_QUANT_MIN_BLOCKS
#define SSW_QUANT_MIN_BLOCKS 4
#endif
constexpr int kMinBlocksPerSm = SSW_QUANT_MIN_BLOCKS;

struct ScaleEntry {
  float inv;  // 1 / s, IEEE (equals the reference's Triton 1.0 / s for every code)
  float s2;   // s * s (exact)
};

__device__ __forceinline__ int clamp_raw(int r) { return r < 1 ? 1 : (r > kMaxRaw ? kMaxRaw : r); }

// Squared error of the 16 values for two candidate reciprocals at once.
// Returns {sse_a, sse_b} packed.
template <int kVariant>
__device__ __forceinline__ uint64_t sse_pair(const uint64_t (&vp)[8], float inv_a, float inv_b) {
  const uint64_t ia = pack2(inv_a, inv_a), ib = pack2(inv_b, inv_b);
  if constexpr (kVariant == kVariantMse) {
    uint64_t acc = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float xa0, xa1, xb0, xb1, da0, da1, db0, db1;
      unpack2(mul2(vp[k], ia), xa0, xa1);
      unpack2(mul2(vp[k], ib), xb0, xb1);
      e2m1_delta2(xa0, xa1, da0, da1);
      e2m1_delta2(xb0, xb1, db0, db1);
      const uint64_t d0 = pack2(da0, db0), d1 = pack2(da1, db1);
      acc = (k == 0) ? mul2(d0, d0) : fma2(d0, d0, acc);
      acc = fma2(d1, d1, acc);
    }
    return acc;
  } else if constexpr (kVariant == kVariantWeighted) {
    // Squares rounded on their own, then summed in element order (importance
    // weights of 1: fma(d^2, 1, acc) == add(d^2, acc)).  Scalar mul.rn /
    // add.rn on purpose: a packed f32x2 multiply feeding a packed add may be
    // fused into one FMA, which rounds differently from the reference.
    float acc_a = 0.0f, acc_b = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float xa0, xa1, xb0, xb1, da0, da1, db0, db1;
      unpack2(mul2(vp[k], ia), xa0, xa1);
      unpack2(mul2(vp[k], ib), xb0, xb1);
      e2m1_delta2(xa0, xa1, da0, da1);
      e2m1_delta2(xb0, xb1, db0, db1);
      const float sa0 = mul_rn(da0, da0), sa1 = mul_rn(da1, da1);
      const float sb0 = mul_rn(db0, db0), sb1 = mul_rn(db1, db1);
      acc_a = (k == 0) ? add_rn(sa1, sa0) : add_rn(sa1, add_rn(sa0, acc_a));
      acc_b = (k == 0) ? add_rn(sb1, sb0) : add_rn(sb1, add_rn(sb0, acc_b));
    }
    return pack2(acc_a, acc_b);
  } else {
    uint64_t s[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float xa0, xa1, xb0, xb1, da0, da1, db0, db1;
      unpack2(mul2(vp[k], ia), xa0, xa1);
      unpack2(mul2(vp[k], ib), xb0, xb1);
      e2m1_delta2(xa0, xa1, da0, da1);
      e2m1_delta2(xb0, xb1, db0, db1);
      const uint64_t d0 = pack2(da0, db0), d1 = pack2(da1, db1);
      s[k] = fma2(d1, d1, mul2(d0, d0));
    }
    return add2(add2(add2(s[0], s[1]), add2(s[2], s[3])), add2(add2(s[4], s[5]), add2(s[6], s[7])));
  }
}

// Single-candidate squared error (the odd candidate of the 11-wide window).
template <int kVariant>
__device__ __forceinline__ float sse_one(const uint64_t (&vp)[8], float inv) {
  const uint64_t i2 = pack2(inv, inv);
  if constexpr (kVariant == kVariantMse) {
    float acc = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float x0, x1, d0, d1;
      unpack2(mul2(vp[k], i2), x0, x1);
      e2m1_delta2(x0, x1, d0, d1);
      acc = (k == 0) ? mul_rn(d0, d0) : fma_rn(d0, d0, acc);
      acc = fma_rn(d1, d1, acc);
    }
    return acc;
  } else if constexpr (kVariant == kVariantWeighted) {
    float acc = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float x0, x1, d0, d1;
      unpack2(mul2(vp[k], i2), x0, x1);
      e2m1_delta2(x0, x1, d0, d1);
      const float s0 = mul_rn(d0, d0), s1 = mul_rn(d1, d1);
      acc = (k == 0) ? add_rn(s1, s0) : add_rn(s1, add_rn(s0, acc));
    }
    return acc;
  } else {
    float s[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float x0, x1, d0, d1;
      unpack2(mul2(vp[k], i2), x0, x1);
      e2m1_delta2(x0, x1, d0, d1);
      s[k] = fma_rn(d1, d1, mul_rn(d0, d0));
    }
    return add_rn(add_rn(add_rn(s[0], s[1]), add_rn(s[2], s[3])),
                  add_rn(add_rn(s[4], s[5]), add_rn(s[6], s[7])));
  }
}

// vLLM's silu_and_mul on a word of two 16-bit values: silu(g) = g / (1 + e^-g)
// in binary32 (expf, IEEE division), rounded to the input type, then times
// the up value in that type (one rounding of the exact product), as
// torch.ops._C.silu_and_mul computes it (vllm 0.22, registered for
// model_executor/layers/activation.py:117-147).
//
// bf16 takes a cheaper binary32 silu that rounds to the same bf16 for every
// one of the 65536 bf16 inputs (checked exhaustively on B200 against vLLM):
// __expf and the approximate division __fdividef, except below -64, where
// 1 + e^-g can exceed 2^126 and __fdividef returns 0; there the IEEE
// division.  f16 keeps expf and IEEE division: the cheaper forms differ from
// vLLM on one or two f16 inputs.
__device__ __forceinline__ float silu_bf16_exact(float g) {
  const float d = 1.0f + __expf(-g);
  return g < -64.0f ? g / d : __fdividef(g, d);
}

template <int kDType>
__device__ __forceinline__ uint32_t silu_mul2(uint32_t g, uint32_t u) {
  if constexpr (kDType == kDTypeBF16) {
    const __nv_bfloat162 gb = *reinterpret_cast<const __nv_bfloat162*>(&g);
    const __nv_bfloat162 s = __floats2bfloat162_rn(silu_bf16_exact(__low2float(gb)),
                                                   silu_bf16_exact(__high2float(gb)));
    const __nv_bfloat162 h = __hmul2(s, *reinterpret_cast<const __nv_bfloat162*>(&u));
    return *reinterpret_cast<const uint32_t*>(&h);
  } else {
    const __half2 gh = *reinterpret_cast<const __half2*>(&g);
    const float g0 = __low2float(gh), g1 = __high2float(gh);
    const __half2 s = __floats2half2_rn(g0 / (1.0f + expf(-g0)), g1 / (1.0f + expf(-g1)));
    const __half2 h = __hmul2(s, *reinterpret_cast<const __half2*>(&u));
    return *reinterpret_cast<const uint32_t*>(&h);
  }
}

// vLLM's RMSNorm output for a word of two bf16 values: bf16((x * r) * w),
// the two products rounded in binary32 (vllm 0.22 rms_norm and
// fused_add_rms_norm, registered for model_executor/layers/layernorm.py;
// matched bit for bit on B200).
// The products run as packed mul.rn.f32x2: each lane rounds as mul.rn.f32.
__device__ __forceinline__ uint32_t rms_norm2(uint32_t x, uint32_t w, uint64_t r2) {
  const uint64_t xp = pack2(__uint_as_float(x << 16), __uint_as_float(x & 0xFFFF0000u));
  const uint64_t wp = pack2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
  float y0, y1;
  unpack2(mul2(mul2(xp, r2), wp), y0, y1);
  const __nv_bfloat162 h = __floats2bfloat162_rn(y0, y1);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ void consider(float mse, int raw, float& best, int& best_raw) {
  // strict '<': NaN never wins and ties keep the earlier (lower-index) candidate
  if (mse < best) {
    best = mse;
    best_raw = raw;
  }
}

__device__ __forceinline__ void consider_pair(uint64_t sse, float s2a, float s2b, int ra, int rb,
                                              float& best, int& best_raw) {
  float ma, mb;
  unpack2(mul2(sse, pack2(s2a, s2b)), ma, mb);
  consider(ma, ra, best, best_raw);
  consider(mb, rb, best, best_raw);
}

// Block |x| maximum straight from the 16-bit inputs.  max.xorsign.abs.{bf16,f16}x2
// keeps the larger magnitude of each lane and ignores NaN operands, like the
// reference's tl.maximum(tl.abs(a), tl.abs(b)).  Because rounding is
// monotonic, max_j |RN(x_j * g)| == RN(max_j |x_j| * |g|) for every block
// whose normalised values hold no NaN; a block holding a NaN has a NaN
// squared error for every candidate, so its scale does not depend on amax.
template <int kDType>
__device__ __forceinline__ float block_absmax_raw(const uint32_t (&w)[8]) {
  uint32_t a[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if constexpr (kDType == kDTypeBF16)
      asm("max.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(a[j]) : "r"(w[2 * j]), "r"(w[2 * j + 1]));
    else
      asm("max.xorsign.abs.f16x2 %0, %1, %2;" : "=r"(a[j]) : "r"(w[2 * j]), "r"(w[2 * j + 1]));
  }
  uint32_t b0, b1, c;
  if constexpr (kDType == kDTypeBF16) {
    asm("max.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(b0) : "r"(a[0]), "r"(a[1]));
    asm("max.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(b1) : "r"(a[2]), "r"(a[3]));
    asm("max.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(c) : "r"(b0), "r"(b1));
    const float lo = __uint_as_float((c & 0x7FFFu) << 16);
    const float hi = __uint_as_float(c & 0x7FFF0000u);
    return fmaxf(lo, hi);
  } else {
    asm("max.xorsign.abs.f16x2 %0, %1, %2;" : "=r"(b0) : "r"(a[0]), "r"(a[1]));
    asm("max.xorsign.abs.f16x2 %0, %1, %2;" : "=r"(b1) : "r"(a[2]), "r"(a[3]));
    asm("max.xorsign.abs.f16x2 %0, %1, %2;" : "=r"(c) : "r"(b0), "r"(b1));
    const float lo = __half2float(__ushort_as_half((unsigned short)(c & 0x7FFFu)));
    const float hi = __half2float(__ushort_as_half((unsigned short)((c >> 16) & 0x7FFFu)));
    return fmaxf(lo, hi);
  }
}

// Unsigned 32-bit division by the per-launch constant bpc_out:
// q = (umulhi(n, magic) + n) >> shift (Granlund & Montgomery 1994, round-up
// multiplier; the 33-bit sum is formed in 64 bits).
__device__ __forceinline__ uint32_t div_bpc(uint32_t n, uint32_t magic, uint32_t shift) {
  return (uint32_t)(((uint64_t)__umulhi(n, magic) + n) >> shift);
}

// Lexicographic (mse, index) minimum of two partial sweeps; index -1 = no
// winner.  Merging the per-lane winners of disjoint candidate subsets this way
// gives the sequential strict-'<' scan's result: the smallest mse, the lowest
// index among equal ones, NaN and +inf never winning.
__device__ __forceinline__ void merge_best(float& best, int& bi, float ob, int oi) {
  if (oi >= 0 && (bi < 0 || ob < best || (ob == best && oi < bi))) {
    best = ob;
    bi = oi;
  }
}

// kLanes lanes share one 16-element block when the grid would leave the GPU
// underfilled (decode-sized inputs): each sweeps the window candidates
// i = sub, sub + kLanes, ... and the lanes merge their winners.  kLanes = 1 is
// the throughput configuration: one lane per block, all 11 candidates.
// kSiluMul: the block's 16 values are h = silu(gate) * up, formed from the
// gate and up halves of a [rows, 2n] input (silu_mul2) instead of loaded.
template <int kVariant, int kMode, int kDType, bool kVec, int kLanes, bool kSiluMul = false,
          bool kNorm = false>
__global__ void __launch_bounds__(kThreads, kMinBlocksPerSm) quant_kernel(QuantParams p) {
  static_assert(kLanes == 1 || (kMode == kModeWindow && (kLanes == 2 || kLanes == 4)),
                "lane sharing applies to the 11-candidate window only");
  static_assert(!kSiluMul || kVec, "the SiLU-and-mul input is read with vector loads");
  static_assert(!kNorm || (kVec && kDType == kDTypeBF16), "the RMSNorm front end is bf16, vector");
  // A GEMM launched as this grid's programmatic dependent may start its
  // prologue now; it reads the codes only after griddepcontrol.wait, which
  // waits for this whole grid to finish.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  constexpr int kBlocksPerWarp = 32 / kLanes;
  // tab  : reciprocal and square of the E4M3 scale of every code 0..127
  //        (code 0 -> 1/0 = inf, used when no candidate wins)
  // tabw : the same for window position j = code + 3 with the code clamped to
  //        [1, 126], so candidate i of base code b is tabw[b + i]
  // tab_s: signed value of every byte (the reference variant's base test)
  __shared__ ScaleEntry tab[128];
  __shared__ ScaleEntry tabw[kWindowTab];
  __shared__ float tab_s[256];
  {
    const uint32_t c = threadIdx.x;  // kThreads == 256
    const float mag = e4m3_value(c & 0x7F);
    tab_s[c] = (c & 0x80) ? -mag : mag;
    if (c < 128) {
      float inv;
      asm("rcp.rn.f32 %0, %1;" : "=f"(inv) : "f"(mag));
      tab[c] = ScaleEntry{inv, mul_rn(mag, mag)};
    }
    if (c < kWindowTab) {
      const float s = e4m3_value((uint32_t)clamp_raw((int)c + kLower));
      float inv;
      asm("rcp.rn.f32 %0, %1;" : "=f"(inv) : "f"(s));
      tabw[c] = ScaleEntry{inv, mul_rn(s, s)};
    }
  }
  __syncthreads();
  if constexpr (kNorm) {
    // Launched as a programmatic dependent of rms_stats_kernel: the tables
    // above were built while it ran; r and the updated residual are read
    // only after it has finished and its writes are visible.
    asm volatile("griddepcontrol.wait;" ::: "memory");
  }

  const float gsi = __ldg(p.input_scale);
  const float abs_gsi = fabsf(gsi);
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t sub = lane % kLanes;  // this lane's share of the block's candidates
  const uint64_t warp = ((uint64_t)blockIdx.x * kThreads + threadIdx.x) >> 5;
  const uint64_t nwarps = ((uint64_t)gridDim.x * kThreads) >> 5;
  const uint32_t bpc_out = p.bpc_out, bpc_in = p.bpc_in;

  for (uint64_t first = warp * kBlocksPerWarp; first < p.nblocks;
       first += nwarps * kBlocksPerWarp) {
    const uint64_t b = first + lane / kLanes;
    const bool valid = b < p.nblocks;
    const uint32_t bb = (uint32_t)b;
    const uint32_t row = valid ? div_bpc(bb, p.div_magic, p.div_shift) : 0;
    const uint32_t col = valid ? bb - row * bpc_out : 0;
    const bool has_data = valid && col < bpc_in;

    // ---- load (bench_kernel/scalesweep_mse_nvfp4_utils.py:232-270)
    uint32_t w[8];
    if (has_data) {
      if constexpr (kSiluMul) {
        const uint16_t* gate = p.input + (uint64_t)row * p.silu_row_elems + (uint64_t)col * 16;
        uint32_t g[8], u[8];
        ld_block_v8(gate, g);
        ld_block_v8(gate + (uint64_t)bpc_in * 16, u);
#pragma unroll
        for (int j = 0; j < 8; ++j) w[j] = silu_mul2<kDType>(g[j], u[j]);
      } else if constexpr (kNorm) {
        const uint16_t* src = p.input + ((uint64_t)row * bpc_in + col) * 16;
        uint32_t xw[8], ww[8];
        ld_block_v8(src, xw);
        ld_block_v8(p.norm_weight + (uint64_t)col * 16, ww);
        const float r = __ldg(p.norm_rstd + row);
        const uint64_t r2 = pack2(r, r);
#pragma unroll
        for (int j = 0; j < 8; ++j) w[j] = rms_norm2(xw[j], ww[j], r2);
      } else {
        const uint16_t* src = p.input + ((uint64_t)row * bpc_in + col) * 16;
        if constexpr (kVec) {
          ld_block_v8(src, w);
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j)
            w[j] = (uint32_t)__ldg(src + 2 * j) | ((uint32_t)__ldg(src + 2 * j + 1) << 16);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) w[j] = 0u;
    }
    // ---- normalise: v = float(x) * gsi
    uint64_t vp[8];
    const uint64_t g2 = pack2(gsi, gsi);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float lo, hi;
      if constexpr (kDType == kDTypeBF16) {
        lo = __uint_as_float(w[j] << 16);
        hi = __uint_as_float(w[j] & 0xFFFF0000u);
      } else {
        lo = __half2float(__ushort_as_half((unsigned short)(w[j] & 0xFFFF)));
        hi = __half2float(__ushort_as_half((unsigned short)(w[j] >> 16)));
      }
      vp[j] = mul2(pack2(lo, hi), g2);
    }

    // ---- block amax (:209-229) and base code (:353-354; reference :347-351)
    float amax;
    if constexpr (kMode == kModeRtn) {
      float m[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float lo, hi;
        unpack2(vp[j], lo, hi);
        m[j] = fmaxf(fabsf(lo), fabsf(hi));
      }
      amax = fmaxf(fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3])),
                   fmaxf(fmaxf(m[4], m[5]), fmaxf(m[6], m[7])));
    } else {
      amax = mul_rn(block_absmax_raw<kDType>(w), abs_gsi);
    }
    const float base = mul_rn(amax, (float)(1.0 / 6.0));
    int base_raw = (int)e4m3_code(base);  // 0..127 for base >= 0 or NaN
    if constexpr (kVariant == kVariantReference) {
      base_raw -= (tab_s[base_raw] > base) ? 1 : 0;
    }
    base_raw = min(base_raw, 127);

    // ---- candidate sweep (:356-382)
    int best_raw = 0;
    if constexpr (kMode == kModeRtn) {
      best_raw = clamp_raw(base_raw);
    } else if constexpr (kMode == kModeWindow && kLanes > 1) {
      const ScaleEntry* wt = tabw + base_raw;  // candidate i -> wt[i]
      constexpr int kSlots = (kWindow + kLanes - 1) / kLanes;  // 3 (4 lanes) or 6 (2 lanes)
      float best = __uint_as_float(0x7F800000u);
      int bi = -1;
#pragma unroll
      for (int t = 0; t + 1 < kSlots; t += 2) {
        // the last lane's final slot may fall past the window: evaluated, never considered
        const int ia = (int)sub + t * kLanes, ib = (int)sub + (t + 1) * kLanes;
        const ScaleEntry ea = wt[min(ia, kWindow - 1)], eb = wt[min(ib, kWindow - 1)];
        float ma, mb;
        unpack2(mul2(sse_pair<kVariant>(vp, ea.inv, eb.inv), pack2(ea.s2, eb.s2)), ma, mb);
        if (ia < kWindow) consider(ma, ia, best, bi);
        if (ib < kWindow) consider(mb, ib, best, bi);
      }
      if constexpr (kSlots % 2) {
        const int i = (int)sub + (kSlots - 1) * kLanes;
        const ScaleEntry e = wt[min(i, kWindow - 1)];
        const float mm = mul_rn(sse_one<kVariant>(vp, e.inv), e.s2);
        if (i < kWindow) consider(mm, i, best, bi);
      }
#pragma unroll
      for (int off = 1; off < kLanes; off <<= 1)
        merge_best(best, bi, __shfl_xor_sync(0xFFFFFFFFu, best, off),
                   __shfl_xor_sync(0xFFFFFFFFu, bi, off));
      best_raw = bi < 0 ? 0 : clamp_raw(base_raw + kLower + bi);
    } else if constexpr (kMode == kModeWindow) {
      const ScaleEntry* wt = tabw + base_raw;  // candidate i -> wt[i]
      float best = __uint_as_float(0x7F800000u);
      int bi = -1;
#pragma unroll
      for (int i = 0; i + 1 < kWindow; i += 2) {
        const ScaleEntry ea = wt[i], eb = wt[i + 1];
        consider_pair(sse_pair<kVariant>(vp, ea.inv, eb.inv), ea.s2, eb.s2, i, i + 1, best, bi);
      }
      {
        const ScaleEntry e = wt[kWindow - 1];
        consider(mul_rn(sse_one<kVariant>(vp, e.inv), e.s2), kWindow - 1, best, bi);
      }
      best_raw = bi < 0 ? 0 : clamp_raw(base_raw + kLower + bi);
    } else {  // full range: every code 1..126 (:360-361)
      float best = __uint_as_float(0x7F800000u);
#pragma unroll 1
      for (int r = 1; r <= kMaxRaw; r += 2) {
        const ScaleEntry ea = tab[r], eb = tab[r + 1];
        consider_pair(sse_pair<kVariant>(vp, ea.inv, eb.inv), ea.s2, eb.s2, r, r + 1, best,
                      best_raw);
      }
    }

    // ---- final codes with the chosen scale (:399-421)
    const float inv = tab[best_raw].inv;
    const uint64_t i2 = pack2(inv, inv);
    float x[16];
#pragma unroll
    for (int j = 0; j < 8; ++j) unpack2(mul2(vp[j], i2), x[2 * j], x[2 * j + 1]);
    const uint32_t lo_word = e2m1x8(x[0], x[1], x[2], x[3], x[4], x[5], x[6], x[7]);
    const uint32_t hi_word = e2m1x8(x[8], x[9], x[10], x[11], x[12], x[13], x[14], x[15]);
    if (valid && sub == 0) {
      if constexpr (kVec) {
        st_v2(p.output + b * 8, lo_word, hi_word);
      } else {
        uint8_t* dst = p.output + b * 8;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          dst[j] = (uint8_t)(lo_word >> (8 * j));
          dst[4 + j] = (uint8_t)(hi_word >> (8 * j));
        }
      }
    }

    // ---- scale store (:384-397), swizzle (:23-43)
    uint64_t off;
    if (p.swizzled) {
      off = (uint64_t)(row >> 7) * ((uint64_t)p.bpc_pad * 128) + (uint64_t)(col >> 2) * 512 +
            (row & 31) * 16 + ((row & 127) >> 5) * 4 + (col & 3);
    } else {
      off = b;
    }
    // One byte per block.  The lanes of a warp hold consecutive columns, so
    // each group of four writes four consecutive bytes of a 512-byte atom:
    // the same sectors as gathering them into one word per group, without
    // the three shuffles (measured 1.4-2.5% faster on B200, identical bytes).
    if (valid && sub == 0) p.output_scale[off] = (uint8_t)best_raw;
  }
}

template <int kVariant, int kMode, int kDType, bool kVec, int kLanes, bool kSiluMul = false,
          bool kNorm = false>
cudaError_t launch_one(const QuantParams& p, int grid, cudaStream_t stream) {
  quant_kernel<kVariant, kMode, kDType, kVec, kLanes, kSiluMul, kNorm>
      <<<grid, kThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

// vLLM's RMSNorm statistics for one row per CTA.  vLLM launches one block of
// kVllmThreads threads per token; its thread t takes the 8-element vectors
// t, t + T, ... of the row, and a CUB block reduction (shuffle-down tree with
// offsets 1..16 in each warp, then the warp sums in order) adds the threads'
// partials.  The 256 threads here each play kVllmThreads / 256 of vLLM's
// threads, keeping every partial and every tree exactly as vLLM forms them.
// kAdd (fused_add_rms_norm): v = bf16(x + residual), written back to the
// residual; each vector's 8 squares are summed from zero before joining the
// thread's partial.  Otherwise (rms_norm) the squares chain straight into it.
template <int kVllmThreads, bool kAdd>
__global__ void __launch_bounds__(kThreads) rms_stats_kernel(const uint16_t* __restrict__ x,
                                                             uint16_t* __restrict__ residual,
                                                             uint32_t n, float eps,
                                                             float* __restrict__ rstd) {
  constexpr int kVirt = kVllmThreads / kThreads;  // vLLM threads per thread here
  static_assert(kVirt >= 1 && kVllmThreads % kThreads == 0 && 4 % kVirt == 0, "thread mapping");
  constexpr int kRounds = 4 / kVirt;        // strides of kVllmThreads vectors per pass
  constexpr int kLoads = kVirt * kRounds;   // 4 vectors of 16 bytes (per input) in flight
  // The quantizer launched after this grid may start (its table prologue)
  // once every CTA here has started.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __shared__ float warp_sums[kVllmThreads / 32];
  const uint64_t base = (uint64_t)blockIdx.x * n;
  const uint32_t chunks = n / 8, lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  float v[kVirt];
#pragma unroll
  for (int q = 0; q < kVirt; ++q) v[q] = 0.0f;
  // Each pass issues all its loads first, then adds them in.  Virtual thread
  // q still takes its vectors t, t + T, t + 2T, ... in that order, so every
  // partial is formed exactly as vLLM forms it.
  for (uint32_t first = 0; first < chunks; first += kRounds * kVllmThreads) {
    uint4 xa[kLoads], ra[kLoads];
#pragma unroll
    for (int i = 0; i < kLoads; ++i) {
      const uint32_t c = first + (i / kVirt) * kVllmThreads + threadIdx.x + (i % kVirt) * kThreads;
      if (c < chunks) {
        xa[i] = *reinterpret_cast<const uint4*>(x + base + (uint64_t)c * 8);
        if constexpr (kAdd) ra[i] = *reinterpret_cast<const uint4*>(residual + base + (uint64_t)c * 8);
      }
    }
#pragma unroll
    for (int i = 0; i < kLoads; ++i) {
      const int q = i % kVirt;
      const uint32_t c = first + (i / kVirt) * kVllmThreads + threadIdx.x + q * kThreads;
      if (c >= chunks) continue;
      const uint32_t xw[4] = {xa[i].x, xa[i].y, xa[i].z, xa[i].w};
      if constexpr (kAdd) {
        const uint32_t rw[4] = {ra[i].x, ra[i].y, ra[i].z, ra[i].w};
        uint32_t zw[4];
        float part = 0.0f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float z0 = add_rn(__uint_as_float(xw[k] << 16), __uint_as_float(rw[k] << 16));
          const float z1 = add_rn(__uint_as_float(xw[k] & 0xFFFF0000u),
                                  __uint_as_float(rw[k] & 0xFFFF0000u));
          const __nv_bfloat162 zb = __floats2bfloat162_rn(z0, z1);
          zw[k] = *reinterpret_cast<const uint32_t*>(&zb);
          const float a0 = __uint_as_float(zw[k] << 16), a1 = __uint_as_float(zw[k] & 0xFFFF0000u);
          part = fma_rn(a0, a0, part);
          part = fma_rn(a1, a1, part);
        }
        *reinterpret_cast<uint4*>(residual + base + (uint64_t)c * 8) =
            make_uint4(zw[0], zw[1], zw[2], zw[3]);
        v[q] = add_rn(v[q], part);
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float a0 = __uint_as_float(xw[k] << 16), a1 = __uint_as_float(xw[k] & 0xFFFF0000u);
          v[q] = fma_rn(a0, a0, v[q]);
          v[q] = fma_rn(a1, a1, v[q]);
        }
      }
    }
  }
#pragma unroll
  for (int q = 0; q < kVirt; ++q) {
    float w = v[q];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float other = __shfl_down_sync(0xFFFFFFFFu, w, o);
      if (lane + o < 32) w = add_rn(w, other);
    }
    if (lane == 0) warp_sums[wid + q * (kThreads / 32)] = w;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float acc = warp_sums[0];
    for (int k = 1; k < kVllmThreads / 32; ++k) acc = add_rn(acc, warp_sums[k]);
    float mean;
    asm("div.rn.f32 %0, %1, %2;" : "=f"(mean) : "f"(acc), "f"((float)n));
    rstd[blockIdx.x] = rsqrtf(add_rn(mean, eps));
  }
}

template <int kDType>
cudaError_t launch_silu_lanes(const QuantParams& p, int lanes, int grid, cudaStream_t s) {
  if (lanes == 4) return launch_one<kVariantMse, kModeWindow, kDType, true, 4, true>(p, grid, s);
  if (lanes == 2) return launch_one<kVariantMse, kModeWindow, kDType, true, 2, true>(p, grid, s);
  if (lanes != 1) return cudaErrorInvalidValue;
  return launch_one<kVariantMse, kModeWindow, kDType, true, 1, true>(p, grid, s);
}

// SiLU-and-mul alone: thread t handles 16-element chunks t, t + stride, ...,
// two per loop trip with all four 32-byte loads issued before either chunk is
// computed (one chunk per trip kept too few bytes in flight to stream HBM).
template <int kDType>
__global__ void __launch_bounds__(kThreads) silu_mul_kernel(const uint16_t* __restrict__ in,
                                                            uint16_t* __restrict__ out,
                                                            uint64_t nchunks, uint32_t cpr,
                                                            uint32_t magic, uint32_t shift) {
  const uint64_t stride = (uint64_t)gridDim.x * kThreads;
  for (uint64_t c0 = (uint64_t)blockIdx.x * kThreads + threadIdx.x; c0 < nchunks;
       c0 += 2 * stride) {
    const uint64_t c1 = c0 + stride;
    const bool two = c1 < nchunks;
    uint32_t g[2][8], u[2][8];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      if (t == 1 && !two) break;
      const uint64_t c = t ? c1 : c0;
      const uint32_t row = div_bpc((uint32_t)c, magic, shift), col = (uint32_t)c - row * cpr;
      const uint16_t* gate = in + (uint64_t)row * cpr * 32 + (uint64_t)col * 16;
      ld_block_v8(gate, g[t]);
      ld_block_v8(gate + (uint64_t)cpr * 16, u[t]);
    }
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      if (t == 1 && !two) break;
      uint32_t h[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) h[k] = silu_mul2<kDType>(g[t][k], u[t][k]);
      uint4* dst = reinterpret_cast<uint4*>(out + (t ? c1 : c0) * 16);
      dst[0] = make_uint4(h[0], h[1], h[2], h[3]);
      dst[1] = make_uint4(h[4], h[5], h[6], h[7]);
    }
  }
}

template <int kVariant, int kMode, int kDType>
cudaError_t launch_lanes(const QuantParams& p, bool vec, int lanes, int grid, cudaStream_t s) {
  if constexpr (kMode == kModeWindow) {
    if (vec && lanes == 4) return launch_one<kVariant, kMode, kDType, true, 4>(p, grid, s);
    if (vec && lanes == 2) return launch_one<kVariant, kMode, kDType, true, 2>(p, grid, s);
  }
  if (lanes != 1) return cudaErrorInvalidValue;
  return vec ? launch_one<kVariant, kMode, kDType, true, 1>(p, grid, s)
             : launch_one<kVariant, kMode, kDType, false, 1>(p, grid, s);
}

template <int kVariant, int kMode>
cudaError_t launch_dtype(const QuantParams& p, int dtype, bool vec, int lanes, int grid,
                         cudaStream_t s) {
  if (dtype == kDTypeBF16) return launch_lanes<kVariant, kMode, kDTypeBF16>(p, vec, lanes, grid, s);
  return launch_lanes<kVariant, kMode, kDTypeF16>(p, vec, lanes, grid, s);
}

}  // namespace

cudaError_t launch_silu_mul_quant(const QuantParams& p, int dtype, int lanes, int grid,
                                  cudaStream_t stream) {
  if (dtype == kDTypeBF16) return launch_silu_lanes<kDTypeBF16>(p, lanes, grid, stream);
  return launch_silu_lanes<kDTypeF16>(p, lanes, grid, stream);
}

// The RMSNorm quantizer is a programmatic dependent launch of the statistics
// kernel before it on the stream (it waits with griddepcontrol.wait).
template <int kLanes>
cudaError_t launch_norm_lanes(const QuantParams& p, int grid, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(
      &cfg, quant_kernel<kVariantMse, kModeWindow, kDTypeBF16, true, kLanes, false, true>, p);
}

cudaError_t launch_norm_quant(const QuantParams& p, int lanes, int grid, cudaStream_t stream) {
  if (lanes == 4) return launch_norm_lanes<4>(p, grid, stream);
  if (lanes == 2) return launch_norm_lanes<2>(p, grid, stream);
  if (lanes != 1) return cudaErrorInvalidValue;
  return launch_norm_lanes<1>(p, grid, stream);
}

cudaError_t launch_rms_stats(const uint16_t* x, uint16_t* residual, uint64_t rows, uint32_t n,
                             float eps, int vllm_threads, float* rstd, cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  const dim3 grid((unsigned)rows);
  if (vllm_threads == 1024) {
    if (residual)
      rms_stats_kernel<1024, true><<<grid, kThreads, 0, stream>>>(x, residual, n, eps, rstd);
    else
      rms_stats_kernel<1024, false><<<grid, kThreads, 0, stream>>>(x, residual, n, eps, rstd);
  } else if (vllm_threads == 256) {
    if (residual)
      rms_stats_kernel<256, true><<<grid, kThreads, 0, stream>>>(x, residual, n, eps, rstd);
    else
      rms_stats_kernel<256, false><<<grid, kThreads, 0, stream>>>(x, residual, n, eps, rstd);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_silu_mul(const uint16_t* input, uint16_t* output, uint64_t rows, uint32_t n,
                            int dtype, int device_sms, cudaStream_t stream) {
  const uint32_t cpr = n / 16;  // chunks per row
  const uint64_t nchunks = rows * cpr;
  if (nchunks == 0) return cudaSuccess;
  uint32_t magic = 0, shift = 0;
  make_divider(cpr, &magic, &shift);
  const uint64_t want = (nchunks + kThreads - 1) / kThreads;
  const uint64_t cap = (uint64_t)device_sms * 8;
  const int grid = (int)(want < cap ? want : cap);
  if (dtype == kDTypeBF16)
    silu_mul_kernel<kDTypeBF16><<<grid, kThreads, 0, stream>>>(input, output, nchunks, cpr, magic,
                                                              shift);
  else
    silu_mul_kernel<kDTypeF16><<<grid, kThreads, 0, stream>>>(input, output, nchunks, cpr, magic,
                                                             shift);
  return cudaGetLastError();
}

void make_divider(uint32_t d, uint32_t* magic, uint32_t* shift) {
  uint32_t l = 0;
  while ((1ull << l) < d) ++l;  // l = ceil(log2 d)
  *shift = l;
  *magic = (uint32_t)((((1ull << l) - d) << 32) / d + 1);
}

int quant_lanes_per_block(uint64_t nblocks, int device_sms, int mode, bool vec) {
  // Every lane of a shared block repeats the load, normalisation and final
  // encode, so sharing costs throughput.  It pays only while the input is so
  // small that the lanes still fit in one CTA per SM: the GPU is mostly idle
  // and the shorter per-lane sweep is pure latency gain (measured on B200:
  // M=16, K=4096 went from 2.98 to 2.54 us; M=128 got slower when shared).
  if (mode != kModeWindow || !vec) return 1;
  const uint64_t one_cta_per_sm = (uint64_t)device_sms * kThreads;
  if (nblocks * 4 <= one_cta_per_sm) return 4;
  if (nblocks * 2 <= one_cta_per_sm) return 2;
  return 1;
}

int quant_grid_size(uint64_t nblocks, int device_sms, int lanes) {
  // 8 warps per CTA, 32 / lanes blocks per warp per iteration; cap at 4
  // resident CTAs per SM and let the grid-stride loop cover the rest.
  const uint64_t per_cta = (uint64_t)(kThreads / lanes);
  uint64_t need = (nblocks + per_cta - 1) / per_cta;
  const uint64_t cap = (uint64_t)device_sms * kMinBlocksPerSm * 4;
  if (need > cap) need = cap;
  if (need < 1) need = 1;
  return (int)need;
}

cudaError_t launch_quant(const QuantParams& p, int variant, int mode, int dtype, bool vec,
                         int lanes, int grid, cudaStream_t stream) {
  if (variant == kVariantMse) {
    if (mode == kModeWindow)
      return launch_dtype<kVariantMse, kModeWindow>(p, dtype, vec, lanes, grid, stream);
    if (mode == kModeFullRange)
      return launch_dtype<kVariantMse, kModeFullRange>(p, dtype, vec, lanes, grid, stream);
    return launch_dtype<kVariantMse, kModeRtn>(p, dtype, vec, lanes, grid, stream);
  }
  if (variant == kVariantWeighted) {
    if (mode == kModeFullRange)
      return launch_dtype<kVariantWeighted, kModeFullRange>(p, dtype, vec, lanes, grid, stream);
    return launch_dtype<kVariantWeighted, kModeWindow>(p, dtype, vec, lanes, grid, stream);
  }
  return launch_dtype<kVariantReference, kModeWindow>(p, dtype, vec, lanes, grid, stream);
}

}  // namespace ssw
