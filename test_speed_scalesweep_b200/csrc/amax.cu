// Per-tensor |x| maximum and the global-scale multiplier for sm_100a.
//
// The reduction runs on the 16-bit patterns: for bf16 and f16 alike,
// (h & 0x7FFF) orders exactly like |x| (sign-magnitude formats), and every
// NaN pattern sorts above +inf, so an unsigned max returns NaN whenever the
// tensor holds one -- the behaviour of torch's x.abs().max() that
// bench_kernel/test_kernel_latency.py:65-70 relies on.  Two lanes are reduced
// per SIMD instruction (__vmaxu2).  Each CTA folds its maximum into
// workspace[0] with one atomicMax; the last CTA to finish (ticket in
// workspace[1]) converts it to float and, on the fused path, evaluates
// (fp8_max*6)/amax the way torch does: reciprocal rounded, then the product
// rounded.  No CTA ever waits for another.
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include "ptx.cuh"
#include "quant.cuh"

namespace ssw {

namespace {

constexpr int kAmaxThreads = 512;

__device__ __forceinline__ float abs_bits_to_float(uint32_t h, int dtype) {
  if (dtype == kDTypeBF16) return __uint_as_float(h << 16);
  return __half2float(__ushort_as_half((unsigned short)h));
}

__device__ __forceinline__ float torch_scale(float amax, float c) {
  float r;
  asm("rcp.rn.f32 %0, %1;" : "=f"(r) : "f"(amax));
  return mul_rn(r, c);
}

template <bool kVec>
__global__ void __launch_bounds__(kAmaxThreads) amax_kernel(AmaxParams p, int dtype) {
  uint32_t m2 = 0;  // two 16-bit running maxima
  const uint64_t tid = (uint64_t)blockIdx.x * kAmaxThreads + threadIdx.x;
  const uint64_t nthreads = (uint64_t)gridDim.x * kAmaxThreads;
  uint64_t scalar_from = 0;
  if constexpr (kVec) {
    const uint64_t nvec = p.numel / 16;  // 32-byte groups
    const uint64_t step = nthreads;
    uint64_t i = tid;
    for (; i + 3 * step < nvec; i += 4 * step) {
      uint32_t w[4][8];
#pragma unroll
      for (int u = 0; u < 4; ++u) ld_block_v8(p.input + (i + u * step) * 16, w[u]);
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int j = 0; j < 8; ++j) m2 = __vmaxu2(m2, w[u][j] & 0x7FFF7FFFu);
    }
    for (; i < nvec; i += step) {
      uint32_t w[8];
      ld_block_v8(p.input + i * 16, w);
#pragma unroll
      for (int j = 0; j < 8; ++j) m2 = __vmaxu2(m2, w[j] & 0x7FFF7FFFu);
    }
    scalar_from = nvec * 16;
  }
  for (uint64_t i = scalar_from + tid; i < p.numel; i += nthreads)
    m2 = __vmaxu2(m2, (uint32_t)__ldg(p.input + i) & 0x7FFFu);

  uint32_t m = max(m2 & 0xFFFFu, m2 >> 16);
  m = __reduce_max_sync(0xFFFFFFFFu, m);
  __shared__ uint32_t warp_max[kAmaxThreads / 32];
  __shared__ bool is_last;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) warp_max[wid] = m;
  __syncthreads();
  if (wid == 0) {
    m = lane < kAmaxThreads / 32 ? warp_max[lane] : 0u;
    m = __reduce_max_sync(0xFFFFFFFFu, m);
    if (lane == 0) {
      atomicMax(&p.workspace[0], m);
      __threadfence();
      const uint32_t ticket = atomicAdd(&p.workspace[1], 1u);
      is_last = ticket == gridDim.x - 1;
    }
  }
  __syncthreads();
  if (is_last && threadIdx.x == 0) {
    __threadfence();
    const uint32_t bits = atomicOr(&p.workspace[0], 0u);
    const float amax = abs_bits_to_float(bits, dtype);
    if (p.amax_out) *p.amax_out = amax;
    if (p.scale_out) *p.scale_out = torch_scale(amax, p.fp8_max_times_6);
  }
}

__global__ void scale_from_amax_kernel(const float* amax, float c, float* out) {
  *out = torch_scale(*amax, c);
}

}  // namespace

int amax_grid_size(uint64_t numel, int device_sms) {
  const uint64_t groups = numel / 16 + 1;
  uint64_t need = (groups + kAmaxThreads - 1) / kAmaxThreads;
  const uint64_t cap = (uint64_t)device_sms * 4;
  if (need > cap) need = cap;
  if (need < 1) need = 1;
  return (int)need;
}

cudaError_t launch_amax(const AmaxParams& p, int dtype, bool vec, int grid, cudaStream_t stream) {
  cudaError_t e = cudaMemsetAsync(p.workspace, 0, 2 * sizeof(uint32_t), stream);
  if (e != cudaSuccess) return e;
  if (vec)
    amax_kernel<true><<<grid, kAmaxThreads, 0, stream>>>(p, dtype);
  else
    amax_kernel<false><<<grid, kAmaxThreads, 0, stream>>>(p, dtype);
  return cudaGetLastError();
}

cudaError_t launch_scale_from_amax(const float* amax, float c, float* out, cudaStream_t stream) {
  scale_from_amax_kernel<<<1, 1, 0, stream>>>(amax, c, out);
  return cudaGetLastError();
}

}  // namespace ssw
