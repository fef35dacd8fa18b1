// Global scale without any caller-provided or allocated device memory.
//
// ssw_global_scale_inv needs an 8-byte device workspace from its caller.
// Some callers cannot provide one: they own only the buffers they hand in.
// One example is a plugin inside an inference engine that plans every device
// byte ahead of time and exposes no workspace to plugins.  Another is a
// service that must keep its device memory footprint fixed once it has
// started, so that it cannot run out of memory later.
//
// This file serves them with a variant of the same reduction whose scratch
// is a file-scope __device__ array.  The array is created when the library is
// loaded on a GPU and kept until the process exits.  Its layout is one
// partial maximum per CTA plus a ticket word.  Each CTA reduces a fixed chunk
// of kStaticChunk elements, so one call handles at most
// kStaticSlots * kStaticChunk elements.
//
// Sharing rules:
//  * Every call on a device uses the same array.  Calls that overlap on the
//    GPU (different streams, or different host threads without ordering)
//    race on it and may return wrong results.  Order them on one stream.
//  * The ticket must start at zero.  It is cleared by a cudaMemsetAsync on
//    the caller's stream before every launch.  The partial slots need no
//    clearing: a call writes slots [0, grid) before the last CTA reads them.
//
// Host code may not use the array's name as a device address: on the host
// it denotes a shadow object, not GPU memory.  The first call on each device,
// with that device current, asks the runtime for the device address with
// cudaGetSymbolAddress and caches it.  That first call should happen before
// any stream capture begins.  The cached address belongs to the device's
// current context: after cudaDeviceReset on a device, this entry point must
// not be called on it again in the same process.
#include <cstdint>
#include <cstdio>
#include <mutex>

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../../include/scalesweep_b200.h"
#include "ptx.cuh"

namespace ssw {
void set_last_error(const char* msg);
}

namespace {

constexpr int kStaticThreads = 512;
constexpr uint32_t kStaticChunk = 32768;  // elements per CTA: 512 threads x 64
constexpr uint32_t kStaticSlots = 8192;   // CTAs per call
constexpr uint32_t kTicketWord = kStaticSlots;
constexpr uint64_t kStaticMaxElems = (uint64_t)kStaticSlots * kStaticChunk;  // 2^28

// 32 KiB of partial maxima + the ticket, padded to a 256-byte multiple.
static __device__ __align__(256) uint32_t g_amax_scratch[kStaticSlots + 64];

std::mutex g_setup_mutex;
uint32_t* g_scratch_ptr[64] = {nullptr};

__device__ __forceinline__ float abs_bits_to_float(uint32_t h, int dtype) {
  if (dtype == SSW_DTYPE_BF16) return __uint_as_float(h << 16);
  return __half2float(__ushort_as_half((unsigned short)h));
}

__global__ void __launch_bounds__(kStaticThreads)
    amax_static_kernel(const uint16_t* __restrict__ input, uint64_t numel, int dtype, int vec,
                       uint32_t* scratch, float fp8_max_times_6, float* scale_out,
                       float* amax_out) {
  const uint64_t lo = (uint64_t)blockIdx.x * kStaticChunk;
  const uint64_t hi = min(lo + kStaticChunk, numel);
  uint32_t m2 = 0;
  if (vec && hi - lo == kStaticChunk) {
    // 4 x 32-byte loads per thread, 16 KiB per load wave across the CTA
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      uint32_t w[8];
      ssw::ld_block_v8(input + lo + ((uint64_t)u * kStaticThreads + threadIdx.x) * 16, w);
#pragma unroll
      for (int j = 0; j < 8; ++j) m2 = __vmaxu2(m2, w[j] & 0x7FFF7FFFu);
    }
  } else {
    for (uint64_t i = lo + threadIdx.x; i < hi; i += kStaticThreads)
      m2 = __vmaxu2(m2, (uint32_t)__ldg(input + i) & 0x7FFFu);
  }
  uint32_t m = max(m2 & 0xFFFFu, m2 >> 16);
  m = __reduce_max_sync(0xFFFFFFFFu, m);
  __shared__ uint32_t warp_max[kStaticThreads / 32];
  __shared__ bool is_last;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) warp_max[wid] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t c = 0;
    for (int i = 0; i < kStaticThreads / 32; ++i) c = max(c, warp_max[i]);
    scratch[blockIdx.x] = c;
    __threadfence();
    is_last = atomicAdd(&scratch[kTicketWord], 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!is_last) return;
  // last CTA: fold every CTA's partial (read past L1), then publish
  __threadfence();
  uint32_t r = 0;
  for (uint32_t i = threadIdx.x; i < gridDim.x; i += kStaticThreads) r = max(r, __ldcg(&scratch[i]));
  r = __reduce_max_sync(0xFFFFFFFFu, r);
  if (lane == 0) warp_max[wid] = r;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t c = 0;
    for (int i = 0; i < kStaticThreads / 32; ++i) c = max(c, warp_max[i]);
    const float amax = abs_bits_to_float(c, dtype);
    float rcp;
    asm("rcp.rn.f32 %0, %1;" : "=f"(rcp) : "f"(amax));
    *scale_out = ssw::mul_rn(rcp, fp8_max_times_6);
    if (amax_out) *amax_out = amax;
    scratch[kTicketWord] = 0u;
  }
}

// Device address of g_amax_scratch on the current device (set up once per
// device).  On failure *step names the call that failed.
cudaError_t scratch_for_current_device(uint32_t** out, const char** step) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    *step = "cudaGetDevice";
    return e;
  }
  if (dev < 0 || dev >= 64) {
    *step = "device index >= 64 (the address cache holds 64 devices)";
    return cudaErrorInvalidDevice;
  }
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_amax_scratch);
    if (e != cudaSuccess) {
      *step = "cudaGetSymbolAddress of the static scratch";
      return e;
    }
    g_scratch_ptr[dev] = static_cast<uint32_t*>(p);
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

// "<prefix><step> failed: <cudaErrorName> (<description>)" into the last-error slot.
void report_cuda(const char* prefix, const char* step, cudaError_t e) {
  char msg[320];
  snprintf(msg, sizeof(msg), "%s%s failed: %s (%s)", prefix, step, cudaGetErrorName(e),
           cudaGetErrorString(e));
  ssw::set_last_error(msg);
}

}  // namespace

extern "C" {

int64_t ssw_global_scale_inv_noalloc_max_numel(void) { return (int64_t)kStaticMaxElems; }

int ssw_global_scale_inv_noalloc(const void* input, int input_dtype, int64_t numel,
                                 float fp8_max, float* input_scale_out, float* amax_out,
                                 void* stream) {
  ssw::set_last_error("");
  if (input_dtype != SSW_DTYPE_BF16 && input_dtype != SSW_DTYPE_F16) {
    ssw::set_last_error("global_scale_inv_noalloc: input dtype must be bf16 or f16");
    return SSW_ERR_INVALID_ARGUMENT;
  }
  if (numel <= 0 || !input || !input_scale_out) {
    ssw::set_last_error("global_scale_inv_noalloc: empty input or null pointer");
    return SSW_ERR_INVALID_ARGUMENT;
  }
  if ((uint64_t)numel > kStaticMaxElems) {
    ssw::set_last_error(
        "global_scale_inv_noalloc: more than 268435456 elements (8192 CTAs x 32768); the "
        "library's static scratch holds one partial per CTA -- use ssw_global_scale_inv with "
        "a workspace for larger tensors");
    return SSW_ERR_INVALID_ARGUMENT;
  }
  if (reinterpret_cast<uintptr_t>(input) % 2) {
    ssw::set_last_error("global_scale_inv_noalloc: misaligned input");
    return SSW_ERR_INVALID_ARGUMENT;
  }
  uint32_t* scratch = nullptr;
  const char* step = nullptr;
  cudaError_t e = scratch_for_current_device(&scratch, &step);
  if (e != cudaSuccess) {
    report_cuda("global_scale_inv_noalloc: ", step, e);
    return SSW_ERR_CUDA;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  e = cudaMemsetAsync(scratch + kTicketWord, 0, sizeof(uint32_t), s);
  if (e != cudaSuccess) {
    report_cuda("global_scale_inv_noalloc: ", "cudaMemsetAsync of the ticket", e);
    return SSW_ERR_CUDA;
  }
  const uint32_t grid = (uint32_t)(((uint64_t)numel + kStaticChunk - 1) / kStaticChunk);
  const int vec = (reinterpret_cast<uintptr_t>(input) % 32) == 0;
  amax_static_kernel<<<grid, kStaticThreads, 0, s>>>(static_cast<const uint16_t*>(input),
                                                     (uint64_t)numel, input_dtype, vec, scratch,
                                                     fp8_max * 6.0f, input_scale_out, amax_out);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    report_cuda("global_scale_inv_noalloc: ", "kernel launch", e);
    return SSW_ERR_CUDA;
  }
  return SSW_OK;
}

}  // extern "C"
