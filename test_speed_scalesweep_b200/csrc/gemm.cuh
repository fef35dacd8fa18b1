// Internal launch interface of the NVFP4 GEMM (not part of the C ABI).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

namespace ssw {
namespace gemm {

struct GemmArgs {
  const uint8_t* a;    // [m, k/2] E2M1 codes
  const uint8_t* b;    // [n, k/2] E2M1 codes
  const uint8_t* sfa;  // swizzled E4M3 scales of A ([round_up(m,128), k/16])
  const uint8_t* sfb;  // swizzled E4M3 scales of B ([n, k/16])
  const float* alpha;  // one device float
  void* out;           // [m, n] bf16
  int64_t m, n, k;
  int* status;         // optional device int: set non-zero if a bounded wait gave up
  void* workspace;     // split-K partials + tile tickets (workspace_bytes(...)), 16B aligned
  // Launched right after the kernel that writes a / sfa (programmatic
  // dependent launch): the GEMM's prologue and first weight loads overlap
  // that kernel's tail; A is read only after griddepcontrol.wait.
  bool dependent_launch = false;
};

size_t smem_bytes();
// Split-K factor for a problem on this many SMs (1 = no split).
int choose_splits(int64_t m, int64_t n, int64_t k, int device_sms);
size_t workspace_bytes(int64_t m, int64_t n, int64_t k, int splits);
cudaError_t launch(const GemmArgs& g, int splits, cudaStream_t stream, const char** why);
// Dense FP4 tensor-core rate probe: `ctas` CTAs (one per SM) each issue
// 4 * iters MMAs of 128 x bn x 64 (bn 128 or 256) and write their elapsed
// SM clock cycles (-1 if the bounded completion wait gave up).
cudaError_t launch_mma_peak(int bn, int iters, int ctas, long long* cycles, int* status,
                            cudaStream_t stream);

}  // namespace gemm
}  // namespace ssw
