// Internal launch interface of the quantizer kernels (not part of the C ABI).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

namespace ssw {

enum { kVariantMse = 0, kVariantReference = 1, kVariantWeighted = 2 };
enum { kModeWindow = 0, kModeFullRange = 1, kModeRtn = 2 };
enum { kDTypeBF16 = 0, kDTypeF16 = 1 };

struct QuantParams {
  const uint16_t* input;      // [rows, bpc_in*16] 16-bit floats
  const float* input_scale;   // one float: 6*fp8_max/amax
  uint8_t* output;            // [rows, bpc_out*8] packed codes
  uint8_t* output_scale;      // swizzled or linear scale bytes
  uint64_t nblocks;           // rows * bpc_out (< 2^32)
  uint32_t bpc_in;            // input blocks per row  (n / 16)
  uint32_t bpc_out;           // output blocks per row (physical_n / 16)
  uint32_t bpc_pad;           // round_up(bpc_out, 4)
  uint32_t div_magic;         // row = (umulhi(b, div_magic) + b) >> div_shift == b / bpc_out
  uint32_t div_shift;
  int swizzled;
  uint64_t silu_row_elems;    // SiLU-and-mul input only: elements per input row (2 * n)
  const uint16_t* norm_weight;  // RMSNorm front end only: bf16 weight [n]
  const float* norm_rstd;       // RMSNorm front end only: 1/rms of each row [rows]
};

// Lanes sharing one block (1, 2 or 4): more than 1 only for the 11-candidate
// window with vector loads, when nblocks x lanes fits one wave.
int quant_lanes_per_block(uint64_t nblocks, int device_sms, int mode, bool vec);
int quant_grid_size(uint64_t nblocks, int device_sms, int lanes);
// Round-up multiplier for unsigned 32-bit division by d >= 1.
void make_divider(uint32_t d, uint32_t* magic, uint32_t* shift);
cudaError_t launch_quant(const QuantParams& p, int variant, int mode, int dtype, bool vec,
                         int lanes, int grid, cudaStream_t stream);
// The "scalesweep_mse" window quantizer on h = silu(gate) * up of an input
// [rows, 2n] (gate = columns 0..n-1, up = n..2n-1), computed on the fly as
// vLLM's silu_and_mul computes it.  Vector loads only (input 32-byte aligned).
cudaError_t launch_silu_mul_quant(const QuantParams& p, int dtype, int lanes, int grid,
                                  cudaStream_t stream);
// The "scalesweep_mse" window quantizer on h = bf16(x * rstd[row] * weight)
// of a bf16 input [rows, n] (RMSNorm's output, formed on the fly).  Vector
// loads only; rstd from launch_rms_stats, which must be the launch just
// before on the same stream: this grid is its programmatic dependent.
cudaError_t launch_norm_quant(const QuantParams& p, int lanes, int grid, cudaStream_t stream);
// vLLM's RMSNorm statistics, per row: rstd[row] = rsqrtf(mean(v^2) + eps) in
// the reduction order of vLLM's rms_norm (residual == nullptr, v = x) or of
// its fused_add_rms_norm (v = bf16(x + residual), written back to residual).
// vllm_threads is the block size vLLM would launch (1024 or 256).
cudaError_t launch_rms_stats(const uint16_t* x, uint16_t* residual, uint64_t rows, uint32_t n,
                             float eps, int vllm_threads, float* rstd, cudaStream_t stream);
// The SiLU-and-mul alone: output [rows, n] = silu(input[:, :n]) * input[:, n:].
cudaError_t launch_silu_mul(const uint16_t* input, uint16_t* output, uint64_t rows, uint32_t n,
                            int dtype, int device_sms, cudaStream_t stream);

// amax / global scale
struct AmaxParams {
  const uint16_t* input;
  uint64_t numel;
  uint32_t* workspace;  // [0] = max |x| bits, [1] = finished-CTA counter
  float* amax_out;      // may be null (fused path)
  float* scale_out;     // may be null (plain amax path)
  float fp8_max_times_6;
};
int amax_grid_size(uint64_t numel, int device_sms);
cudaError_t launch_amax(const AmaxParams& p, int dtype, bool vec, int grid, cudaStream_t stream);
cudaError_t launch_scale_from_amax(const float* amax, float fp8_max_times_6, float* out,
                                   cudaStream_t stream);

}  // namespace ssw
