// C ABI of the scale-sweep NVFP4 library: argument validation, launch-shape
// selection and error reporting.  Declarations and contracts live in
// include/scalesweep_b200.h.
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>

#include <cuda_runtime.h>

#include "../../include/scalesweep_b200.h"
#include "gemm.cuh"
#include "quant.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(SSW_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

int device_sms(int* sms) {
  static int cache[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev >= 0 && dev < 64 && cache[dev] > 0) {
    *sms = cache[dev];
    return SSW_OK;
  }
  int v = 0;
  e = cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
  if (dev >= 0 && dev < 64) cache[dev] = v;
  *sms = v;
  return SSW_OK;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// silu_mul: `input` is [num_rows, 2n] and the quantized values are
// silu(input[:, :n]) * input[:, n:] (scalesweep_mse window only).
int quant_out(const char* name, int variant, int mode, const void* input, int input_dtype,
              int64_t num_rows, int64_t n, int64_t physical_n, const float* input_scale,
              uint8_t* output, uint8_t* output_scale, int swizzled, void* stream,
              bool silu_mul = false, const uint16_t* norm_weight = nullptr,
              const float* norm_rstd = nullptr) {
  g_last_error.clear();
  if (input_dtype != SSW_DTYPE_BF16 && input_dtype != SSW_DTYPE_F16)
    return fail(SSW_ERR_INVALID_ARGUMENT, "%s: input dtype must be bf16 or f16 (got %d)", name,
                input_dtype);
  if (num_rows < 0 || n < 0 || physical_n < 0)
    return fail(SSW_ERR_INVALID_ARGUMENT, "%s: negative size", name);
  if (n % 16)
    return fail(SSW_ERR_INVALID_ARGUMENT, "%s: the last input dimension must be a multiple of 16 (got %lld)",
                name, (long long)n);
  if (physical_n % 16)
    return fail(SSW_ERR_INVALID_ARGUMENT, "%s: padded_n must be a multiple of 16 (got %lld)", name,
                (long long)physical_n);
  if (physical_n < n)
    return fail(SSW_ERR_INVALID_ARGUMENT, "%s: padded_n (%lld) must be >= n (%lld)", name,
                (long long)physical_n, (long long)n);
  if (variant == ssw::kVariantReference && physical_n != n)
    return fail(SSW_ERR_INVALID_ARGUMENT,
                "%s: The reference ScaleSweep kernel does not support padded_n different from the "
                "input width.",
                name);
  const uint64_t bpc_out = (uint64_t)physical_n / 16, bpc_in = (uint64_t)n / 16;
  const uint64_t nblocks = (uint64_t)num_rows * bpc_out;
  if (nblocks == 0) return SSW_OK;
  if (nblocks >= (1ull << 32) || (uint64_t)num_rows >= (1ull << 31))
    return fail(SSW_ERR_INVALID_ARGUMENT, "%s: %llu blocks exceed the 2^32 per-call limit", name,
                (unsigned long long)nblocks);
  if (!output || !output_scale || !input_scale || (bpc_in > 0 && !input))
    return fail(SSW_ERR_INVALID_ARGUMENT, "%s: null pointer", name);
  if (!aligned(input, 2) || !aligned(input_scale, 4))
    return fail(SSW_ERR_INVALID_ARGUMENT, "%s: misaligned input or input_scale pointer", name);

  ssw::QuantParams p;
  p.input = static_cast<const uint16_t*>(input);
  p.input_scale = input_scale;
  p.output = output;
  p.output_scale = output_scale;
  p.nblocks = nblocks;
  p.bpc_in = (uint32_t)bpc_in;
  p.bpc_out = (uint32_t)bpc_out;
  p.bpc_pad = (uint32_t)((bpc_out + 3) / 4 * 4);
  ssw::make_divider(p.bpc_out, &p.div_magic, &p.div_shift);
  p.swizzled = swizzled ? 1 : 0;
  p.silu_row_elems = silu_mul ? 2 * (uint64_t)n : 0;
  p.norm_weight = norm_weight;
  p.norm_rstd = norm_rstd;
  const bool vec = aligned(input, 32) && aligned(output, 8);
  if (silu_mul && !vec)
    return fail(SSW_ERR_INVALID_ARGUMENT,
                "%s: input must be 32-byte aligned and output 8-byte aligned", name);

  int sms = 0;
  int st = device_sms(&sms);
  if (st != SSW_OK) return st;
  const int lanes = ssw::quant_lanes_per_block(nblocks, sms, mode, vec);
  const int grid = ssw::quant_grid_size(nblocks, sms, lanes);
  cudaError_t e =
      silu_mul      ? ssw::launch_silu_mul_quant(p, input_dtype, lanes, grid,
                                                 static_cast<cudaStream_t>(stream))
      : norm_weight ? ssw::launch_norm_quant(p, lanes, grid, static_cast<cudaStream_t>(stream))
                    : ssw::launch_quant(p, variant, mode, input_dtype, vec, lanes, grid,
                                        static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, name);
  return SSW_OK;
}

int amax_common(const char* name, const void* input, int input_dtype, int64_t numel,
                float fp8_max, float* scale_out, float* amax_out, void* workspace,
                void* stream) {
  g_last_error.clear();
  if (input_dtype != SSW_DTYPE_BF16 && input_dtype != SSW_DTYPE_F16)
    return fail(SSW_ERR_INVALID_ARGUMENT, "%s: input dtype must be bf16 or f16", name);
  if (numel <= 0)
    return fail(SSW_ERR_INVALID_ARGUMENT, "%s: the maximum of an empty tensor is undefined", name);
  if (!input || !workspace || (!scale_out && !amax_out))
    return fail(SSW_ERR_INVALID_ARGUMENT, "%s: null pointer", name);
  if (!aligned(input, 2) || !aligned(workspace, 4))
    return fail(SSW_ERR_INVALID_ARGUMENT, "%s: misaligned input or workspace", name);
  int sms = 0;
  int st = device_sms(&sms);
  if (st != SSW_OK) return st;
  ssw::AmaxParams p;
  p.input = static_cast<const uint16_t*>(input);
  p.numel = (uint64_t)numel;
  p.workspace = static_cast<uint32_t*>(workspace);
  p.amax_out = amax_out;
  p.scale_out = scale_out;
  p.fp8_max_times_6 = fp8_max * 6.0f;
  const bool vec = aligned(input, 32);
  cudaError_t e = ssw::launch_amax(p, input_dtype, vec, ssw::amax_grid_size(p.numel, sms),
                                   static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, name);
  return SSW_OK;
}

int gemm_shape_check(const char* name, int64_t m, int64_t n, int64_t k) {
  if (m < 0 || n <= 0 || k <= 0)
    return fail(SSW_ERR_INVALID_ARGUMENT, "%s: bad sizes m=%lld n=%lld k=%lld", name,
                (long long)m, (long long)n, (long long)k);
  if (k % 256)
    return fail(SSW_ERR_UNSUPPORTED, "%s: k must be a multiple of 256 (got %lld)", name,
                (long long)k);
  if (n % 64)
    return fail(SSW_ERR_UNSUPPORTED, "%s: n must be a multiple of 64 (got %lld)", name,
                (long long)n);
  if (m >= (1ll << 31) || n >= (1ll << 31) || k >= (1ll << 31))
    return fail(SSW_ERR_INVALID_ARGUMENT, "%s: sizes must be below 2^31", name);
  return SSW_OK;
}

int gemm_common(const char* name, const uint8_t* a, const uint8_t* b, const uint8_t* a_scale,
                const uint8_t* b_scale, const float* alpha, void* out, int64_t m, int64_t n,
                int64_t k, void* workspace, int64_t workspace_bytes, int* status, void* stream,
                bool dependent_launch) {
  int st = gemm_shape_check(name, m, n, k);
  if (st != SSW_OK || m == 0) return st;
  if (!a || !b || !a_scale || !b_scale || !alpha || !out)
    return fail(SSW_ERR_INVALID_ARGUMENT, "%s: null pointer", name);
  if (!aligned(a, 16) || !aligned(b, 16) || !aligned(a_scale, 16) || !aligned(b_scale, 16) ||
      !aligned(out, 16) || !aligned(alpha, 4) || (workspace && !aligned(workspace, 16)))
    return fail(SSW_ERR_INVALID_ARGUMENT, "%s: operands must be 16-byte aligned", name);
  int sms = 0;
  st = device_sms(&sms);
  if (st != SSW_OK) return st;
  int splits = ssw::gemm::choose_splits(m, n, k, sms);
  // without (enough) workspace the GEMM runs unsplit
  if (splits > 1 &&
      (!workspace || workspace_bytes < (int64_t)ssw::gemm::workspace_bytes(m, n, k, splits)))
    splits = 1;
  ssw::gemm::GemmArgs g{a, b, a_scale, b_scale, alpha, out, m, n, k, status, workspace};
  g.dependent_launch = dependent_launch;
  const char* why = "launch";
  cudaError_t e = ssw::gemm::launch(g, splits, static_cast<cudaStream_t>(stream), &why);
  if (e != cudaSuccess) return cuda_fail(e, why);
  return SSW_OK;
}

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

// Workspace of the fused quantize + GEMM call: A's codes, A's swizzled
// scales, then the GEMM's split-K scratch.
struct QuantGemmLayout {
  size_t codes, scales, gemm, total;
};
QuantGemmLayout quant_gemm_layout(int64_t m, int64_t n, int64_t k, int sms) {
  QuantGemmLayout l;
  l.codes = align256((size_t)m * (size_t)(k / 2));
  l.scales = align256((size_t)((m + 127) / 128 * 128) * (size_t)((k / 16 + 3) / 4 * 4));
  l.gemm = ssw::gemm::workspace_bytes(m, n, k, ssw::gemm::choose_splits(m, n, k, sms));
  l.total = l.codes + l.scales + l.gemm;
  return l;
}

}  // namespace

namespace ssw {
// Lets other translation units of the library report through ssw_last_error().
void set_last_error(const char* msg) { g_last_error = msg ? msg : ""; }
}  // namespace ssw

extern "C" {

int ssw_abi_version(void) { return SSW_ABI_VERSION; }

const char* ssw_status_string(int status) {
  switch (status) {
    case SSW_OK: return "ok";
    case SSW_ERR_INVALID_ARGUMENT: return "invalid argument";
    case SSW_ERR_UNSUPPORTED: return "unsupported";
    case SSW_ERR_CUDA: return "CUDA error";
    case SSW_ERR_TIMEOUT: return "device wait timed out";
    default: return "unknown status";
  }
}

const char* ssw_last_error(void) { return g_last_error.c_str(); }

int ssw_scalesweep_mse_nvfp4_quant_out(const void* input, int input_dtype, int64_t num_rows,
                                       int64_t n, int64_t physical_n, const float* input_scale,
                                       uint8_t* output, uint8_t* output_scale,
                                       int is_sf_swizzled_layout, void* stream) {
  return quant_out("scalesweep_mse_nvfp4_quant_out", ssw::kVariantMse, ssw::kModeWindow, input,
                   input_dtype, num_rows, n, physical_n, input_scale, output, output_scale,
                   is_sf_swizzled_layout, stream);
}

int ssw_scalesweep_mse128_nvfp4_quant_out(const void* input, int input_dtype, int64_t num_rows,
                                          int64_t n, int64_t physical_n,
                                          const float* input_scale, uint8_t* output,
                                          uint8_t* output_scale, int is_sf_swizzled_layout,
                                          void* stream) {
  return quant_out("scalesweep_mse128_nvfp4_quant_out", ssw::kVariantMse, ssw::kModeFullRange,
                   input, input_dtype, num_rows, n, physical_n, input_scale, output, output_scale,
                   is_sf_swizzled_layout, stream);
}

int ssw_scalesweep_mse_reference_nvfp4_quant_out(const void* input, int input_dtype,
                                                 int64_t num_rows, int64_t n, int64_t physical_n,
                                                 const float* input_scale, uint8_t* output,
                                                 uint8_t* output_scale,
                                                 int is_sf_swizzled_layout, void* stream) {
  return quant_out("scalesweep_mse_reference_nvfp4_quant_out", ssw::kVariantReference,
                   ssw::kModeWindow, input, input_dtype, num_rows, n, physical_n, input_scale,
                   output, output_scale, is_sf_swizzled_layout, stream);
}

int ssw_scalesweep_nvfp4_quant_out(const void* input, int input_dtype, int64_t num_rows,
                                   int64_t n, int64_t physical_n, const float* input_scale,
                                   uint8_t* output, uint8_t* output_scale,
                                   int is_sf_swizzled_layout, void* stream) {
  return quant_out("scalesweep_nvfp4_quant_out", ssw::kVariantWeighted, ssw::kModeWindow, input,
                   input_dtype, num_rows, n, physical_n, input_scale, output, output_scale,
                   is_sf_swizzled_layout, stream);
}

int ssw_scalesweep128_nvfp4_quant_out(const void* input, int input_dtype, int64_t num_rows,
                                      int64_t n, int64_t physical_n, const float* input_scale,
                                      uint8_t* output, uint8_t* output_scale,
                                      int is_sf_swizzled_layout, void* stream) {
  return quant_out("scalesweep128_nvfp4_quant_out", ssw::kVariantWeighted, ssw::kModeFullRange,
                   input, input_dtype, num_rows, n, physical_n, input_scale, output, output_scale,
                   is_sf_swizzled_layout, stream);
}

int ssw_silu_and_mul(const void* input, int input_dtype, int64_t num_rows, int64_t n,
                     void* output, void* stream) {
  g_last_error.clear();
  const char* name = "silu_and_mul";
  if (input_dtype != SSW_DTYPE_BF16 && input_dtype != SSW_DTYPE_F16)
    return fail(SSW_ERR_INVALID_ARGUMENT, "%s: input dtype must be bf16 or f16 (got %d)", name,
                input_dtype);
  if (num_rows < 0 || n < 0) return fail(SSW_ERR_INVALID_ARGUMENT, "%s: negative size", name);
  if (n % 16)
    return fail(SSW_ERR_INVALID_ARGUMENT, "%s: n must be a multiple of 16 (got %lld)", name,
                (long long)n);
  const uint64_t chunks = (uint64_t)num_rows * (uint64_t)(n / 16);
  if (chunks == 0) return SSW_OK;
  if (chunks >= (1ull << 32))
    return fail(SSW_ERR_INVALID_ARGUMENT, "%s: %llu 16-element chunks exceed the 2^32 per-call limit",
                name, (unsigned long long)chunks);
  if (!input || !output) return fail(SSW_ERR_INVALID_ARGUMENT, "%s: null pointer", name);
  if (!aligned(input, 32) || !aligned(output, 16))
    return fail(SSW_ERR_INVALID_ARGUMENT,
                "%s: input must be 32-byte aligned and output 16-byte aligned", name);
  int sms = 0;
  int st = device_sms(&sms);
  if (st != SSW_OK) return st;
  cudaError_t e = ssw::launch_silu_mul(static_cast<const uint16_t*>(input),
                                       static_cast<uint16_t*>(output), (uint64_t)num_rows,
                                       (uint32_t)n, input_dtype, sms,
                                       static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, name);
  return SSW_OK;
}

int ssw_silu_and_mul_scalesweep_mse_nvfp4_quant_out(const void* input, int input_dtype,
                                                    int64_t num_rows, int64_t n,
                                                    const float* input_scale, uint8_t* output,
                                                    uint8_t* output_scale,
                                                    int is_sf_swizzled_layout, void* stream) {
  return quant_out("silu_and_mul_scalesweep_mse_nvfp4_quant_out", ssw::kVariantMse,
                   ssw::kModeWindow, input, input_dtype, num_rows, n, n, input_scale, output,
                   output_scale, is_sf_swizzled_layout, stream, /*silu_mul=*/true);
}

int ssw_rms_norm_scalesweep_mse_nvfp4_quant_out(const void* input, void* residual,
                                                const void* weight, float eps, int64_t num_rows,
                                                int64_t n, const float* input_scale,
                                                uint8_t* output, uint8_t* output_scale,
                                                int is_sf_swizzled_layout, float* rstd_workspace,
                                                void* stream) {
  g_last_error.clear();
  const char* name = "rms_norm_scalesweep_mse_nvfp4_quant_out";
  if (num_rows < 0 || n <= 0) return fail(SSW_ERR_INVALID_ARGUMENT, "%s: bad sizes", name);
  if (n % 16)
    return fail(SSW_ERR_INVALID_ARGUMENT, "%s: n must be a multiple of 16 (got %lld)", name,
                (long long)n);
  // every check the quantizer makes is made here too, before the statistics
  // kernel runs: a call that fails leaves the residual untouched
  if (num_rows >= (1ll << 31) || n >= (1ll << 31) ||
      (uint64_t)num_rows * (uint64_t)(n / 16) >= (1ull << 32))
    return fail(SSW_ERR_INVALID_ARGUMENT, "%s: sizes must be below 2^31 and blocks below 2^32",
                name);
  if (num_rows == 0) return SSW_OK;
  if (!input || !weight || !rstd_workspace || !input_scale || !output || !output_scale)
    return fail(SSW_ERR_INVALID_ARGUMENT, "%s: null pointer", name);
  if (!aligned(input, 32) || !aligned(weight, 32) || (residual && !aligned(residual, 32)) ||
      !aligned(rstd_workspace, 4) || !aligned(input_scale, 4) || !aligned(output, 8))
    return fail(SSW_ERR_INVALID_ARGUMENT,
                "%s: input, residual and weight must be 32-byte aligned, output 8-byte, "
                "input_scale and rstd_workspace 4-byte", name);
  int sms = 0;
  const int sst = device_sms(&sms);
  if (sst != SSW_OK) return sst;
  // vLLM launches 1024 threads per token below 256 tokens and 256 from there
  const int vllm_threads = num_rows < 256 ? 1024 : 256;
  cudaError_t e = ssw::launch_rms_stats(static_cast<const uint16_t*>(input),
                                        static_cast<uint16_t*>(residual), (uint64_t)num_rows,
                                        (uint32_t)n, eps, vllm_threads, rstd_workspace,
                                        static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, name);
  // the normalised values come from the updated residual in the fused-add form
  return quant_out(name, ssw::kVariantMse, ssw::kModeWindow, residual ? residual : input,
                   SSW_DTYPE_BF16, num_rows, n, n, input_scale, output, output_scale,
                   is_sf_swizzled_layout, stream, false, static_cast<const uint16_t*>(weight),
                   rstd_workspace);
}

int ssw_rtn_nvfp4_quant_out(const void* input, int input_dtype, int64_t num_rows, int64_t n,
                            int64_t physical_n, const float* input_scale, uint8_t* output,
                            uint8_t* output_scale, int is_sf_swizzled_layout, void* stream) {
  return quant_out("rtn_nvfp4_quant_out", ssw::kVariantMse, ssw::kModeRtn, input, input_dtype,
                   num_rows, n, physical_n, input_scale, output, output_scale,
                   is_sf_swizzled_layout, stream);
}

int64_t ssw_nvfp4_gemm_workspace_bytes(int64_t m, int64_t n, int64_t k) {
  int sms = 0;
  if (m <= 0 || n <= 0 || k <= 0 || n % 64 || k % 256 || device_sms(&sms) != SSW_OK) return 0;
  return (int64_t)ssw::gemm::workspace_bytes(m, n, k, ssw::gemm::choose_splits(m, n, k, sms));
}

int ssw_nvfp4_gemm(const uint8_t* a, const uint8_t* b, const uint8_t* a_scale,
                   const uint8_t* b_scale, const float* alpha, void* out, int64_t m, int64_t n,
                   int64_t k, void* workspace, int64_t workspace_bytes, int* status,
                   void* stream) {
  g_last_error.clear();
  return gemm_common("nvfp4_gemm", a, b, a_scale, b_scale, alpha, out, m, n, k, workspace,
                     workspace_bytes, status, stream, false);
}

int ssw_nvfp4_gemm_dependent(const uint8_t* a, const uint8_t* b, const uint8_t* a_scale,
                             const uint8_t* b_scale, const float* alpha, void* out, int64_t m,
                             int64_t n, int64_t k, void* workspace, int64_t workspace_bytes,
                             int* status, void* stream) {
  g_last_error.clear();
  return gemm_common("nvfp4_gemm_dependent", a, b, a_scale, b_scale, alpha, out, m, n, k,
                     workspace, workspace_bytes, status, stream, true);
}

int ssw_nvfp4_mma_rate_probe(int bn, int iters, long long* cycles_out, int* status,
                             void* stream) {
  g_last_error.clear();
  if (bn != 128 && bn != 256)
    return fail(SSW_ERR_INVALID_ARGUMENT, "nvfp4_mma_rate_probe: bn must be 128 or 256");
  if (iters <= 0 || iters > (1 << 14))
    return fail(SSW_ERR_INVALID_ARGUMENT, "nvfp4_mma_rate_probe: iters must be in [1, 16384]");
  if (!cycles_out) return fail(SSW_ERR_INVALID_ARGUMENT, "nvfp4_mma_rate_probe: null pointer");
  int sms = 0;
  int st = device_sms(&sms);
  if (st != SSW_OK) return st;
  cudaError_t e = ssw::gemm::launch_mma_peak(bn, iters, sms, cycles_out, status,
                                             static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "nvfp4_mma_rate_probe launch");
  return SSW_OK;
}

int64_t ssw_nvfp4_quant_gemm_workspace_bytes(int64_t m, int64_t n, int64_t k) {
  int sms = 0;
  if (m <= 0 || n <= 0 || k <= 0 || n % 64 || k % 256 || device_sms(&sms) != SSW_OK) return 0;
  return (int64_t)quant_gemm_layout(m, n, k, sms).total;
}

int ssw_nvfp4_quant_gemm(const void* x, int x_dtype, const float* x_scale, const uint8_t* b,
                         const uint8_t* b_scale, const float* alpha, void* out, int64_t m,
                         int64_t n, int64_t k, void* workspace, int64_t workspace_bytes,
                         int* status, void* stream) {
  g_last_error.clear();
  const char* name = "nvfp4_quant_gemm";
  int st = gemm_shape_check(name, m, n, k);
  if (st != SSW_OK || m == 0) return st;
  int sms = 0;
  st = device_sms(&sms);
  if (st != SSW_OK) return st;
  const QuantGemmLayout lay = quant_gemm_layout(m, n, k, sms);
  if (!workspace || !aligned(workspace, 256) || workspace_bytes < (int64_t)lay.total)
    return fail(SSW_ERR_INVALID_ARGUMENT,
                "%s: workspace must be 256-byte aligned and hold %llu bytes", name,
                (unsigned long long)lay.total);
  uint8_t* codes = static_cast<uint8_t*>(workspace);
  uint8_t* scales = codes + lay.codes;
  st = quant_out(name, ssw::kVariantMse, ssw::kModeWindow, x, x_dtype, m, k, k, x_scale, codes,
                 scales, 1, stream);
  if (st != SSW_OK) return st;
  return gemm_common(name, codes, b, scales, b_scale, alpha, out, m, n, k, scales + lay.scales,
                     (int64_t)lay.gemm, status, stream, /*dependent_launch=*/true);
}

int64_t ssw_absmax_workspace_bytes(void) { return 8; }

int ssw_absmax(const void* input, int input_dtype, int64_t numel, float* amax_out,
               void* workspace, void* stream) {
  return amax_common("absmax", input, input_dtype, numel, 0.0f, nullptr, amax_out, workspace,
                     stream);
}

int ssw_global_scale_from_amax(const float* amax, float fp8_max, float* input_scale_out,
                               void* stream) {
  g_last_error.clear();
  if (!amax || !input_scale_out)
    return fail(SSW_ERR_INVALID_ARGUMENT, "global_scale_from_amax: null pointer");
  cudaError_t e = ssw::launch_scale_from_amax(amax, fp8_max * 6.0f, input_scale_out,
                                              static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "global_scale_from_amax");
  return SSW_OK;
}

int ssw_global_scale_inv(const void* input, int input_dtype, int64_t numel, float fp8_max,
                         float* input_scale_out, float* amax_out, void* workspace,
                         void* stream) {
  if (!input_scale_out) {
    g_last_error = "global_scale_inv: null input_scale_out";
    return SSW_ERR_INVALID_ARGUMENT;
  }
  return amax_common("global_scale_inv", input, input_dtype, numel, fp8_max, input_scale_out,
                     amax_out, workspace, stream);
}

}  // extern "C"
