/*
 * scalesweep_b200 -- C ABI of the B200 (sm_100a) scale-sweep NVFP4 quantizer.
 *
 * Plain pointers and sizes only.  Every data pointer is a CUDA device pointer
 * of the current device unless stated otherwise; `stream` is a cudaStream_t
 * passed as void* (NULL = legacy default stream).  All entry points are
 * asynchronous with respect to the host, enqueue on `stream`, never allocate,
 * never synchronise, and return an ssw_status.  On failure a message is
 * available from ssw_last_error() (thread-local).
 *
 * Output layout (identical to the reference):
 *   output       uint8 [num_rows, physical_n/2]; element 2j in the low nibble,
 *                element 2j+1 in the high nibble of byte j (E2M1 codes).
 *   output_scale swizzled: bytes of [round_up(num_rows,128), round_up(physical_n/16,4)]
 *                in the CUTLASS 128x4 scale-factor layout; linear: [num_rows,
 *                physical_n/16].  Bytes of the swizzled padding (rows >= num_rows,
 *                block columns >= physical_n/16) are left untouched.
 *   input_scale  one float on the device: the multiplier 6*fp8_max/amax that
 *                the reference calls "global_scale_inv".
 */
#ifndef SCALESWEEP_B200_H_
#define SCALESWEEP_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SSW_ABI_VERSION 1

typedef enum {
  SSW_OK = 0,
  SSW_ERR_INVALID_ARGUMENT = 1, /* shape, dtype, alignment or pointer problem */
  SSW_ERR_UNSUPPORTED = 2,      /* valid request the library does not implement */
  SSW_ERR_CUDA = 3,             /* a CUDA runtime call failed (launch, attribute) */
  SSW_ERR_TIMEOUT = 4           /* a bounded device-side wait gave up */
} ssw_status;

typedef enum { SSW_DTYPE_BF16 = 0, SSW_DTYPE_F16 = 1 } ssw_dtype;

/* Library / error reporting. */
int ssw_abi_version(void);
const char* ssw_status_string(int status);
const char* ssw_last_error(void);

/*
 * Scale-sweep MSE quantizer, "scalesweep_mse" backend: round-to-nearest base
 * code, 11 candidates [base-3, base+7] clamped to [1,126], fp32 SSE as a
 * sequential FMA chain over elements 0..15, strict '<' argmin (ties -> lowest
 * candidate).  physical_n >= n: block columns past n/16 are quantized as zero
 * blocks (the reference's padded_n path).
 * Replaces bench_kernel/scalesweep_mse_nvfp4_utils.py:462-477
 * (scalesweep_mse_nvfp4_quant_out) and its launcher :424-459.
 */
int ssw_scalesweep_mse_nvfp4_quant_out(const void* input, int input_dtype, int64_t num_rows,
                                       int64_t n, int64_t physical_n, const float* input_scale,
                                       uint8_t* output, uint8_t* output_scale,
                                       int is_sf_swizzled_layout, void* stream);

/*
 * Full-range "scalesweep_mse128": candidates are every E4M3 code 1..126.
 * Replaces bench_kernel/scalesweep_mse_nvfp4_utils.py:480-495
 * (scalesweep_mse128_nvfp4_quant_out).
 */
int ssw_scalesweep_mse128_nvfp4_quant_out(const void* input, int input_dtype, int64_t num_rows,
                                          int64_t n, int64_t physical_n,
                                          const float* input_scale, uint8_t* output,
                                          uint8_t* output_scale, int is_sf_swizzled_layout,
                                          void* stream);

/*
 * "scalesweep_mse_reference" variant: base code rounded DOWN (largest E4M3
 * <= amax/6), SSE as the pairwise tree ((s01+s23)+(s45+s67))+((s89+sAB)+(sCD+sEF)).
 * physical_n must equal n (SSW_ERR_INVALID_ARGUMENT otherwise), as in the reference.
 * Replaces bench_kernel/scalesweep_mse_reference_nvfp4_utils.py:412-445
 * (scalesweep_mse_nvfp4_quant_out).
 */
int ssw_scalesweep_mse_reference_nvfp4_quant_out(const void* input, int input_dtype,
                                                 int64_t num_rows, int64_t n, int64_t physical_n,
                                                 const float* input_scale, uint8_t* output,
                                                 uint8_t* output_scale,
                                                 int is_sf_swizzled_layout, void* stream);

/*
 * Importance-weighted "scalesweep" backend (window) and "scalesweep128"
 * (full range 1..126): same sweep, but every squared error is rounded on its
 * own and then summed in element order, because the reference multiplies it
 * by a per-column importance weight first (always 1 from its host code).
 * Replaces bench_kernel/scalesweep_nvfp4_utils.py:344-368 (and the launcher :305-341)
 * (scalesweep_nvfp4_quant_out, scalesweep128_nvfp4_quant_out).
 */
int ssw_scalesweep_nvfp4_quant_out(const void* input, int input_dtype, int64_t num_rows,
                                   int64_t n, int64_t physical_n, const float* input_scale,
                                   uint8_t* output, uint8_t* output_scale,
                                   int is_sf_swizzled_layout, void* stream);
int ssw_scalesweep128_nvfp4_quant_out(const void* input, int input_dtype, int64_t num_rows,
                                      int64_t n, int64_t physical_n, const float* input_scale,
                                      uint8_t* output, uint8_t* output_scale,
                                      int is_sf_swizzled_layout, void* stream);

/*
 * SiLU-and-mul, the producer of the MLP down projection's activation:
 *   output[r, c] = silu(input[r, c]) * input[r, n + c],  input [num_rows, 2n],
 * output [num_rows, n], both bf16 or both f16.  silu(g) = g / (1 + e^-g) in
 * binary32 (IEEE division), rounded to the input type; the product is rounded
 * once.  Bit for bit what vLLM's silu_and_mul computes (vllm 0.22
 * torch.ops._C.silu_and_mul, model_executor/layers/activation.py:117-147),
 * checked on every bf16 and f16 gate value.  n % 16 == 0, input 32-byte and
 * output 16-byte aligned, num_rows * n / 16 < 2^32.
 */
int ssw_silu_and_mul(const void* input, int input_dtype, int64_t num_rows, int64_t n,
                     void* output, void* stream);

/*
 * SiLU-and-mul fused into the "scalesweep_mse" quantizer: the same codes and
 * scales as ssw_scalesweep_mse_nvfp4_quant_out applied to the output of
 * ssw_silu_and_mul, without writing that bf16 intermediate.  input is
 * [num_rows, 2n] (gate, then up); output [num_rows, n/2]; no padding
 * (physical_n = n).  Input 32-byte and output 8-byte aligned.
 * This is the role of vLLM's silu_and_mul_nvfp4_quant, which its
 * fuse_act_quant pass substitutes for silu_and_mul + scaled_fp4_quant
 * (vllm 0.22 compilation/passes/fusion/act_quant_fusion.py:124-172); the
 * reference turns that pass off (run_bench_tune.sh:24,31) so that its own
 * quantizer runs unfused.
 */
int ssw_silu_and_mul_scalesweep_mse_nvfp4_quant_out(const void* input, int input_dtype,
                                                    int64_t num_rows, int64_t n,
                                                    const float* input_scale, uint8_t* output,
                                                    uint8_t* output_scale,
                                                    int is_sf_swizzled_layout, void* stream);

/*
 * RMSNorm fused into the "scalesweep_mse" quantizer: the codes and scales
 * ssw_scalesweep_mse_nvfp4_quant_out would write for vLLM's RMSNorm output,
 * without writing that bf16 intermediate.  bf16 only; input [num_rows, n],
 * weight [n], n % 16 == 0; no padding (physical_n = n).
 *   residual == NULL : the normalised values are vLLM's rms_norm(input, weight, eps).
 *   residual != NULL : vLLM's fused_add_rms_norm: residual <- bf16(input + residual)
 *                      (in place), and the normalised values are rms_norm(residual).
 * Bit for bit vLLM's result: its per-token block size (1024 threads below 256
 * tokens, 256 from there), its vector and CUB reduction order, rsqrtf of the
 * IEEE mean, and one rounding of x * r * w were matched on a B200.
 * rstd_workspace: num_rows floats of device scratch (1/rms per row, left
 * there).  input, residual and weight 32-byte aligned, output 8-byte.
 * This is the role of vLLM's fuse_norm_quant pass (vllm 0.22
 * config/compilation.py:121-123) for this quantizer; the reference turns that
 * pass off (run_bench_tune.sh:24,31).
 */
int ssw_rms_norm_scalesweep_mse_nvfp4_quant_out(const void* input, void* residual,
                                                const void* weight, float eps, int64_t num_rows,
                                                int64_t n, const float* input_scale,
                                                uint8_t* output, uint8_t* output_scale,
                                                int is_sf_swizzled_layout, float* rstd_workspace,
                                                void* stream);

/*
 * Plain round-to-nearest NVFP4 comparator: scale code = clamp(e4m3(amax/6),1,126),
 * codes = e2m1(v / scale), same layouts.  Stands in for vLLM's
 * scaled_fp4_quant.out that bench_kernel/custom.py:24-31 dispatches "cutlass"/"vllm" to.
 */
int ssw_rtn_nvfp4_quant_out(const void* input, int input_dtype, int64_t num_rows, int64_t n,
                            int64_t physical_n, const float* input_scale, uint8_t* output,
                            uint8_t* output_scale, int is_sf_swizzled_layout, void* stream);

/*
 * Per-tensor |x| maximum.  Writes max|x| (NaN if any element is NaN, like
 * torch's x.abs().max()) to amax_out[0].  `workspace` is caller-provided device
 * scratch of at least ssw_absmax_workspace_bytes() bytes, 4-byte aligned; it
 * is reset by the call itself (calls sharing a workspace must not overlap).
 * Replaces the x.abs().max() half of bench_kernel/test_kernel_latency.py:65-70.
 */
int64_t ssw_absmax_workspace_bytes(void);
int ssw_absmax(const void* input, int input_dtype, int64_t numel, float* amax_out,
               void* workspace, void* stream);

/*
 * input_scale = (fp8_max * 6) / amax, evaluated as torch evaluates
 * `(fp8_max * 6.0) / amax_tensor`: reciprocal(amax) rounded, then times
 * fp8_max*6 rounded.  amax and out are device floats.
 * Replaces the division of bench_kernel/test_kernel_latency.py:65-70.
 */
int ssw_global_scale_from_amax(const float* amax, float fp8_max, float* input_scale_out,
                               void* stream);

/*
 * Fused single-launch amax + input_scale: one pass over `input` (the last CTA
 * to finish turns the reduced amax into the scale), result in
 * input_scale_out[0] and, if amax_out is non-NULL, amax in amax_out[0].
 * Same workspace rules as ssw_absmax.
 * Replaces bench_kernel/test_kernel_latency.py:65-75 (global_scale_inv).
 */
int ssw_global_scale_inv(const void* input, int input_dtype, int64_t numel, float fp8_max,
                         float* input_scale_out, float* amax_out, void* workspace,
                         void* stream);

/*
 * Block-scaled NVFP4 GEMM on the tcgen05 tensor cores:
 *   out[m, n] (bf16) = alpha[0] * sum_k (a[m,k] * a_scale[m,k/16]) * (b[n,k] * b_scale[n,k/16])
 * a: [m, k/2] E2M1 codes, b: [n, k/2] E2M1 codes (both K-major, element 2j in
 * the low nibble), a_scale / b_scale: E4M3 scales in the CUTLASS 128x4
 * swizzled layout (as written by the quantizers above, is_sf_swizzled_layout=1),
 * out: [m, n] bf16 row-major.  Requires k % 256 == 0 and n % 64 == 0
 * (SSW_ERR_UNSUPPORTED otherwise) and 16-byte aligned pointers.
 * When the output has too few 128x128 tiles to fill the GPU and K is long
 * enough, the K loop is split across CTAs.  Splitting is opted into with a
 * `workspace` of ssw_nvfp4_gemm_workspace_bytes(m, n, k) bytes (0 when no
 * split is planned); with a NULL or smaller workspace the GEMM runs unsplit.
 * Up to 8 splits of a tile run as one thread-block cluster and add their
 * partials in distributed shared memory (the workspace is then unused);
 * more splits add them through the workspace.  Calls sharing a workspace
 * must not overlap.  `status` (optional, device int) becomes non-zero if a
 * bounded device wait gave up.
 * Replaces vLLM's cutlass_scaled_fp4_mm, which the W4A4 linear layer calls
 * after activation quantization (vllm 0.22 model_executor/kernels/linear/
 * nvfp4/cutlass.py:64-71; the reference's fallback restatement is
 * benchmark_nvfp4_tokens.py:84-106).
 */
int64_t ssw_nvfp4_gemm_workspace_bytes(int64_t m, int64_t n, int64_t k);
int ssw_nvfp4_gemm(const uint8_t* a, const uint8_t* b, const uint8_t* a_scale,
                   const uint8_t* b_scale, const float* alpha, void* out, int64_t m, int64_t n,
                   int64_t k, void* workspace, int64_t workspace_bytes, int* status,
                   void* stream);

/* ssw_nvfp4_gemm launched as a programmatic dependent of the kernel before it
 * on the stream (typically the quantizer that wrote a and a_scale).  Its
 * prologue and the loads of b and b_scale may overlap that kernel; a and
 * a_scale are read only after it has finished and its writes are visible.
 * Correct after any kernel (one that does not signal early is simply waited
 * for); the split-K path through global memory launches without the
 * dependency.  Same arguments, results and errors as ssw_nvfp4_gemm.
 * Replaces the same vLLM call as ssw_nvfp4_gemm (cutlass_scaled_fp4_mm right
 * after scaled_fp4_quant, vllm/model_executor/kernels/linear/nvfp4/
 * cutlass.py:56-71).
 */
int ssw_nvfp4_gemm_dependent(const uint8_t* a, const uint8_t* b, const uint8_t* a_scale,
                             const uint8_t* b_scale, const float* alpha, void* out, int64_t m,
                             int64_t n, int64_t k, void* workspace, int64_t workspace_bytes,
                             int* status, void* stream);

/* Measures the dense FP4 tensor-core rate this GEMM is bounded by.  No
 * reference counterpart: it gives the measured peak that GEMM roofline
 * fractions are taken against.  One CTA per SM issues 4 * iters back-to-back
 * kind::mxf4nvf4 MMAs of 128 x bn x 64 (bn 128 or 256): the GEMM's own
 * instruction, descriptors and TMEM layout, on operands already in shared
 * memory, with no loads.  cycles_out (device, one int64 per SM) receives each
 * CTA's elapsed SM clock cycles, -1 where the bounded completion wait gave up
 * (then *status is set).  FLOPs per CTA = 2 * 128 * bn * 64 * 4 * iters.
 * iters <= 16384.  Needs the whole GPU: one CTA holds an SM's TMEM.
 */
int ssw_nvfp4_mma_rate_probe(int bn, int iters, long long* cycles_out, int* status,
                             void* stream);

/*
 * A W4A4 linear layer's activation quantization and GEMM in one call:
 * x [m, k] (bf16/f16) is quantized with the "scalesweep_mse" sweep
 * (x_scale = its input_scale, as for ssw_scalesweep_mse_nvfp4_quant_out) into
 * codes and swizzled scales in `workspace`, then
 *   out[m, n] (bf16) = alpha[0] * (A (.) sfA) (B (.) sfB)^T
 * as ssw_nvfp4_gemm computes it, bit for bit.  The GEMM is launched as a
 * programmatic dependent of the quantizer: its prologue and its first
 * stages of weight loads overlap the quantizer; it reads A only after the
 * quantizer has finished.  workspace: 256-byte aligned, at least
 * ssw_nvfp4_quant_gemm_workspace_bytes(m, n, k) bytes (A's codes and scales,
 * then the GEMM's split-K scratch).  Same limits as ssw_nvfp4_gemm.
 * Replaces the scaled_fp4_quant + cutlass_scaled_fp4_mm pair of vLLM's W4A4
 * linear layer (vllm 0.22 model_executor/kernels/linear/nvfp4/cutlass.py:56-71),
 * with the quantizer the reference hooks in there.
 */
int64_t ssw_nvfp4_quant_gemm_workspace_bytes(int64_t m, int64_t n, int64_t k);
int ssw_nvfp4_quant_gemm(const void* x, int x_dtype, const float* x_scale, const uint8_t* b,
                         const uint8_t* b_scale, const float* alpha, void* out, int64_t m,
                         int64_t n, int64_t k, void* workspace, int64_t workspace_bytes,
                         int* status, void* stream);

/*
 * ssw_global_scale_inv without any device memory from the caller.  No
 * counterpart in the reference: the reference computes the global scale with
 * torch, which allocates.  This entry point is for callers that own only the
 * input and output buffers -- a plugin inside an engine that plans all device
 * memory up front and gives plugins no workspace, or a service that must keep
 * its device memory fixed after start-up.  It allocates nothing and needs no
 * workspace; its scratch is a
 * 32 KiB static __device__ array inside the library (held on every GPU that
 * loads the library until exit), one partial maximum per 32768-element chunk.
 * Limits and rules:
 *   - numel <= ssw_global_scale_inv_noalloc_max_numel() (2^28); larger sizes
 *     return SSW_ERR_INVALID_ARGUMENT with a message;
 *   - all calls share the scratch: calls that overlap on the GPU race, so
 *     order them on one stream;
 *   - the first call on a device looks up the scratch address for that
 *     device; make it before any stream capture;
 *   - the address is cached per device for the process: do not call this
 *     on a device again after cudaDeviceReset on it;
 *   - a CUDA failure returns SSW_ERR_CUDA and ssw_last_error() names the
 *     failing step and the CUDA error name.
 * Results equal ssw_global_scale_inv's bit for bit.
 */
int64_t ssw_global_scale_inv_noalloc_max_numel(void);
int ssw_global_scale_inv_noalloc(const void* input, int input_dtype, int64_t numel,
                                 float fp8_max, float* input_scale_out, float* amax_out,
                                 void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SCALESWEEP_B200_H_ */
