// Block-scaled NVFP4 GEMM on the 5th-generation tensor cores (sm_100a):
//
//   D[m, n] = alpha * sum_k (A[m,k] * sfA[m, k/16]) * (B[n,k] * sfB[n, k/16])      (bf16 out)
//
// A: E2M1 codes [M, K/2] bytes (K-major, element 2j in the low nibble),
// B: E2M1 codes [N, K/2] bytes, sfA / sfB: E4M3 scales in the CUTLASS 128x4
// swizzled layout that the quantizer writes, alpha: one device float.  This is
// the operation vLLM's cutlass_scaled_fp4_mm performs for a W4A4 linear layer
// (vllm 0.22 model_executor/kernels/linear/nvfp4/cutlass.py:64-71).
//
// One CTA computes one 128 x 128 output tile:
//   warp 0 (one lane)  : producer.  TMA tiled loads of the A and B code tiles
//                        (128 rows x 128 bytes, 128B swizzle; no multicast)
//                        and 1-D bulk copies of the four 512-byte scale atoms
//                        of each operand per 256-wide K block, into a
//                        3-stage shared-memory ring guarded by mbarriers.
//   Two CTAs share an SM (110 KiB shared memory and 256 TMEM columns each), so
//   one CTA's epilogue overlaps the other's main loop.
//   warp 1 (one lane)  : tensor-core issuer.  Copies each stage's scale atoms
//                        to TMEM (tcgen05.cp 32x128b.warpx4), then issues
//                        4 x tcgen05.mma kind::mxf4nvf4.block_scale.block16
//                        (M=128, N=128, K=64) accumulating fp32 in TMEM, and
//                        releases the stage with tcgen05.commit.
//   warps 0-3          : epilogue.  tcgen05.ld of the 128 x 128 fp32
//                        accumulator (one TMEM lane quadrant per warp),
//                        x alpha, round to bf16, store.
// Every mbarrier wait is bounded; a wait that gives up records an error code
// in *status and the CTA still frees its TMEM before returning.
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "gemm.cuh"

namespace ssw {
namespace gemm {
namespace {

constexpr int kThreads = 128;
constexpr int kBM = 128, kBN = 128;
constexpr int kBKBytes = 128;                // 256 fp4 values per row per K block
constexpr int kStages = 3;                   // 3 x 36 KiB: two CTAs fit one SM
constexpr int kATile = kBM * kBKBytes;       // 16 KiB
constexpr int kBTile = kBN * kBKBytes;       // 16 KiB
constexpr int kSFTile = 4 * 512;             // four 128x4 scale atoms (K block of 256)
constexpr int kStageBytes = kATile + kBTile + 2 * kSFTile;
constexpr int kTmemCols = 256;               // 128 accumulator + 16 SFA + 16 SFB, pow2
constexpr int kColSFA = 128, kColSFB = 144;
constexpr int kMaxSplits = 16;
// Split-K reduction: 128 rows x 32 fp32 columns of one split's partial
// (16 KiB, contiguous in the partial layout) per ring slot.
constexpr int kRedChunkBytes = kBM * 32 * 4;
constexpr int kRedSlots = kStages * kStageBytes / kRedChunkBytes;
constexpr uint32_t kWaitLimit = 1u << 24;    // bounded spin (each try_wait may suspend briefly)

struct __align__(8) Barriers {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t acc_full;
  uint64_t red_full[kRedSlots];  // split-K reduction: partial chunk landed in ring slot
  uint32_t tmem_base;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// Bounded wait for the mbarrier phase with the given parity; false = gave up.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory matrix descriptor (tcgen05): start>>4 [0,14), LBO>>4 [16,30),
// SBO>>4 [32,46), version 1 [46,48), layout type [61,64).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo,
                                              uint32_t layout) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46) | ((uint64_t)layout << 61);
}
constexpr uint32_t kLayoutSW128 = 2, kLayoutNone = 0;

// Instruction descriptor, kind::mxf4nvf4 with E4M3 scales: A/B format E2M1 (1)
// [7,10) [10,13), K-major A and B, N>>3 [17,23), scale format UE4M3 (0) [23],
// M>>4 [24,29), dense K=64.
constexpr uint32_t kIdesc = (1u << 7) | (1u << 10) | ((uint32_t)(kBN >> 3) << 17) |
                            ((uint32_t)(kBM >> 4) << 24);

__device__ __forceinline__ void mma_nvf4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], "
      "[%6], p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accum), "r"(sfa_tmem), "r"(sfb_tmem));
}

__device__ __forceinline__ void copy_sf_to_tmem(uint32_t tmem, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(tmem), "l"(sdesc));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// One warp reads its 32-lane quadrant: lane i gets 32 consecutive fp32 columns.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, "
      "%10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, "
      "%26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
        "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]),
        "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]),
        "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 fp32 values x alpha -> 32 bf16 (64 contiguous bytes).
__device__ __forceinline__ void store_row32_bf16(__nv_bfloat16* dst, const uint32_t (&v)[32],
                                                 float alpha) {
  uint32_t packed[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float lo = __uint_as_float(v[2 * i]) * alpha;
    const float hi = __uint_as_float(v[2 * i + 1]) * alpha;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(packed[i]) : "f"(hi), "f"(lo));
  }
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i)
    d[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
}

__device__ __forceinline__ void record_error(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

__global__ void __launch_bounds__(kThreads, 2)
    nvfp4_gemm_kernel(const __grid_constant__ CUtensorMap map_a,
                      const __grid_constant__ CUtensorMap map_b, const uint8_t* __restrict__ sfa,
                      const uint8_t* __restrict__ sfb, const float* __restrict__ alpha_ptr,
                      __nv_bfloat16* __restrict__ out, int m, int n, int k, int* status,
                      float* __restrict__ partials, uint32_t* __restrict__ tile_tickets) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte aligned stage ring (128B-swizzled tiles need 1024 B alignment)
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  Barriers* bars = reinterpret_cast<Barriers*>(smem + kStages * kStageBytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tile = blockIdx.x, m_tile = blockIdx.y;
  const int splits = gridDim.z, split = blockIdx.z;
  const int kblocks_all = k / 256;
  // this CTA's slice of the K blocks (split-K when gridDim.z > 1)
  const int kb_begin = (int)(((long long)split * kblocks_all) / splits);
  const int kb_end = (int)(((long long)(split + 1) * kblocks_all) / splits);
  const int kblocks = kb_end - kb_begin;
  const uint64_t sf_row_stride = (uint64_t)(k / 16) * 128;  // bytes per 128-row scale slab
  const uint8_t* sfa_tile = sfa + (uint64_t)m_tile * sf_row_stride;
  const uint8_t* sfb_tile = sfb + (uint64_t)n_tile * sf_row_stride;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    mbar_init(&bars->acc_full, 1);
    for (int r = 0; r < kRedSlots; ++r) mbar_init(&bars->red_full[r], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_a)));
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_b)));
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&bars->tmem_base)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem = bars->tmem_base;
  bool ok = true;

  if (warp == 0 && lane == 0) {
    // ---------------- producer
    for (int kb = 0; kb < kblocks && ok; ++kb) {
      const int s = kb % kStages;
      const uint32_t round = kb / kStages;
      if (round > 0 && !mbar_wait(&bars->empty[s], (round - 1) & 1)) {
        record_error(status, 1);
        ok = false;
        break;
      }
      uint8_t* st = smem + s * kStageBytes;
      mbar_expect_tx(&bars->full[s], kStageBytes);
      const int gkb = kb_begin + kb;  // global K block
      tma_load_2d(st, &map_a, &bars->full[s], gkb * kBKBytes, m_tile * kBM);
      tma_load_2d(st + kATile, &map_b, &bars->full[s], gkb * kBKBytes, n_tile * kBN);
      bulk_load(st + kATile + kBTile, sfa_tile + (uint64_t)gkb * kSFTile, kSFTile,
                &bars->full[s]);
      bulk_load(st + kATile + kBTile + kSFTile, sfb_tile + (uint64_t)gkb * kSFTile, kSFTile,
                &bars->full[s]);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- tensor-core issuer
    for (int kb = 0; kb < kblocks && ok; ++kb) {
      const int s = kb % kStages;
      if (!mbar_wait(&bars->full[s], (kb / kStages) & 1)) {
        record_error(status, 2);
        ok = false;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;");
      uint8_t* st = smem + s * kStageBytes;
      const uint32_t a_base = smem_u32(st), b_base = smem_u32(st + kATile);
      const uint32_t sfa_base = smem_u32(st + kATile + kBTile);
      const uint32_t sfb_base = sfa_base + kSFTile;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        // one 512-byte atom = 32 rows x 16 B; 8-row core matrices 128 B apart
        copy_sf_to_tmem(tmem + kColSFA + 4 * j, smem_desc(sfa_base + 512 * j, 16, 128, kLayoutNone));
        copy_sf_to_tmem(tmem + kColSFB + 4 * j, smem_desc(sfb_base + 512 * j, 16, 128, kLayoutNone));
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        // K step j: 64 fp4 values = 32 bytes into each 128-byte swizzled row
        const uint64_t adesc = smem_desc(a_base + 32 * j, 16, 1024, kLayoutSW128);
        const uint64_t bdesc = smem_desc(b_base + 32 * j, 16, 1024, kLayoutSW128);
        mma_nvf4(tmem, adesc, bdesc, tmem + kColSFA + 4 * j, tmem + kColSFB + 4 * j,
                 (kb | j) != 0);
      }
      mma_commit(&bars->empty[s]);
    }
    mma_commit(&bars->acc_full);
  }
  __syncwarp();

  // ---------------- epilogue: every warp reads its 32 accumulator lanes
  const bool acc_ok = mbar_wait(&bars->acc_full, 0);
  if (!acc_ok) record_error(status, 3);
  asm volatile("tcgen05.fence::after_thread_sync;");
  const float alpha = __ldg(alpha_ptr);
  const int row = m_tile * kBM + warp * 32 + lane;
  const int tile_id = m_tile * gridDim.x + n_tile;
  const uint64_t tile_elems = (uint64_t)kBM * kBN;
  // split-K: this CTA's fp32 partial tile, stored as [32 column groups][128 rows] float4
  float* my_part = splits > 1 ? partials + ((uint64_t)split * gridDim.x * gridDim.y + tile_id) *
                                               tile_elems
                              : nullptr;
#pragma unroll 1
  for (int c = 0; c < kBN; c += 32) {
    uint32_t v[32];
    const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c;
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
          "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]),
          "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]),
          "=r"(v[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    if (!acc_ok || row >= m) continue;
    if (splits > 1) {
      // partial layout [column group of 4][row]: lanes (rows) of a warp write
      // 32 consecutive float4s
      float4* dst = reinterpret_cast<float4*>(my_part) + (warp * 32 + lane);
#pragma unroll
      for (int q = 0; q < 8; ++q)
        dst[(c / 4 + q) * kBM] =
            make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                        __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3]));
      continue;
    }
    uint32_t packed[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float lo = __uint_as_float(v[2 * i]) * alpha;
      const float hi = __uint_as_float(v[2 * i + 1]) * alpha;
      asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(packed[i]) : "f"(hi), "f"(lo));
    }
    uint4* dst = reinterpret_cast<uint4*>(out + (uint64_t)row * n + (uint64_t)n_tile * kBN + c);
#pragma unroll
    for (int q = 0; q < 4; ++q)
      dst[q] = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
  }
  if (splits > 1) {
    // The last split to finish this tile adds every split's partial in split
    // order (deterministic) and writes bf16; nobody waits for another CTA.
    // Its stage ring is idle now: the other splits' partials come in by bulk
    // copy, kRedSlots chunks in flight, only the tile's valid rows; this
    // CTA's own partial is still in TMEM.
    __shared__ bool last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      last = atomicAdd(&tile_tickets[tile_id], 1u) == (uint32_t)(splits - 1);
      __threadfence();
      asm volatile("fence.proxy.async.global;" ::: "memory");
    }
    __syncthreads();
    const int valid_rows = min(kBM, m - m_tile * kBM);
    if (last && acc_ok && valid_rows * (kBN / 4) <= 2 * 4 * kThreads) {
      // Few valid rows (decode): at most two passes of plain loads, every
      // split's value in flight at once.
      __threadfence();
      // Coalesced pass over the tile's valid rows: float4 i covers column
      // group i/valid_rows, row i%valid_rows (partials are stored [group][row]);
      // every split's value is loaded first, then added in split order.
      const int n4 = valid_rows * (kBN / 4);
      const uint64_t split_stride4 = (uint64_t)gridDim.x * gridDim.y * (tile_elems / 4);
      const float4* part0 = reinterpret_cast<const float4*>(partials) + (uint64_t)tile_id *
                                                                            (tile_elems / 4);
      // four float4 positions per thread per pass: 4 x splits loads in flight
      constexpr int kUnroll = 4;
      for (int i0 = threadIdx.x; i0 < n4; i0 += kThreads * kUnroll) {
        float4 acc[kUnroll];
        uint64_t off[kUnroll];
        bool ok4[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int i = i0 + u * kThreads;
          ok4[u] = i < n4;
          const int ii = ok4[u] ? i : 0;
          off[u] = (uint64_t)(ii / valid_rows) * kBM + (ii % valid_rows);
          acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll 1
        for (int sp0 = 0; sp0 < splits; sp0 += 4) {
          float4 p[4][kUnroll];
#pragma unroll
          for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int u = 0; u < kUnroll; ++u)
              if (sp0 + q < splits && ok4[u])
                p[q][u] = __ldcg(part0 + (sp0 + q) * split_stride4 + off[u]);
#pragma unroll
          for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int u = 0; u < kUnroll; ++u)
              if (sp0 + q < splits && ok4[u]) {  // split order, fixed
                acc[u].x += p[q][u].x;
                acc[u].y += p[q][u].y;
                acc[u].z += p[q][u].z;
                acc[u].w += p[q][u].w;
              }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          if (!ok4[u]) continue;
          const int i = i0 + u * kThreads;
          const int r = i % valid_rows, c4 = i / valid_rows;
          uint32_t lo, hi;
          asm("cvt.rn.bf16x2.f32 %0, %1, %2;"
              : "=r"(lo) : "f"(acc[u].y * alpha), "f"(acc[u].x * alpha));
          asm("cvt.rn.bf16x2.f32 %0, %1, %2;"
              : "=r"(hi) : "f"(acc[u].w * alpha), "f"(acc[u].z * alpha));
          *reinterpret_cast<uint2*>(out + (uint64_t)(m_tile * kBM + r) * n +
                                    (uint64_t)n_tile * kBN + 4 * c4) = make_uint2(lo, hi);
        }
      }
      if (threadIdx.x == 0) tile_tickets[tile_id] = 0u;
    } else if (last && acc_ok) {
      const int others = splits - 1;
      const int loads = (kBN / 32) * others;
      const uint64_t split_stride = (uint64_t)gridDim.x * gridDim.y * tile_elems;
      const float* tile_part0 = partials + (uint64_t)tile_id * tile_elems;
      const uint32_t run_bytes = (uint32_t)valid_rows * 16u;
      // load j: column chunk j / others of the (j % others)-th other split, as
      // one copy of valid_rows x 16 B per column group of 4
      auto issue = [&](int j) {
        const int c = j / others, o = j % others, sp = o < split ? o : o + 1;
        const int slot = j % kRedSlots;
        const float* src = tile_part0 + sp * split_stride + (uint64_t)c * (kRedChunkBytes / 4);
        mbar_expect_tx(&bars->red_full[slot], 8u * run_bytes);
#pragma unroll 1
        for (int i = 0; i < 8; ++i)
          bulk_load(smem + slot * kRedChunkBytes + i * kBM * 16, src + i * kBM * 4, run_bytes,
                    &bars->red_full[slot]);
      };
      if (threadIdx.x == 0)
        for (int j = 0; j < loads && j < kRedSlots; ++j) issue(j);
      const int r = warp * 32 + lane;  // row within the tile
      bool red_ok = true;
      int j = 0;
#pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c) {
        float acc[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = 0.0f;
#pragma unroll 1
        for (int sp = 0; sp < splits; ++sp) {
          if (sp == split) {
            uint32_t v[32];
            tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(c * 32), v);
#pragma unroll
            for (int i = 0; i < 32; ++i) acc[i] += __uint_as_float(v[i]);
            continue;
          }
          const int slot = j % kRedSlots;
          if (red_ok && mbar_wait(&bars->red_full[slot], (uint32_t)(j / kRedSlots) & 1u)) {
            // slot layout [column group of 4][row]: lanes read consecutive float4s
            const float4* src = reinterpret_cast<const float4*>(smem + slot * kRedChunkBytes);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float4 p4 = src[i * kBM + r];
              acc[4 * i] += p4.x;
              acc[4 * i + 1] += p4.y;
              acc[4 * i + 2] += p4.z;
              acc[4 * i + 3] += p4.w;
            }
          } else if (red_ok) {
            red_ok = false;
            record_error(status, 5);
          }
          __syncthreads();  // slot fully read before it is refilled
          if (threadIdx.x == 0 && j + kRedSlots < loads) issue(j + kRedSlots);
          ++j;
        }
        const int grow = m_tile * kBM + r;
        if (grow < m && red_ok) {
          uint32_t v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(acc[i]);
          store_row32_bf16(out + (uint64_t)grow * n + (uint64_t)n_tile * kBN + c * 32, v, alpha);
        }
      }
      if (threadIdx.x == 0) tile_tickets[tile_id] = 0u;
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols));
  }
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

bool make_code_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t row_bytes,
                   uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {row_bytes, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {(cuuint32_t)kBKBytes, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

}  // namespace

size_t smem_bytes() { return kStages * kStageBytes + sizeof(Barriers) + 1024; }

int choose_splits(int64_t m, int64_t n, int64_t k, int device_sms) {
  // Split K only when the output tiles leave SMs idle and K is long enough
  // that every split keeps at least 8 K blocks: a split CTA's fixed cost
  // (prologue, pipeline fill, fp32 partial round trip) outweighs the gain on
  // short K (measured on B200: K=4096 decode shapes ran slower split).
  const int64_t tiles = (n / kBN) * ((m + kBM - 1) / kBM);
  const int64_t kblocks = k / 256;
  if (tiles >= device_sms || kblocks < 24) return 1;
  int64_t s = (device_sms + tiles - 1) / tiles;
  if (s > kblocks / 8) s = kblocks / 8;
  if (s > kMaxSplits) s = kMaxSplits;
  return s < 1 ? 1 : (int)s;
}

size_t workspace_bytes(int64_t m, int64_t n, int64_t k, int splits) {
  if (splits <= 1) return 0;
  const int64_t tiles = (n / kBN) * ((m + kBM - 1) / kBM);
  return (size_t)splits * tiles * kBM * kBN * sizeof(float) + (size_t)tiles * sizeof(uint32_t);
}

cudaError_t launch(const GemmArgs& g, int splits, cudaStream_t stream, const char** why) {
  CUtensorMap map_a, map_b;
  if (!make_code_map(&map_a, g.a, (uint64_t)g.m, (uint64_t)g.k / 2, kBM) ||
      !make_code_map(&map_b, g.b, (uint64_t)g.n, (uint64_t)g.k / 2, kBN)) {
    *why = "cuTensorMapEncodeTiled failed";
    return cudaErrorInvalidValue;
  }
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    *why = "cudaGetDevice";
    return e;
  }
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    e = cudaFuncSetAttribute(nvfp4_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem_bytes());
    if (e != cudaSuccess) {
      *why = "cudaFuncSetAttribute";
      return e;
    }
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const unsigned gx = (unsigned)(g.n / kBN), gy = (unsigned)((g.m + kBM - 1) / kBM);
  float* partials = nullptr;
  uint32_t* tickets = nullptr;
  if (splits > 1) {
    partials = static_cast<float*>(g.workspace);
    tickets = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(g.workspace) +
                                          (size_t)splits * gx * gy * kBM * kBN * sizeof(float));
    e = cudaMemsetAsync(tickets, 0, (size_t)gx * gy * sizeof(uint32_t), stream);
    if (e != cudaSuccess) {
      *why = "cudaMemsetAsync";
      return e;
    }
  }
  dim3 grid(gx, gy, (unsigned)splits);
  nvfp4_gemm_kernel<<<grid, kThreads, smem_bytes(), stream>>>(
      map_a, map_b, g.sfa, g.sfb, g.alpha, static_cast<__nv_bfloat16*>(g.out), (int)g.m, (int)g.n,
      (int)g.k, g.status, partials, tickets);
  return cudaGetLastError();
}

}  // namespace gemm
}  // namespace ssw
