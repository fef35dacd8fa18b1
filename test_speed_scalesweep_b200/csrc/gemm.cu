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
// Two kernels, chosen per problem by choose_tile_n:
// - nvfp4_gemm_pair_kernel (large M, more 256 x 256 tiles than SM pairs):
//   persistent clusters of two CTAs sharing each 256 x 256 tile through
//   tcgen05.mma.cta_group::2; described at its definition.
// - nvfp4_gemm_kernel: one CTA computes one 128 x BN output tile (BN = 256,
//   128 or 64) with six warps:
//   warp 4 (one lane)  : producer.  TMA tiled loads of the A and B code tiles
//                        (128B swizzle; no multicast) and 1-D bulk copies of
//                        the 512-byte scale atoms of each operand per
//                        256-deep K block, into a shared-memory ring guarded
//                        by mbarriers.
//   warps 0-3          : scale factors, then epilogue.  Per stage they copy
//                        the scale atoms from shared memory into that stage's
//                        TMEM columns with tcgen05.st (warp w owns TMEM lanes
//                        32w..32w+31), then arrive on the stage's hardware
//                        named barrier.  After the main loop: tcgen05.ld of
//                        the fp32 accumulator, x alpha, round to bf16, store.
//   warp 5             : TMEM allocation and the tensor-core issue stream:
//                        4 x tcgen05.mma kind::mxf4nvf4.block_scale.block16
//                        (M=128, N=BN, K=64) per K block, released with
//                        tcgen05.commit.  It waits on named barriers only and
//                        never touches shared memory inside its loop: on B200
//                        a shared-memory access by the issuing warp waits for
//                        its queued MMAs to drain.
// Every mbarrier wait is bounded; a wait that gives up records an error code
// in *status and the CTA still frees its TMEM before returning.
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "gemm.cuh"

namespace ssw {
namespace gemm {
namespace {

// Warps 0-3 move each stage's scale factors into TMEM and later run the
// epilogue (warp w owns TMEM lanes 32w..32w+31); warp 4 is the TMA producer;
// warp 5 allocates TMEM and issues the MMAs.
constexpr int kThreads = 192;
constexpr int kEpiThreads = 128;
constexpr int kWarpProducer = 4, kWarpMma = 5;
constexpr int kBM = 128;
constexpr int kBKBytes = 128;                // 256 fp4 values per row per K block
constexpr int kMaxStages = 8;
constexpr int kATile = kBM * kBKBytes;       // 16 KiB
constexpr int kSFTile = 4 * 512;             // four 128x4 scale atoms (K block of 256)
constexpr int kMaxSplits = 16;
// Split-K reduces across a thread-block cluster (distributed shared memory)
// up to this many splits (the portable cluster size), in global memory above.
constexpr int kMaxClusterSplits = 8;
// Split-K reduction: 128 rows x 32 fp32 columns of one split's partial
// (16 KiB, contiguous in the partial layout) per ring slot.
constexpr int kRedChunkBytes = kBM * 32 * 4;
constexpr int kMaxRedSlots = 8;

// Output tile 128 x BN with a STAGES-deep ring.
// - Throughput (BN=128, 3 stages): two CTAs share an SM, so one CTA's scale
//   copies and epilogue overlap the other's MMAs.
// - Decode (BN=64, 7 stages): one CTA per SM keeps 7 K blocks in flight.
//   With few CTAs the weight stream is bound by the DRAM round trip per
//   stage, not by bytes.
template <int BN, int STAGES>
struct Tile {
  static_assert(BN == 256 || BN == 128 || BN == 64, "tile width");
  static_assert(STAGES <= kMaxStages, "ring depth");
  static constexpr int kBTile = BN * kBKBytes;
  // 128-row scale slabs of B per tile (one for BN <= 128)
  static constexpr int kSFBSlabs = BN > 128 ? BN / 128 : 1;
  static constexpr int kStageBytes = kATile + kBTile + (1 + kSFBSlabs) * kSFTile;
  // accumulator (BN fp32 columns), then per stage 16 SFA + 16 x slabs SFB
  // columns, allocated as a power of two
  static constexpr int kColSF = BN;
  static constexpr int kSFStageCols = 16 + 16 * kSFBSlabs;
  static constexpr int kUsedCols = BN + STAGES * kSFStageCols;
  static constexpr int kTmemCols = kUsedCols <= 128 ? 128 : (kUsedCols <= 256 ? 256 : 512);
  // CTAs sharing an SM: what the shared memory allows (two 3-stage rings)
  static constexpr int kCtasPerSm = STAGES <= 3 ? 2 : 1;
  static constexpr int kRedSlots = STAGES * kStageBytes / kRedChunkBytes > kMaxRedSlots
                                        ? kMaxRedSlots
                                        : STAGES * kStageBytes / kRedChunkBytes;
  static_assert(kRedSlots <= kMaxRedSlots, "reduction slots");
  // Instruction descriptor, kind::mxf4nvf4 with E4M3 scales: A/B format E2M1
  // (1) [7,10) [10,13), K-major A and B, N>>3 [17,23), scale format UE4M3 (0)
  // [23], M>>4 [24,29), dense K=64.
  static constexpr uint32_t kIdesc = (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                     ((uint32_t)(kBM >> 4) << 24);
};
constexpr uint32_t kWaitLimit = 1u << 24;    // bounded spin (each try_wait may suspend briefly)

struct __align__(8) Barriers {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t acc_full;
  uint64_t red_full[kMaxRedSlots];  // split-K reduction: partial chunk landed in ring slot
  uint32_t tmem_base;
  uint32_t last_flag;  // split-K: this CTA reduces the tile
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
constexpr uint32_t kLayoutSW128 = 2;  // 128-byte swizzle (layout type field)

__device__ __forceinline__ void mma_nvf4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t sfa_tmem, uint32_t sfb_tmem,
                                         uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], "
      "[%6], p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum), "r"(sfa_tmem), "r"(sfb_tmem));
}

// One warp writes its 32-lane quadrant: lane i stores 16 consecutive columns.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void epilogue_sync() {  // warps 0-3 only
  asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
}

// Stage s's scales are in TMEM: the four scale warps arrive and the MMA warp
// waits on hardware named barrier 2 + s.  A named barrier, not an mbarrier:
// on B200 a shared-memory access by the warp that issues tcgen05.mma waits
// for its queued MMAs to drain (measured: one mbarrier wait per four K=64
// MMAs cost ~280 cycles), so the MMA warp touches no shared memory in its
// loop.  At most one arrival per stage is outstanding: the scale warps reach
// stage s again only after full[s] of the next round, which needs this
// round's MMAs to have retired.
constexpr int kStageBarrierBase = 2;
constexpr int kStageBarrierThreads = kEpiThreads + 32;
__device__ __forceinline__ void stage_arrive(int s) {
  asm volatile("bar.arrive %0, %1;" ::"r"(kStageBarrierBase + s), "n"(kStageBarrierThreads)
               : "memory");
}
__device__ __forceinline__ void stage_wait(int s) {
  asm volatile("bar.sync %0, %1;" ::"r"(kStageBarrierBase + s), "n"(kStageBarrierThreads)
               : "memory");
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

// Rows of the A box: all 128, or for a single partial M tile its rows
// rounded up to 8.  Host and device use the same rule.
__host__ __device__ __forceinline__ int a_box_rows(int64_t m) {
  return m < kBM ? (int)((m + 7) / 8 * 8) : kBM;
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The shared::cluster address of the same shared-memory offset in CTA `rank`.
__device__ __forceinline__ uint32_t cluster_addr(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

// Four floats from another CTA's shared memory (shared::cluster address).
__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ void record_error(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, Tile<BN, STAGES>::kCtasPerSm)
    nvfp4_gemm_kernel(const __grid_constant__ CUtensorMap map_a,
                      const __grid_constant__ CUtensorMap map_b, const uint8_t* __restrict__ sfa,
                      const uint8_t* __restrict__ sfb, const float* __restrict__ alpha_ptr,
                      __nv_bfloat16* __restrict__ out, int m, int n, int k, int* status,
                      float* __restrict__ partials, uint32_t* __restrict__ tile_tickets,
                      int cluster_red, int pdl_wait) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte aligned stage ring (128B-swizzled tiles need 1024 B alignment)
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  using T = Tile<BN, STAGES>;
  constexpr int kStages = STAGES;
  constexpr int kBN = BN, kBTile = T::kBTile, kStageBytes = T::kStageBytes;
  constexpr int kTmemCols = T::kTmemCols, kColSF = T::kColSF;
  constexpr int kRedSlots = T::kRedSlots;
  constexpr int kPartStride = BN + 4;  // cluster split-K: fp32 partial row stride (floats)
  static_assert(STAGES * T::kStageBytes >= kBM * kPartStride * 4, "partial fits the ring");
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
  // a 128-row scale slab covers 128 / BN output tiles; the MMA reads this
  // tile's rows from TMEM columns (row % 128) / 32, so a 64-wide tile in the
  // upper half of its slab starts 2 columns in
  constexpr int kSFBSlabs = T::kSFBSlabs, kSFStageCols = T::kSFStageCols;
  const uint8_t* sfb_tile = sfb + ((uint64_t)n_tile * kBN / 128) * sf_row_stride;
  const uint32_t sfb_col_shift =
      kBN < 128 ? (uint32_t)((n_tile % (128 / (kBN < 128 ? kBN : 128))) * (kBN / 32)) : 0u;
  // A single, partial M tile (decode batches) loads only its rows, rounded up
  // to the 8-row swizzle atom; the stale rows after them only reach output
  // rows that are never stored.  Saves tile ingress when it is the bound.
  const int a_rows = a_box_rows(m);

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
  if (warp == kWarpMma) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&bars->tmem_base)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem = bars->tmem_base;

  if (warp == kWarpProducer) {
    if (lane == 0) {
      // ---------------- producer
      auto load_b = [&](int kb) {  // weights: never written by the previous kernel
        const int s = kb % kStages, gkb = kb_begin + kb;
        uint8_t* st = smem + s * kStageBytes;
        tma_load_2d(st + kATile, &map_b, &bars->full[s], gkb * kBKBytes, n_tile * kBN);
#pragma unroll
        for (int slab = 0; slab < kSFBSlabs; ++slab)
          bulk_load(st + kATile + kBTile + (1 + slab) * kSFTile,
                    sfb_tile + slab * sf_row_stride + (uint64_t)gkb * kSFTile, kSFTile,
                    &bars->full[s]);
      };
      // With a dependent launch (after the quantizer that writes A): arm the
      // first stages and start their weight loads, then wait for the
      // previous grid before the first read of A or its scales.
      int early = 0;
      if (pdl_wait) {
        early = kblocks < kStages ? kblocks : kStages;
        for (int kb = 0; kb < early; ++kb) {
          mbar_expect_tx(&bars->full[kb], kStageBytes - (kBM - a_rows) * kBKBytes);
          load_b(kb);
        }
        asm volatile("griddepcontrol.wait;" ::: "memory");
      }
      for (int kb = 0; kb < kblocks; ++kb) {
        const int s = kb % kStages;
        const uint32_t round = kb / kStages;
        if (round > 0 && !mbar_wait(&bars->empty[s], (round - 1) & 1)) {
          record_error(status, 1);
          break;
        }
        uint8_t* st = smem + s * kStageBytes;
        if (kb >= early) {
          mbar_expect_tx(&bars->full[s], kStageBytes - (kBM - a_rows) * kBKBytes);
          load_b(kb);
        }
        const int gkb = kb_begin + kb;  // global K block
        tma_load_2d(st, &map_a, &bars->full[s], gkb * kBKBytes, m_tile * kBM);
        bulk_load(st + kATile + kBTile, sfa_tile + (uint64_t)gkb * kSFTile, kSFTile,
                  &bars->full[s]);
      }
    }
    __syncwarp();
  } else if (warp == kWarpMma) {
    // ---------------- tensor-core issuer: MMAs only, the scales are already in TMEM.
    // The whole warp meets the scale warps at each stage's named barrier;
    // lane 0 issues.  Nothing in this loop reads or writes shared memory.
    for (int kb = 0; kb < kblocks; ++kb) {
      const int s = kb % kStages;
      stage_wait(s);  // the scale warps saw full[s] and stored this stage's scales
      if (lane == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;");
        uint8_t* st = smem + s * kStageBytes;
        const uint32_t a_base = smem_u32(st), b_base = smem_u32(st + kATile);
        const uint32_t col_sfa = tmem + kColSF + s * kSFStageCols;
        const uint32_t col_sfb = col_sfa + 16 + sfb_col_shift;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          // K step j: 64 fp4 values = 32 bytes into each 128-byte swizzled row
          const uint64_t adesc = smem_desc(a_base + 32 * j, 16, 1024, kLayoutSW128);
          const uint64_t bdesc = smem_desc(b_base + 32 * j, 16, 1024, kLayoutSW128);
          // step j's B scales: 4 columns per 128-row slab
          mma_nvf4(tmem, adesc, bdesc, T::kIdesc, col_sfa + 4 * j, col_sfb + 4 * kSFBSlabs * j,
                   (kb | j) != 0);
        }
        mma_commit(&bars->empty[s]);
      }
      __syncwarp();
    }
    if (lane == 0) mma_commit(&bars->acc_full);
    __syncwarp();
  } else {
    // ---------------- scale factors: shared memory -> TMEM, one warp per lane quadrant.
    // Atom j of a stage holds the K=64 step j scales of 128 rows as 32 rows of
    // 16 B; its row r carries rows r, r+32, r+64, r+96.  Lane r of every
    // quadrant gets those four words in columns 4j..4j+3, the layout
    // tcgen05.cp.32x128b.warpx4 would produce.
    const uint32_t quad_base = tmem + ((uint32_t)(warp * 32) << 16);
    bool sf_ok = true;
    for (int kb = 0; kb < kblocks; ++kb) {
      const int s = kb % kStages;
      if (sf_ok && !mbar_wait(&bars->full[s], (kb / kStages) & 1)) {
        record_error(status, 6);
        sf_ok = false;
      }
      // SFA: columns 4j..4j+3.  SFB: per step j, 4 columns per 128-row slab.
      uint32_t ra[16], rb[16 * kSFBSlabs];
      const uint8_t* sf_st = smem + s * kStageBytes + kATile + kBTile;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint4 a4 = make_uint4(0u, 0u, 0u, 0u);
        if (sf_ok) a4 = *reinterpret_cast<const uint4*>(sf_st + 512 * j + 16 * lane);
        ra[4 * j] = a4.x, ra[4 * j + 1] = a4.y, ra[4 * j + 2] = a4.z, ra[4 * j + 3] = a4.w;
#pragma unroll
        for (int slab = 0; slab < kSFBSlabs; ++slab) {
          uint4 b4 = make_uint4(0u, 0u, 0u, 0u);
          if (sf_ok)
            b4 = *reinterpret_cast<const uint4*>(sf_st + (1 + slab) * kSFTile + 512 * j + 16 * lane);
          uint32_t* d = rb + 4 * (kSFBSlabs * j + slab);
          d[0] = b4.x, d[1] = b4.y, d[2] = b4.z, d[3] = b4.w;
        }
      }
      // the previous user of these columns (K block kb - kStages) has finished:
      // full[s] for this round completes only after the producer saw its MMAs
      // retire through empty[s]
      const uint32_t stage_cols = quad_base + kColSF + s * kSFStageCols;
      tmem_st16(stage_cols, ra);
#pragma unroll
      for (int h = 0; h < kSFBSlabs; ++h)
        tmem_st16(stage_cols + 16 + 16 * h, *reinterpret_cast<const uint32_t(*)[16]>(rb + 16 * h));
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;");
      stage_arrive(s);
    }

    // ---------------- epilogue: warp w reads accumulator lanes 32w..32w+31
    const bool acc_ok = mbar_wait(&bars->acc_full, 0);
    if (!acc_ok) record_error(status, 3);
    asm volatile("tcgen05.fence::after_thread_sync;");
    const float alpha = __ldg(alpha_ptr);
    const int row = m_tile * kBM + warp * 32 + lane;
    const int tile_id = m_tile * gridDim.x + n_tile;
    const uint64_t tile_elems = (uint64_t)kBM * kBN;
    // split-K: this CTA's fp32 partial tile, stored as [32 column groups][128 rows] float4
    float* my_part = splits > 1 ? partials + ((uint64_t)split * gridDim.x * gridDim.y +
                                              tile_id) * tile_elems
                                : nullptr;
#pragma unroll 1
    for (int c = 0; c < kBN; c += 32) {
      uint32_t v[32];
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c, v);
      if (!acc_ok || row >= m) continue;
      if (splits > 1 && cluster_red) {
        // this CTA's fp32 partial, row-major in its idle ring, rows padded by
        // 4 floats so the 32 rows of a warp's float4 writes spread over the banks
        float* prow = reinterpret_cast<float*>(smem) + (warp * 32 + lane) * kPartStride + c;
#pragma unroll
        for (int q = 0; q < 8; ++q)
          *reinterpret_cast<float4*>(prow + 4 * q) =
              make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                          __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3]));
        continue;
      }
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
      store_row32_bf16(out + (uint64_t)row * n + (uint64_t)n_tile * kBN + c, v, alpha);
    }
    if (splits > 1 && !cluster_red) {
      // The last split to finish this tile adds every split's partial in split
      // order (deterministic) and writes bf16; nobody waits for another CTA.
      __threadfence();
      epilogue_sync();
      if (threadIdx.x == 0) {
        bars->last_flag =
            atomicAdd(&tile_tickets[tile_id], 1u) == (uint32_t)(splits - 1) ? 1u : 0u;
        __threadfence();
        asm volatile("fence.proxy.async.global;" ::: "memory");
      }
      epilogue_sync();
      const bool last = bars->last_flag != 0;
      const int valid_rows = min(kBM, m - m_tile * kBM);
      if (last && acc_ok && valid_rows * (kBN / 4) <= 2 * 4 * kEpiThreads) {
        // Few valid rows (decode): at most two passes of plain loads, every
        // split's value in flight at once.
        __threadfence();
        const int n4 = valid_rows * (kBN / 4);
        const uint64_t split_stride4 = (uint64_t)gridDim.x * gridDim.y * (tile_elems / 4);
        const float4* part0 =
            reinterpret_cast<const float4*>(partials) + (uint64_t)tile_id * (tile_elems / 4);
        // four float4 positions per thread per pass: 4 x splits loads in flight
        constexpr int kUnroll = 4;
        for (int i0 = threadIdx.x; i0 < n4; i0 += kEpiThreads * kUnroll) {
          float4 acc[kUnroll];
          uint64_t off[kUnroll];
          bool ok4[kUnroll];
#pragma unroll
          for (int u = 0; u < kUnroll; ++u) {
            const int i = i0 + u * kEpiThreads;
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
            const int i = i0 + u * kEpiThreads;
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
        // More rows: the ring is idle now, so the other splits' partials come
        // in by bulk copy, kRedSlots chunks in flight, only the valid rows;
        // this CTA's own partial is still in TMEM.
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
            epilogue_sync();  // slot fully read before it is refilled
            if (threadIdx.x == 0 && j + kRedSlots < loads) issue(j + kRedSlots);
            ++j;
          }
          const int grow = m_tile * kBM + r;
          if (grow < m && red_ok) {
            uint32_t v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(acc[i]);
            store_row32_bf16(out + (uint64_t)grow * n + (uint64_t)n_tile * kBN + c * 32, v,
                             alpha);
          }
        }
        if (threadIdx.x == 0) tile_tickets[tile_id] = 0u;
      }
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  if (splits > 1 && cluster_red) {
    // Split-K across the cluster (one CTA per K slice of this tile): every
    // partial is staged; CTA r adds rows r, r + splits, ... of all partials
    // in split order (deterministic) through distributed shared memory and
    // writes bf16.  All threads of every CTA reach both cluster barriers.
    cluster_sync();
    const uint32_t rank = cluster_rank();
    const int valid_rows = min(kBM, m - m_tile * kBM);
    const int my_rows = valid_rows > (int)rank ? (valid_rows - (int)rank + splits - 1) / splits : 0;
    constexpr int kCol4 = kBN / 4;
    const uint32_t part_base = smem_u32(smem);
    uint32_t bases[kMaxClusterSplits];
#pragma unroll
    for (int j = 0; j < kMaxClusterSplits; ++j)
      bases[j] = j < splits ? cluster_addr(part_base, (uint32_t)j) : 0u;
    const float alpha = __ldg(alpha_ptr);
#pragma unroll 1
    for (int it = threadIdx.x; it < my_rows * kCol4; it += kThreads) {
      const int r = (int)rank + splits * (it / kCol4), c4 = it % kCol4;
      const uint32_t off = (uint32_t)((r * kPartStride + c4 * 4) * 4);
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int j = 0; j < kMaxClusterSplits; ++j) {
        if (j < splits) {  // split order, fixed
          const float4 p = ld_dsmem_f4(bases[j] + off);
          acc.x += p.x;
          acc.y += p.y;
          acc.z += p.z;
          acc.w += p.w;
        }
      }
      uint32_t lo, hi;
      asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(lo) : "f"(acc.y * alpha), "f"(acc.x * alpha));
      asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(hi) : "f"(acc.w * alpha), "f"(acc.z * alpha));
      *reinterpret_cast<uint2*>(out + (uint64_t)(m_tile * kBM + r) * n +
                                (uint64_t)n_tile * kBN + 4 * c4) = make_uint2(lo, hi);
    }
    cluster_sync();  // no CTA frees its partial while another still reads it
  }
  if (warp == kWarpMma) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols));
  }
}

// ---------------------------------------------------------------------------
// Pair configuration (large M): clusters of two CTAs on two SMs, persistent
// over 256 x 256 output tiles, with tcgen05.mma.cta_group::2 (M=256, N=256,
// K=64).  For each tile each CTA loads its own 128 rows of A and 128 of the
// tile's 256 rows of B; the leader (cluster rank 0) issues one MMA stream that
// reads both CTAs' shared memory at the same offsets and writes rows 0-127 of
// D into the leader's TMEM and rows 128-255 into the peer's.  Per 256-deep K
// block each SM moves 32 KiB of code tiles for a 128 x 256 share of the
// output, against 48 KiB in a one-CTA 128 x 256 tile; L2-to-shared-memory
// ingress is what bounds these shapes.
// Scales (measured on B200): each CTA's TMEM holds the A scales of its own 128
// rows (4 columns per K=64 step) and the B scales of all 256 tile rows (8
// columns per step), the columns the one-CTA 256-wide tile uses.
//
// Warps (both CTAs; 15 warps):
//   0-3   scale factors: shared memory -> this CTA's TMEM (warp w owns lanes
//         32w..32w+31)
//   4-11  epilogue, two warps per TMEM lane quadrant (w % 4), 128 columns
//         each: TMEM -> registers (bf16), release the accumulator, then per
//         32 x 32 block through a swizzled shared-memory buffer to global,
//         8 rows x 64 B per store instruction, while the next tile's main
//         loop runs.  Measured on B200: stores straight from registers (32
//         rows per instruction) stalled the next tile's start by ~1.6 us, and
//         TMA stores slowed the main loop's TMA loads by ~12%.
//   12    producer (one lane): this CTA's tiles and scale atoms by TMA
//   13    TMEM allocation; in the leader the MMA issue stream
//   14    leader only, gate: waits until the peer's stage is ready
// TMEM (512 columns): accumulator 0-255, scale factors 256-495 (5 stages).
// With one accumulator the MMAs of the next tile wait for the epilogue's
// TMEM reads, not for its global stores.
//
// Barriers (every wait bounded; stage ring and tile counters continue across
// tiles):
//   full[s]      each CTA: its own A/B tiles and scale atoms landed (its own
//                loads complete on it; a TMA load completing on the other
//                CTA's barrier stalled the issuing CTA's later copies on B200)
//   peer_rdy[s]  leader: the peer's four scale warps saw the peer's full[s]
//                and stored its scales in TMEM (remote arrivals)
//   empty[s]     each CTA: the MMAs of stage s retired (one commit per CTA)
//   acc_full     each CTA: its half of the accumulator is final (per tile)
//   acc_empty    leader: all eight epilogue warps of the pair read the
//                accumulator (4 local + 4 remote arrivals, per tile)
// The gate, the leader's scale warps and the MMA warp meet on the stage's
// hardware named barrier, so the MMA warp waits on mbarriers only at tile
// boundaries, where its queue drains anyway.  Waits on barriers that the
// other CTA signals spin on test_wait with acquire at cluster scope (a
// suspended try_wait woke ~0.4 us late after a remote arrival on B200); the
// remote arrivals are relaxed (see mbar_arrive_cluster_relaxed).
constexpr int kPairStages = 5;
constexpr int kTilePair = 512;  // choose_tile_n's code for the pair configuration
constexpr int kPairThreads = 480;
constexpr int kPairWarpEpi = 4, kPairEpiWarps = 8;
constexpr int kPairWarpProducer = 12, kPairWarpMma = 13, kPairWarpGate = 14;
// epilogue staging: one 32 x 32 bf16 block per epilogue warp, its 16-byte
// chunks XOR-swizzled by row so both the row writes and the coalesced reads
// are free of bank conflicts
constexpr int kPairStoreBlock = 32 * 32 * 2;
constexpr int kPairStoreBytes = kPairEpiWarps * kPairStoreBlock;
constexpr int kPairStageThreads = kEpiThreads + 64;  // scale warps + gate + MMA
struct PairTile {
  static constexpr int kStageBytes = kATile + kBM * kBKBytes + 3 * kSFTile;  // A, B half, 3 atoms
  static constexpr int kColSF = 256;
  static constexpr int kSFStageCols = 48;  // 16 SFA + 32 SFB (two 128-row slabs)
  static constexpr int kTmemCols = 512;
  static_assert(kColSF + kPairStages * kSFStageCols <= kTmemCols, "TMEM columns");
  // M=256 (M>>4 = 16), N=256 (N>>3 = 32); otherwise as Tile::kIdesc
  static constexpr uint32_t kIdesc = (1u << 7) | (1u << 10) | (32u << 17) | (16u << 24);
};

struct __align__(8) PairBarriers {
  uint64_t full[kMaxStages];
  uint64_t peer_rdy[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t acc_full;
  uint64_t acc_empty;
  uint32_t tmem_base;
};

__device__ __forceinline__ void mbar_arrive_local(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Relaxed remote arrival.  Its callers publish tcgen05 data movement (stores
// of scales, loads of the accumulator) that they have waited for
// (tcgen05.wait::st / ::ld) and ordered before the arrival with
// tcgen05.fence::before_thread_sync; they have no generic-proxy writes for a
// release to carry.  A release at cluster scope (like fence.acq_rel.cluster)
// held the arriving warp ~0.6 us per arrival on B200, which serialised the
// peer's stages.
__device__ __forceinline__ void mbar_arrive_cluster_relaxed(uint32_t bar) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar)
               : "memory");
}

// Bounded wait for barriers the other CTA signals: a non-suspending
// test_wait spin with acquire at cluster scope (no separate fence).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

__device__ __forceinline__ void mma_nvf4_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                              uint32_t idesc, uint32_t sfa_tmem,
                                              uint32_t sfb_tmem, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], "
      "[%6], p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum), "r"(sfa_tmem), "r"(sfb_tmem));
}

// Pair stage barrier: the leader's scale warps and gate warp arrive, the MMA
// warp waits (hardware named barrier 2 + s, 192 threads).
__device__ __forceinline__ void pair_stage_arrive(int s) {
  asm volatile("bar.arrive %0, %1;" ::"r"(kStageBarrierBase + s), "n"(kPairStageThreads)
               : "memory");
}
__device__ __forceinline__ void pair_stage_wait(int s) {
  asm volatile("bar.sync %0, %1;" ::"r"(kStageBarrierBase + s), "n"(kPairStageThreads)
               : "memory");
}

// Arrive on a barrier (shared::cluster address, either CTA) once this
// thread's pair MMAs retire.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

// 256-row x 256-column tile t of a grid with n_pairs tiles per row.
struct PairTileCoord {
  int m_pair, n_pair;
};
__device__ __forceinline__ PairTileCoord pair_tile_coord(int t, int n_pairs) {
  return {t / n_pairs, t % n_pairs};
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPairThreads, 1)
    nvfp4_gemm_pair_kernel(const __grid_constant__ CUtensorMap map_a,
                           const __grid_constant__ CUtensorMap map_b,
                           const uint8_t* __restrict__ sfa, const uint8_t* __restrict__ sfb,
                           const float* __restrict__ alpha_ptr, __nv_bfloat16* __restrict__ out,
                           int m, int n, int k, int* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // same 1024-aligned offsets in both CTAs: the pair MMA reads the peer's
  // tiles at the leader's descriptor addresses
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  using T = PairTile;
  constexpr int kStages = kPairStages, kStageBytes = T::kStageBytes;
  constexpr int kBHalfOff = kATile, kSFOff = kATile + kBM * kBKBytes;
  uint8_t* store_buf = smem + kStages * kStageBytes;  // 1024-aligned
  PairBarriers* bars =
      reinterpret_cast<PairBarriers*>(smem + kStages * kStageBytes + kPairStoreBytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  // tiles cluster_id, cluster_id + clusters, ... (both CTAs walk the same list)
  const int cluster_id = (int)(blockIdx.x >> 1), clusters = (int)(gridDim.x >> 1);
  const int n_pairs = n / 256, tiles = n_pairs * ((m + 2 * kBM - 1) / (2 * kBM));
  const int kblocks = k / 256;
  const uint64_t sf_row_stride = (uint64_t)(k / 16) * 128;
  const int m_slabs = (m + kBM - 1) / kBM;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->peer_rdy[s], 4);
      mbar_init(&bars->empty[s], 1);
    }
    mbar_init(&bars->acc_full, 1);
    mbar_init(&bars->acc_empty, 2 * kPairEpiWarps);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_a)));
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_b)));
  }
  if (warp == kPairWarpMma) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&bars->tmem_base)),
                 "n"(T::kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  cluster_sync();  // both CTAs' barriers are initialised before any remote arrival
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem = bars->tmem_base;

  if (warp == kPairWarpProducer) {
    if (lane == 0) {
      // ---------------- producer (both CTAs): this CTA's tiles and scales
      int it = 0;  // stage counter, continued across tiles
      bool ok = true;
      for (int t = cluster_id; t < tiles && ok; t += clusters) {
        const PairTileCoord tc = pair_tile_coord(t, n_pairs);
        // The upper CTA of a last pair tile may lie wholly past M: it still
        // supplies its B rows, its A box reads the TMA fill and its A scales
        // come from the last slab (rows that are never stored).
        const int m_half = tc.m_pair * 2 + (int)rank;
        const uint8_t* sfa_tile = sfa + (uint64_t)min(m_half, m_slabs - 1) * sf_row_stride;
        const uint8_t* sfb_tile = sfb + (uint64_t)(tc.n_pair * 2) * sf_row_stride;
        const int b_row = (tc.n_pair * 2 + (int)rank) * kBM;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % kStages;
          const uint32_t round = it / kStages;
          // the peer's empty[s] is signalled by the leader's commit
          if (round > 0 && !mbar_wait(&bars->empty[s], (round - 1) & 1)) {
            record_error(status, 1);
            ok = false;
            break;
          }
          uint8_t* st = smem + s * kStageBytes;
          uint64_t* full = &bars->full[s];
          mbar_expect_tx(full, kStageBytes);
          tma_load_2d(st, &map_a, full, kb * kBKBytes, m_half * kBM);
          tma_load_2d(st + kBHalfOff, &map_b, full, kb * kBKBytes, b_row);
          bulk_load(st + kSFOff, sfa_tile + (uint64_t)kb * kSFTile, kSFTile, full);
          bulk_load(st + kSFOff + kSFTile, sfb_tile + (uint64_t)kb * kSFTile, kSFTile, full);
          bulk_load(st + kSFOff + 2 * kSFTile, sfb_tile + sf_row_stride + (uint64_t)kb * kSFTile,
                    kSFTile, full);
        }
      }
    }
    __syncwarp();
  } else if (warp == kPairWarpMma) {
    if (rank == 0) {
      // ---------------- pair MMA issuer (leader only)
      const uint32_t empty_own = smem_u32(&bars->empty[0]);
      const uint32_t empty_peer = cluster_addr(empty_own, 1);
      const uint32_t acc_own = smem_u32(&bars->acc_full);
      const uint32_t acc_peer = cluster_addr(acc_own, 1);
      int it = 0, ti = 0;
      bool ok = true;
      for (int t = cluster_id; t < tiles; t += clusters, ++ti) {
        // both CTAs' epilogue warps have read the previous tile's accumulator
        if (ti > 0) {
          if (lane == 0 && ok && !mbar_wait_cluster(&bars->acc_empty, (uint32_t)(ti - 1) & 1u)) {
            record_error(status, 9);
            ok = false;
          }
          __syncwarp();
        }
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % kStages;
          pair_stage_wait(s);  // both CTAs' tiles landed and both CTAs' scales are in TMEM
          if (lane == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;");
            uint8_t* st = smem + s * kStageBytes;
            const uint32_t a_base = smem_u32(st), b_base = smem_u32(st + kBHalfOff);
            const uint32_t col_sfa = tmem + T::kColSF + s * T::kSFStageCols;
            const uint32_t col_sfb = col_sfa + 16;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint64_t adesc = smem_desc(a_base + 32 * j, 16, 1024, kLayoutSW128);
              const uint64_t bdesc = smem_desc(b_base + 32 * j, 16, 1024, kLayoutSW128);
              mma_nvf4_pair(tmem, adesc, bdesc, T::kIdesc, col_sfa + 4 * j, col_sfb + 8 * j,
                            (kb | j) != 0);
            }
            const uint32_t off = (uint32_t)(s * sizeof(uint64_t));
            mma_commit_pair(empty_own + off);
            mma_commit_pair(empty_peer + off);
          }
          __syncwarp();
        }
        if (lane == 0) {
          mma_commit_pair(acc_own);
          mma_commit_pair(acc_peer);
        }
        __syncwarp();
      }
    }
  } else if (warp == kPairWarpGate) {
    if (rank == 0) {
      // ---------------- gate (leader): the peer's stage is ready
      bool ok = true;
      int it = 0;
      for (int t = cluster_id; t < tiles; t += clusters) {
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % kStages;
          const uint32_t parity = (uint32_t)(it / kStages) & 1u;
          if (lane == 0 && ok && !mbar_wait_cluster(&bars->peer_rdy[s], parity)) {
            record_error(status, 8);
            ok = false;
          }
          __syncwarp();
          pair_stage_arrive(s);
        }
      }
    }
  } else if (warp < kPairWarpEpi) {
    // ---------------- scale factors (both CTAs): shared memory -> TMEM
    const uint32_t quad_base = tmem + ((uint32_t)(warp * 32) << 16);
    const uint32_t peer_rdy0 = cluster_addr(smem_u32(&bars->peer_rdy[0]), 0);
    bool sf_ok = true;
    int it = 0;
    for (int t = cluster_id; t < tiles; t += clusters) {
      for (int kb = 0; kb < kblocks; ++kb, ++it) {
        const int s = it % kStages;
        const uint32_t parity = (uint32_t)(it / kStages) & 1u;
        if (sf_ok && !mbar_wait(&bars->full[s], parity)) {
          record_error(status, 6);
          sf_ok = false;
        }
        // SFA: columns 4j..4j+3.  SFB: 8 columns per step j, slab h at 4h.
        uint32_t ra[16], rb[32];
        const uint8_t* sf_st = smem + s * kStageBytes + kSFOff;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint4 a4 = make_uint4(0u, 0u, 0u, 0u);
          if (sf_ok) a4 = *reinterpret_cast<const uint4*>(sf_st + 512 * j + 16 * lane);
          ra[4 * j] = a4.x, ra[4 * j + 1] = a4.y, ra[4 * j + 2] = a4.z, ra[4 * j + 3] = a4.w;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint4 b4 = make_uint4(0u, 0u, 0u, 0u);
            if (sf_ok)
              b4 = *reinterpret_cast<const uint4*>(sf_st + (1 + h) * kSFTile + 512 * j +
                                                   16 * lane);
            uint32_t* d = rb + 4 * (2 * j + h);
            d[0] = b4.x, d[1] = b4.y, d[2] = b4.z, d[3] = b4.w;
          }
        }
        // columns free: full[s] of this round follows empty[s] of the last
        const uint32_t stage_cols = quad_base + T::kColSF + s * T::kSFStageCols;
        tmem_st16(stage_cols, ra);
        tmem_st16(stage_cols + 16, *reinterpret_cast<const uint32_t(*)[16]>(rb));
        tmem_st16(stage_cols + 32, *reinterpret_cast<const uint32_t(*)[16]>(rb + 16));
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;");
        if (rank == 0) {
          pair_stage_arrive(s);
        } else {
          __syncwarp();
          // the peer's tiles landed (full[s]) and its scales are in TMEM
          if (lane == 0)
            mbar_arrive_cluster_relaxed(peer_rdy0 + (uint32_t)(s * sizeof(uint64_t)));
        }
      }
    }
  } else {
    // ---------------- epilogue (both CTAs): TMEM lanes 32q..32q+31, columns 128h..128h+127
    const int e = warp - kPairWarpEpi, q = warp & 3, h = e >> 2;
    const uint32_t quad = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(h * 128);
    const uint32_t acc_empty_leader = cluster_addr(smem_u32(&bars->acc_empty), 0);
    uint8_t* blk = store_buf + e * kPairStoreBlock;
    const float alpha = __ldg(alpha_ptr);
    bool ok = true;
    int ti = 0;
    for (int t = cluster_id; t < tiles; t += clusters, ++ti) {
      const PairTileCoord tc = pair_tile_coord(t, n_pairs);
      uint32_t got = 0;
      if (lane == 0 && ok) {
        // the leader's acc_full is signalled by its own commit, the peer's remotely
        got = (rank == 0 ? mbar_wait(&bars->acc_full, (uint32_t)ti & 1u)
                         : mbar_wait_cluster(&bars->acc_full, (uint32_t)ti & 1u))
                  ? 1u
                  : 0u;
        if (!got) record_error(status, 3);
      }
      const bool acc_ok = __shfl_sync(0xffffffffu, got, 0) != 0;
      ok = ok && acc_ok;
      asm volatile("tcgen05.fence::after_thread_sync;");
      // this warp's 32 rows x 128 columns as bf16 pairs: 64 registers per lane
      uint32_t packed[64];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld32(quad + (uint32_t)(c * 32), v);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float lo = __uint_as_float(v[2 * i]) * alpha;
          const float hi = __uint_as_float(v[2 * i + 1]) * alpha;
          asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(packed[16 * c + i]) : "f"(hi), "f"(lo));
        }
      }
      // accumulator read: release it to the leader's MMA warp, then store
      asm volatile("tcgen05.fence::before_thread_sync;");
      __syncwarp();
      if (lane == 0) {
        if (rank == 0)
          mbar_arrive_local(&bars->acc_empty);
        else
          mbar_arrive_cluster_relaxed(acc_empty_leader);
      }
      const int row0 = (tc.m_pair * 2 + (int)rank) * kBM + q * 32;
      if (!acc_ok || row0 >= m) continue;  // rows past M: nothing to store
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        __syncwarp();  // previous block read back
        // row `lane`: 16-byte chunk j at chunk j ^ ((row >> 1) & 3)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          *reinterpret_cast<uint4*>(blk + lane * 64 + ((j ^ ((lane >> 1) & 3)) * 16)) =
              make_uint4(packed[16 * c + 4 * j], packed[16 * c + 4 * j + 1],
                         packed[16 * c + 4 * j + 2], packed[16 * c + 4 * j + 3]);
        __syncwarp();
        // lanes 4r..4r+3 store the 64 bytes of row r (+8i): 8 rows per instruction
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int r = (lane >> 2) + 8 * i, j = lane & 3;
          const uint4 v4 =
              *reinterpret_cast<const uint4*>(blk + r * 64 + ((j ^ ((r >> 1) & 3)) * 16));
          if (row0 + r < m)
            *reinterpret_cast<uint4*>(out + (uint64_t)(row0 + r) * n + tc.n_pair * 256 +
                                      h * 128 + c * 32 + j * 8) = v4;
        }
      }
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  cluster_sync();  // no CTA leaves while its peer may still touch its memory
  if (warp == kPairWarpMma) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "n"(T::kTmemCols));
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

template <int BN, int STAGES>
size_t smem_bytes_for() {
  return STAGES * Tile<BN, STAGES>::kStageBytes + sizeof(Barriers) + 1024;
}

size_t smem_bytes() { return smem_bytes_for<128, 3>(); }

size_t smem_bytes_pair() {
  return kPairStages * PairTile::kStageBytes + kPairStoreBytes + sizeof(PairBarriers) + 1024;
}

int choose_splits(int64_t m, int64_t n, int64_t k, int device_sms) {
  // Split K only when the output tiles leave SMs idle, one wave of CTAs at
  // most.  Up to kMaxClusterSplits splits of a tile form one CTA cluster and
  // add their partials in distributed shared memory, so a split needs only 4
  // K blocks of work.  More splits (very long K) reduce through global
  // memory, whose round trip (~2 us to publish a partial) needs at least 8 K
  // blocks per split.  Measured on B200 (128-wide tiles, CUDA-graph replay):
  // - long K (>= 32 K blocks): M=128, K=14336 19.9 -> 12.1 us;
  // - a short K only for a partial M tile, in 4 or more splits (M=64,
  //   N=4096, K=4096: 7.7 -> 6.8 us; a full 128-row tile gains nothing);
  // - the 128-wide split tiles run two CTAs per SM, so over several M tiles,
  //   and for tiles of <= 32 rows at a short K, a wave holds 2 x SMs CTAs
  //   (M=256, N=4096, K=14336: 16.8 -> 15.3 us in 4 splits instead of 2;
  //   M=16, N=6144, K=4096: 7.5 -> 6.9 us in 4 instead of none);
  // - over several M tiles, powers of two: clusters of 3 pack badly next to
  //   the second CTA of an SM (M=384, N=4096, K=14336: 27.0 us in 3 splits,
  //   20.8 in 2).
  // N % 128 == 64 runs the unsplit 64-wide tile only
  if (n % 128) return 1;
  const int64_t tiles = (n / 128) * ((m + kBM - 1) / kBM);
  const int64_t kblocks = k / 256;
  const bool long_k = kblocks >= 32;
  const int64_t wave =
      (m > kBM || (!long_k && m <= 32)) ? 2 * (int64_t)device_sms : (int64_t)device_sms;
  if (tiles >= wave) return 1;
  if (!long_k && !(m <= 96 && kblocks >= 16)) return 1;
  int64_t s = wave / tiles;
  if (m > kBM) {
    int64_t p = 1;
    while (p * 2 <= s) p *= 2;
    s = p;
  }
  if (s > kblocks / 4) s = kblocks / 4;
  if (s > kMaxClusterSplits) {
    s = s < kblocks / 8 ? s : kblocks / 8;
    if (s > kMaxSplits) s = kMaxSplits;
    if (s < kMaxClusterSplits) s = kMaxClusterSplits;
  }
  if (s < (long_k ? 2 : 4)) return 1;
  return (int)s;
}

int choose_tile_n(int64_t m, int64_t n, int splits, int device_sms) {
  // 256-wide tiles: A is shared by 256 columns, and tile ingress bounds these
  // GEMMs.  More 256 x 256 tiles than co-resident CTA pairs: the persistent
  // pair kernel (its epilogue overlaps the next tile; measured on B200 it
  // loses to the one-CTA tile when every pair gets a single tile).  Else,
  // enough 128 x 256 tiles to occupy most SMs (from ~60% of them the wide
  // tile wins): one CTA per 128 x 256 tile.
  // N % 128 == 64: 64-wide tiles; the last one is the first half of a
  // 128-row scale slab (swizzled scale buffers hold whole slabs).
  if (n % 128) return 64;
  // The wide tile also serves a single M tile, down to decode sizes, when
  // its 128 x 256 tiles fill the SMs (N=28672, K=4096: M=128 14.1 -> 12.1
  // us, M=16 11.4 -> 9.7 us).
  const int64_t m_tiles = (m + kBM - 1) / kBM;
  if (splits <= 1 && n % 256 == 0) {
    if (m > kBM && (n / 256) * ((m + 2 * kBM - 1) / (2 * kBM)) > device_sms / 2) return kTilePair;
    if ((n / 256) * m_tiles * 5 >= (int64_t)device_sms * 3) return 256;
  }
  // 128-wide N tiles that do not fill the SMs stream the weights through
  // twice as many 64-wide tiles, as long as those still fit one wave of one
  // CTA per SM (each CTA's TMA stream is latency-bound, so more CTAs move
  // more bytes; M=256, N=4096: 9.2 -> 8.0 us).  Split-K keeps 128.
  if (splits > 1 || n % 64 != 0) return 128;
  if (m > kBM) return (n / 64) * m_tiles <= device_sms ? 64 : 128;
  return (n / 128) < device_sms ? 64 : 128;
}

size_t workspace_bytes(int64_t m, int64_t n, int64_t k, int splits) {
  if (splits <= 1) return 0;
  const int64_t tiles = (n / 128) * ((m + kBM - 1) / kBM);
  return (size_t)splits * tiles * kBM * 128 * sizeof(float) + (size_t)tiles * sizeof(uint32_t);
}

namespace {

template <int BN, int STAGES>
cudaError_t launch_bn(const GemmArgs& g, int splits, cudaStream_t stream, const char** why) {
  CUtensorMap map_a, map_b;
  if (!make_code_map(&map_a, g.a, (uint64_t)g.m, (uint64_t)g.k / 2, (uint32_t)a_box_rows(g.m)) ||
      !make_code_map(&map_b, g.b, (uint64_t)g.n, (uint64_t)g.k / 2, BN)) {
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
    e = cudaFuncSetAttribute(nvfp4_gemm_kernel<BN, STAGES>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem_bytes_for<BN, STAGES>());
    if (e != cudaSuccess) {
      *why = "cudaFuncSetAttribute";
      return e;
    }
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const unsigned gx = (unsigned)(g.n / BN), gy = (unsigned)((g.m + kBM - 1) / kBM);
  dim3 grid(gx, gy, (unsigned)splits);
  // the K slices of a tile form one cluster and reduce in distributed shared memory
  const bool cluster = splits > 1 && splits <= kMaxClusterSplits;
  float* partials = nullptr;
  uint32_t* tickets = nullptr;
  if (splits > 1 && !cluster) {
    partials = static_cast<float*>(g.workspace);
    tickets = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(g.workspace) +
                                          (size_t)splits * gx * gy * kBM * BN * sizeof(float));
    e = cudaMemsetAsync(tickets, 0, (size_t)gx * gy * sizeof(uint32_t), stream);
    if (e != cudaSuccess) {
      *why = "cudaMemsetAsync";
      return e;
    }
  }
  // a dependent launch directly after the kernel that writes A (the memset
  // of the global-memory split path would stand between them)
  const bool pdl = g.dependent_launch && (splits <= 1 || cluster);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes_for<BN, STAGES>();
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned na = 0;
  if (cluster) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = (unsigned)splits;
    ++na;
  }
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  e = cudaLaunchKernelEx(&cfg, nvfp4_gemm_kernel<BN, STAGES>, map_a, map_b, g.sfa, g.sfb, g.alpha,
                         static_cast<__nv_bfloat16*>(g.out), (int)g.m, (int)g.n, (int)g.k,
                         g.status, partials, tickets, cluster ? 1 : 0, pdl ? 1 : 0);
  if (e != cudaSuccess) *why = "cudaLaunchKernelEx";
  return e;
}

cudaError_t launch_pair(const GemmArgs& g, cudaStream_t stream, const char** why) {
  CUtensorMap map_a, map_b;
  if (!make_code_map(&map_a, g.a, (uint64_t)g.m, (uint64_t)g.k / 2, kBM) ||
      !make_code_map(&map_b, g.b, (uint64_t)g.n, (uint64_t)g.k / 2, kBM)) {
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
    e = cudaFuncSetAttribute(nvfp4_gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem_bytes_pair());
    if (e != cudaSuccess) {
      *why = "cudaFuncSetAttribute";
      return e;
    }
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  // persistent: one cluster per co-resident pair of SMs, at most one per tile
  static int max_clusters[64] = {0};
  int clusters = dev >= 0 && dev < 64 ? max_clusters[dev] : 0;
  if (clusters <= 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(kPairThreads, 1, 1);
    cfg.dynamicSmemBytes = smem_bytes_pair();
    if (cudaOccupancyMaxActiveClusters(&clusters, nvfp4_gemm_pair_kernel, &cfg) != cudaSuccess ||
        clusters <= 0) {
      cudaGetLastError();  // clear a failed query
      int sms = 148;
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      clusters = sms / 2;
    }
    if (dev >= 0 && dev < 64) max_clusters[dev] = clusters;
  }
  const int64_t tiles = (g.n / 256) * ((g.m + 2 * kBM - 1) / (2 * kBM));
  if (tiles < clusters) clusters = (int)tiles;
  dim3 grid((unsigned)clusters * 2, 1, 1);
  nvfp4_gemm_pair_kernel<<<grid, kPairThreads, smem_bytes_pair(), stream>>>(
      map_a, map_b, g.sfa, g.sfb, g.alpha, static_cast<__nv_bfloat16*>(g.out), (int)g.m,
      (int)g.n, (int)g.k, g.status);
  return cudaGetLastError();
}

// Dense FP4 tensor-core rate: one CTA per SM issues back-to-back
// kind::mxf4nvf4 MMAs (128 x BN x 64, the GEMM kernel's own instruction,
// descriptors and TMEM layout) on tiles already in shared memory, with no
// loads, scale copies or epilogue.  The operands are whatever the shared
// memory and TMEM hold: every E2M1 code is a finite value, and the results are
// never read.  The MMA count per CTA stays small enough that the bounded
// completion wait cannot give up before the MMAs finish.
constexpr int kPeakThreads = 128;
constexpr size_t kPeakSmem = 200 * 1024;  // forces one CTA per SM (TMEM is not shared)

template <int BN>
__global__ void __launch_bounds__(kPeakThreads, 1)
    nvfp4_mma_peak_kernel(int iters, long long* cycles, int* status) {
  using T = Tile<BN, 1>;
  extern __shared__ __align__(1024) uint8_t peak_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(peak_raw) + 1023) &
                                             ~uintptr_t(1023));
  __shared__ uint64_t done_bar;
  __shared__ uint32_t tmem_slot;
  const int warp = threadIdx.x >> 5;
  constexpr uint32_t kCols = 512;
  if (threadIdx.x == 0) {
    mbar_init(&done_bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&tmem_slot)),
                 "r"(kCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem = tmem_slot;
  if (threadIdx.x == 0) {
    const uint32_t a_base = smem_u32(smem), b_base = smem_u32(smem + kATile);
    const uint32_t col_sfa = tmem + BN, col_sfb = col_sfa + 16;
    const long long t0 = clock64();
    for (int it = 0; it < iters; ++it) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint64_t adesc = smem_desc(a_base + 32 * j, 16, 1024, kLayoutSW128);
        const uint64_t bdesc = smem_desc(b_base + 32 * j, 16, 1024, kLayoutSW128);
        mma_nvf4(tmem, adesc, bdesc, T::kIdesc, col_sfa + 4 * j,
                 col_sfb + 4 * T::kSFBSlabs * j, (it | j) != 0);
      }
    }
    mma_commit(&done_bar);
    const bool ok = mbar_wait(&done_bar, 0);
    const long long t1 = clock64();
    if (!ok) record_error(status, 1);
    cycles[blockIdx.x] = ok ? t1 - t0 : -1;
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols));
}

}  // namespace

cudaError_t launch(const GemmArgs& g, int splits, cudaStream_t stream, const char** why) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int tile_n = choose_tile_n(g.m, g.n, splits, sms);
  if (tile_n == kTilePair) return launch_pair(g, stream, why);
  if (tile_n == 256) return launch_bn<256, 4>(g, 1, stream, why);
  if (tile_n == 64) return launch_bn<64, 7>(g, 1, stream, why);
  return launch_bn<128, 3>(g, splits, stream, why);
}


cudaError_t launch_mma_peak(int bn, int iters, int ctas, long long* cycles, int* status,
                            cudaStream_t stream) {
  if (bn == 256) {
    cudaError_t e = cudaFuncSetAttribute(nvfp4_mma_peak_kernel<256>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)kPeakSmem);
    if (e != cudaSuccess) return e;
    nvfp4_mma_peak_kernel<256><<<ctas, kPeakThreads, kPeakSmem, stream>>>(iters, cycles, status);
  } else {
    cudaError_t e = cudaFuncSetAttribute(nvfp4_mma_peak_kernel<128>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)kPeakSmem);
    if (e != cudaSuccess) return e;
    nvfp4_mma_peak_kernel<128><<<ctas, kPeakThreads, kPeakSmem, stream>>>(iters, cycles, status);
  }
  return cudaGetLastError();
}

}  // namespace gemm
}  // namespace ssw
