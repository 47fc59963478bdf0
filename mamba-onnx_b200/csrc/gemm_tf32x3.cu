// fp32-accurate GEMM on the sm_100a tensor cores (3xTF32), for the dense
// projections of a Mamba model around the scan op (in_proj, out_proj and
// the tied LM head of a Mamba block stack; the reference project leaves
// these GEMMs to its caller, benchmarks/profiler.py:18-150).
//
// C[m][n] (+)= sum_k A[m][k] * B[n][k], both operands K-contiguous, computed
// as A_hi B_hi + A_hi B_lo + A_lo B_hi on tcgen05 TF32 MMAs with an FP32
// accumulator in tensor memory, where X_hi = tf32(X) and X_lo = tf32(X -
// X_hi) (round to nearest, mamba_split_tf32). Each product then carries a
// relative error of at most ~3 * 2^-22 (the dropped X_lo Y_lo term and the
// rounding of the lo parts), the same order as the fp32 rounding of the
// accumulation itself.
//
// One CTA = one 128 x BN output tile (BN = 64, 128 or 192), 6, 10 or 14 warps:
// * the producer warp's lane 0 streams 32-wide K blocks of A_hi, A_lo,
//   B_hi, B_lo by TMA (128-byte swizzle, 4, 3 or 2 stages);
// * the MMA warp's lane 0 waits for a stage, issues 4 K-steps x 3
//   products of tcgen05.mma.kind::tf32 (M = 128, N = BN, K = 8) into a
//   TMEM accumulator that starts from zero for every K block (corrections
//   first, then hi*hi), and commits the stage back to the producer and the
//   accumulator to the accumulator warps (two accumulators alternate);
// * 4, 8 or 12 accumulator warps (warp w owns TMEM lanes 32(w%4)..+31 = tile
//   rows, and 64 columns) read each K block's sums (tcgen05.ld), add them to
//   fp32 registers, then store C with arbitrary strides, optionally adding
//   a second matrix C_in (which may be C itself): coalesced, through a
//   shared-memory transpose when C is row-major (store_sums).
// A second kernel computes 256 x BN tiles on CTA pairs (cta_group::2 MMAs,
// gemm_tf32x3_pair_kernel); the host picks pairs or single CTAs per shape.
// Every mbarrier wait is bounded (mamba_gemm error word on timeout).
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/mamba_model_ops.h"
#include "../../include/mamba_scan.h"
#include "scan_device.cuh"
#include "scan_kernels.h"

namespace mamba_gemm {

using mamba_scan::smem_u32;

constexpr int BM = 128, BK = 32;  // BK fp32 = 128 bytes: one swizzled row

// Single-CTA tile configurations: 128 x 64 with a 4-stage ring (48 KB per
// stage), 128 x 128 with 3 stages (64 KB), 128 x 192 with 2 stages (80 KB).
// The host picks the width with the fewest waves x (128 + BN), the operand
// rows a CTA streams per K block being 2 * 128 + 2 * BN, then CTA pairs
// (further down) when they cost no more; products with few output tiles
// split K (plan_gemm). Per SM and K block the time goes to moving operands
// through shared memory (TMA writes in, every MMA reading its A and whole B
// slices out) as much as to the MMAs themselves.
//
// Warps 0..kAccWarps-1 accumulate and store: warp w owns TMEM lanes
// 32(w%4)..+31 (tile rows) and columns [64(w/4), 64(w/4) + 64), so two or
// three warps share each SM sub-partition and hide each other's TMEM load
// latency; then one TMA producer warp and one MMA warp.
//
// Two fp32 accumulators of BN columns (alternate K blocks). The tensor
// core's accumulation into TMEM loses accuracy with every update (on K =
// 1536 one accumulator over the whole K ended 5x further from float64 than
// an fp32 GEMM), so each K block starts from zero and the accumulator warps
// fold it into fp32 registers with round-to-nearest adds. Within a block the
// 8 correction products (~2^-11 of the sums) go first, while the
// accumulator is small, then the 4 hi*hi products: the corrections' own
// rounding stays at their scale.
template <int BN_, int kStages_>
struct Cfg {
  static constexpr int BN = BN_, kStages = kStages_;
  static constexpr int kAccCols = 64;  // running sums per accumulator thread
  static constexpr int kAccWarps = 4 * BN / kAccCols;
  static constexpr int kAccThreads = 32 * kAccWarps;
  static constexpr int kProducerWarp = kAccWarps, kMmaWarp = kAccWarps + 1;
  static constexpr int kThreads = 32 * (kAccWarps + 2);
  static constexpr uint32_t kATile = BM * BK * 4, kBTile = BN * BK * 4;
  static constexpr uint32_t kStageBytes = 2 * kATile + 2 * kBTile;
  static constexpr int kTmemCols = (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
  struct __align__(1024) Smem {
    float a_hi[kStages][BM * BK];
    float a_lo[kStages][BM * BK];
    float b_hi[kStages][BN * BK];
    float b_lo[kStages][BN * BK];
    uint64_t full[kStages];
    uint64_t empty[kStages];
    uint64_t acc_full[2];   // a K block's sums are in TMEM accumulator b (tcgen05.commit)
    uint64_t acc_empty[2];  // the accumulator warps have read accumulator b
    uint32_t tmem_base;
  };
  static constexpr size_t kSmemBytes = sizeof(Smem) + 1024;  // + room to align the base
  static_assert(kSmemBytes <= 227 * 1024, "shared memory per CTA");
  static constexpr size_t kStageBuffers = (size_t)kStages * kStageBytes;  // a_hi .. b_lo
};
using Cfg64 = Cfg<64, 4>;
using Cfg128 = Cfg<128, 3>;
using Cfg192 = Cfg<192, 2>;

struct GemmMaps {
  CUtensorMap a_hi, a_lo, b_hi, b_lo;
};

struct GemmParams {
  float* c;
  const float* c_in;  // NULL: C = A B^T; else C = C_in + A B^T (C's strides)
  int64_t ldc_m, ldc_n;
  int M, N, K;
  // split K: grid.z = the number of splits; split z takes K blocks
  // [z * kb_per_split, (z + 1) * kb_per_split) and writes its partial sums
  // at c + z * slice (slice 0 and kb_per_split = all blocks when unsplit)
  int kb_per_split;
  int64_t slice;
};

__device__ int g_gemm_device_error = 0;

// ------------------------------------------------------------ PTX wrappers

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor of a K-major tile of rows of 32 fp32 (128
// bytes) written by TMA with the 128-byte swizzle: start address >> 4 in
// bits [0,14), leading byte offset 16 B (unused for swizzled K-major) in
// [16,30), stride byte offset 1024 B (between 8-row groups) in [32,46),
// descriptor version 1 in [46,48), base offset 0, layout type 2 =
// SWIZZLE_128B in [61,64) (the sm_100 UMMA SmemDescriptor; CUTLASS
// cute/arch/mma_sm100_desc.hpp).
__device__ __forceinline__ uint64_t sw128_desc(const void* tile) {
  const uint32_t a = smem_u32(tile);
  return (uint64_t)((a >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor of kind::tf32, D = F32, A = B = TF32, both K-major,
// N >> 3 in bits [17,23), M >> 4 in bits [24,29) (UMMA InstrDescriptor).
template <int BN>
__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                         uint32_t accumulate) {
  constexpr uint32_t kInstrDesc = (1u << 4) | (2u << 7) | (2u << 10) |
                                  ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
  asm volatile(
      "{\n\t"
      ".reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t"
      "}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(kInstrDesc), "r"(accumulate)
      : "memory");
}

// The mbarrier receives one arrival once every tcgen05 operation this
// thread issued before has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane (32x32b.x32);
// complete only after tmem_wait().
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------- epilogue

// Floats of shared memory one accumulator warp uses to transpose its block
// of sums (32 rows of kCols, one padding column: conflict-free both ways).
template <int kCols>
constexpr int kStoreScratch = 32 * (kCols + 1);

// Writes one accumulator warp's block of sums to C (at `c`, p's strides and
// sizes; a split's partial slice or C itself): lane l holds the kCols
// sums of row m_base + l, columns n_base... (acc[j/2].x / .y = column j),
// C[m][n] = (C_in[m][n] +) sum. C_in may be C itself: every element is read
// and written by the same thread, and each batch of reads is issued before
// the batch's writes (C and C_in may alias, so the compiler cannot do it).
// Column-major C (ldc_m == 1): the lanes' rows are consecutive addresses, so
// each column is one coalesced store. Otherwise the block goes through
// `scratch` (this warp's kStoreScratch<kCols> floats) and comes back one row
// at a time, the lanes on consecutive columns.
template <int kCols>
__device__ __forceinline__ void store_sums(const GemmParams& p, float* c,
                                           const float2 (&acc)[kCols / 2], int64_t m_base,
                                           int64_t n_base, float* scratch, int lane) {
  // elements per batch of reads: 8 keeps the 576-thread 256-wide pair tile
  // (96 registers a thread) from spilling (16: LM head 386 -> 349 us at 8)
  constexpr int kBatch = 8;
  if (p.ldc_m == 1) {
    const int64_t m = m_base + lane;
    const bool m_ok = m < p.M;
#pragma unroll
    for (int j0 = 0; j0 < kCols; j0 += kBatch) {
      float in[kBatch];
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        const int64_t n = n_base + j0 + j;
        in[j] = (p.c_in && m_ok && n < p.N) ? p.c_in[m + n * p.ldc_n] : 0.f;
      }
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        const int64_t n = n_base + j0 + j;
        const float a = ((j0 + j) & 1) ? acc[(j0 + j) / 2].y : acc[(j0 + j) / 2].x;
        if (m_ok && n < p.N) c[m + n * p.ldc_n] = p.c_in ? in[j] + a : a;
      }
    }
    return;
  }
  constexpr int kStride = kCols + 1, kPerRow = kCols / 32, kRows = kBatch / kPerRow;
#pragma unroll
  for (int j = 0; j < kCols; ++j)
    scratch[lane * kStride + j] = (j & 1) ? acc[j / 2].y : acc[j / 2].x;
  __syncwarp();
#pragma unroll 1
  for (int r0 = 0; r0 < 32; r0 += kRows) {
    float v[kRows][kPerRow], in[kRows][kPerRow];
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      const int64_t m = m_base + r0 + r;
#pragma unroll
      for (int h = 0; h < kPerRow; ++h) {
        const int64_t n = n_base + h * 32 + lane;
        v[r][h] = scratch[(r0 + r) * kStride + h * 32 + lane];
        in[r][h] = (p.c_in && m < p.M && n < p.N) ? p.c_in[m * p.ldc_m + n * p.ldc_n] : 0.f;
      }
    }
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      const int64_t m = m_base + r0 + r;
#pragma unroll
      for (int h = 0; h < kPerRow; ++h) {
        const int64_t n = n_base + h * 32 + lane;
        if (m < p.M && n < p.N) c[m * p.ldc_m + n * p.ldc_n] = p.c_in ? in[r][h] + v[r][h] : v[r][h];
      }
    }
  }
}

// ------------------------------------------------------------------ kernel

template <class C>
__global__ void __launch_bounds__(C::kThreads, 1)
    gemm_tf32x3_kernel(const __grid_constant__ GemmMaps maps, const GemmParams p) {
  constexpr int BN = C::BN, kStages = C::kStages, kAccCols = C::kAccCols;
  static_assert((size_t)C::kAccWarps * kStoreScratch<C::kAccCols> * 4 <= C::kStageBuffers,
                "the store transposes fit in the stage buffers");
  constexpr int kProducerWarp = C::kProducerWarp, kMmaWarp = C::kMmaWarp;
  extern __shared__ uint8_t smem_raw[];
  typename C::Smem& sm = *reinterpret_cast<typename C::Smem*>(
      smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // M tiles vary fastest: the CTAs running together share B tiles (the
  // larger operand of a wide GEMM such as an LM head), read from HBM once
  const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
  // this CTA's K blocks: [kb_begin, kb_begin + nk)
  const int kb_begin = (int)blockIdx.z * p.kb_per_split;
  const int nk = min((p.K + BK - 1) / BK - kb_begin, p.kb_per_split);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mamba_scan::mbar_init(&sm.full[s], 1);
      mamba_scan::mbar_init(&sm.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mamba_scan::mbar_init(&sm.acc_full[b], 1);
      mamba_scan::mbar_init(&sm.acc_empty[b], C::kAccThreads);
    }
    mamba_scan::fence_mbarrier_init();
  }
  if (warp == kProducerWarp && lane == 0) {
    mamba_scan::prefetch_tensormap(&maps.a_hi);
    mamba_scan::prefetch_tensormap(&maps.a_lo);
    mamba_scan::prefetch_tensormap(&maps.b_hi);
    mamba_scan::prefetch_tensormap(&maps.b_lo);
  }
  if (warp == 0) {  // the whole warp allocates the accumulators' TMEM columns
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&sm.tmem_base)),
                 "r"(C::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  // launched as a programmatic dependent launch: the set-up above overlaps
  // the previous kernel; the operands and C are touched only after it ends
  mamba_scan::pdl_trigger();
  mamba_scan::pdl_wait();

  if (warp == kProducerWarp) {
    if (lane == 0) {
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % kStages;
        if (kb >= kStages &&
            !mamba_scan::mbar_wait(&sm.empty[s], (uint32_t)((kb / kStages) - 1) & 1u,
                                   &g_gemm_device_error))
          break;
        mamba_scan::mbar_arrive_expect_tx(&sm.full[s], C::kStageBytes);
        const int k0 = (kb_begin + kb) * BK;
        tma_load_2d(sm.a_hi[s], &maps.a_hi, &sm.full[s], k0, m0);
        tma_load_2d(sm.a_lo[s], &maps.a_lo, &sm.full[s], k0, m0);
        tma_load_2d(sm.b_hi[s], &maps.b_hi, &sm.full[s], k0, n0);
        tma_load_2d(sm.b_lo[s], &maps.b_lo, &sm.full[s], k0, n0);
      }
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      // K block kb accumulates from zero into TMEM buffer kb & 1 (hi*hi in
      // its first BN columns, the corrections in the next BN), which the
      // accumulator warps drain before block kb + 2 reuses it.
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % kStages, b = kb & 1;
        if (kb >= 2 && !mamba_scan::mbar_wait(&sm.acc_empty[b], (uint32_t)((kb >> 1) - 1) & 1u,
                                              &g_gemm_device_error))
          break;
        if (!mamba_scan::mbar_wait(&sm.full[s], (uint32_t)(kb / kStages) & 1u,
                                   &g_gemm_device_error))
          break;
        tc_fence_after();
        const uint32_t t = tmem + (uint32_t)(b * BN);
        const uint64_t ah = sw128_desc(sm.a_hi[s]), al = sw128_desc(sm.a_lo[s]);
        const uint64_t bh = sw128_desc(sm.b_hi[s]), bl = sw128_desc(sm.b_lo[s]);
#pragma unroll
        for (int k = 0; k < BK / 8; ++k) {
          const uint64_t off = (uint64_t)(k * 32) >> 4;  // 8 tf32 = 32 bytes along the row
          mma_tf32<BN>(t, al + off, bh + off, k > 0 ? 1u : 0u);
          mma_tf32<BN>(t, ah + off, bl + off, 1u);
        }
#pragma unroll
        for (int k = 0; k < BK / 8; ++k) {
          const uint64_t off = (uint64_t)(k * 32) >> 4;
          mma_tf32<BN>(t, ah + off, bh + off, 1u);
        }
        mma_commit(&sm.empty[s]);     // the stage is free once these MMAs have read it
        mma_commit(&sm.acc_full[b]);  // and the block's sums are ready
      }
    }
    __syncwarp();
  } else {
    // accumulator warps: each thread keeps kAccCols sums of its tile row in
    // registers, adding every K block's (hi*hi + corrections) with
    // round-to-nearest fp32 adds (packed pairs).
    const int quarter = warp & 3, col0 = (warp >> 2) * kAccCols;
    float2 acc[kAccCols / 2];
#pragma unroll
    for (int j = 0; j < kAccCols / 2; ++j) acc[j] = make_float2(0.f, 0.f);
    bool ok = true;
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)col0;
    for (int kb = 0; kb < nk; ++kb) {
      const int b = kb & 1;
      ok = mamba_scan::mbar_wait(&sm.acc_full[b], (uint32_t)(kb >> 1) & 1u, &g_gemm_device_error);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const uint32_t t = lane_base + (uint32_t)(b * BN);
      // 64 columns per wait for the 128-column tile; 32 for the 192-column
      // one, whose 14 warps leave 128 registers per thread
      constexpr int kMax = (C::kThreads <= 320) ? 64 : 32;
#pragma unroll
      for (int c0 = 0; c0 < kAccCols; c0 += kMax) {
        uint32_t v[kMax];
#pragma unroll
        for (int c = 0; c < kMax; c += 32)
          tmem_ld32(t + (uint32_t)(c0 + c), *reinterpret_cast<uint32_t(*)[32]>(v + c));
        tmem_wait();
#pragma unroll
        for (int j = 0; j < kMax / 2; ++j)
          acc[c0 / 2 + j] = __fadd2_rn(acc[c0 / 2 + j], make_float2(__uint_as_float(v[2 * j]),
                                                                    __uint_as_float(v[2 * j + 1])));
      }
      tc_fence_before();
      mbar_arrive(&sm.acc_empty[b]);
    }
    // after the last block every stage has landed and been read by the
    // MMAs: the stage buffers are free for the transposes of the stores
    if (__all_sync(0xffffffffu, ok))
      store_sums<kAccCols>(p, p.c + (int64_t)blockIdx.z * p.slice, acc,
                           (int64_t)m0 + quarter * 32, (int64_t)n0 + col0,
                           reinterpret_cast<float*>(&sm) + warp * kStoreScratch<kAccCols>, lane);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(C::kTmemCols)
                 : "memory");
  }
}

// ------------------------------------------------- CTA-pair (2-SM) kernel

// The same GEMM on a pair of CTAs (a cluster of 2 on neighbouring SMs) that
// computes one 256 x BN output tile with tcgen05.mma.cta_group::2: each CTA
// holds 128 rows of the A tiles and half (BN/2 rows) of the B tiles, and the
// tensor cores of the pair read both halves. Per K block a CTA streams
// (2 * 128 + 2 * BN/2) x 128 bytes instead of (2 * 128 + 2 * BN) x 128 for
// the same 128 x BN outputs of its own: the B tile crosses from L2 once per
// pair. Each CTA loads its own halves by plain TMA tile loads, completing on
// the leader CTA's stage barrier; the leader's MMA warp issues the MMAs and
// signals both CTAs' barriers (stage free, accumulator ready) at once; each
// CTA drains its own 128 TMEM lanes (its 128 tile rows) and tells the
// leader through its accumulator-free barrier. Every wait is bounded.
template <int BN_, int kStages_>
struct Cfg2 {
  static constexpr int BN = BN_, kStages = kStages_;
  static constexpr int kHalfN = BN / 2;  // B rows held by each CTA of the pair
  static constexpr int kAccCols = 64;
  static constexpr int kAccWarps = 4 * BN / kAccCols;
  static constexpr int kAccThreads = 32 * kAccWarps;
  static constexpr int kProducerWarp = kAccWarps, kMmaWarp = kAccWarps + 1;
  static constexpr int kThreads = 32 * (kAccWarps + 2);
  static constexpr uint32_t kATile = BM * BK * 4, kBTile = kHalfN * BK * 4;
  static constexpr uint32_t kStageBytes = 2 * kATile + 2 * kBTile;  // one CTA's share
  static constexpr int kTmemCols = (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
  struct __align__(1024) Smem {
    float a_hi[kStages][BM * BK];
    float a_lo[kStages][BM * BK];
    float b_hi[kStages][kHalfN * BK];
    float b_lo[kStages][kHalfN * BK];
    uint64_t full[kStages];   // leader: both CTAs' tiles of a stage have landed
    uint64_t empty[kStages];  // each CTA: the pair's MMAs have read the stage
    uint64_t acc_full[2];     // each CTA: a K block's sums are in TMEM buffer b
    uint64_t acc_empty[2];    // leader: both CTAs' accumulator warps have read buffer b
    uint32_t tmem_base;
  };
  static constexpr size_t kSmemBytes = sizeof(Smem) + 1024;
  static_assert(kSmemBytes <= 227 * 1024, "shared memory per CTA");
  static constexpr size_t kStageBuffers = (size_t)kStages * kStageBytes;  // a_hi .. b_lo
};
using Cfg2x64 = Cfg2<64, 4>;
using Cfg2x128 = Cfg2<128, 4>;
using Cfg2x192 = Cfg2<192, 3>;
using Cfg2x256 = Cfg2<256, 3>;

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cluster address of the same shared-memory location in CTA `rank`.
__device__ __forceinline__ uint32_t map_to_rank(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}

// 2-D TMA load into this CTA's shared memory, completing on the mbarrier at
// shared::cluster address `bar` (the pair's leader).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar,
                                                 int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

// Instruction descriptor of kind::tf32 for the pair: M = 256.
template <int BN>
__device__ __forceinline__ void mma_tf32_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                              uint32_t accumulate) {
  constexpr uint32_t kInstrDesc = (1u << 4) | (2u << 7) | (2u << 10) |
                                  ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
  asm volatile(
      "{\n\t"
      ".reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t"
      "}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(kInstrDesc), "r"(accumulate)
      : "memory");
}

// One arrival on the barrier at the same offset in both CTAs of the pair
// once the MMAs issued so far have completed.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"((uint16_t)0x3)
      : "memory");
}

// An arrival on a barrier of either CTA of the pair (CTA-scope release: the
// waiting side orders TMEM accesses through tcgen05 fences, not through
// this arrival, so no cluster-wide memory fence is needed).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}

template <class C>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(C::kThreads, 1)
    gemm_tf32x3_pair_kernel(const __grid_constant__ GemmMaps maps, const GemmParams p) {
  constexpr int BN = C::BN, kStages = C::kStages, kAccCols = C::kAccCols;
  static_assert((size_t)C::kAccWarps * kStoreScratch<C::kAccCols> * 4 <= C::kStageBuffers,
                "the store transposes fit in the stage buffers");
  constexpr int kProducerWarp = C::kProducerWarp, kMmaWarp = C::kMmaWarp;
  extern __shared__ uint8_t smem_raw[];
  typename C::Smem& sm = *reinterpret_cast<typename C::Smem*>(
      smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0: the leader, which issues the MMAs
  // pairs along M vary fastest; this CTA's A rows and B rows
  const int m0 = (blockIdx.x >> 1) * 256 + (int)rank * BM;
  const int n0 = blockIdx.y * BN;
  // this CTA's K blocks: [kb_begin, kb_begin + nk)
  const int kb_begin = (int)blockIdx.z * p.kb_per_split;
  const int nk = min((p.K + BK - 1) / BK - kb_begin, p.kb_per_split);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mamba_scan::mbar_init(&sm.full[s], 1);
      mamba_scan::mbar_init(&sm.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mamba_scan::mbar_init(&sm.acc_full[b], 1);
      mamba_scan::mbar_init(&sm.acc_empty[b], 2 * C::kAccWarps);
    }
    mamba_scan::fence_mbarrier_init();
  }
  if (warp == kProducerWarp && lane == 0) {
    mamba_scan::prefetch_tensormap(&maps.a_hi);
    mamba_scan::prefetch_tensormap(&maps.a_lo);
    mamba_scan::prefetch_tensormap(&maps.b_hi);
    mamba_scan::prefetch_tensormap(&maps.b_lo);
  }
  if (warp == 0) {  // the same warp of both CTAs allocates the pair's TMEM columns
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&sm.tmem_base)),
                 "r"(C::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  mamba_scan::pdl_trigger();
  mamba_scan::pdl_wait();

  if (warp == kProducerWarp) {
    if (lane == 0) {
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % kStages;
        if (kb >= kStages &&
            !mamba_scan::mbar_wait(&sm.empty[s], (uint32_t)((kb / kStages) - 1) & 1u,
                                   &g_gemm_device_error))
          break;
        // the leader's barrier counts both CTAs' bytes of the stage
        if (rank == 0) mamba_scan::mbar_arrive_expect_tx(&sm.full[s], 2 * C::kStageBytes);
        const uint32_t bar = map_to_rank(&sm.full[s], 0);
        const int k0 = (kb_begin + kb) * BK;
        tma_load_2d_pair(sm.a_hi[s], &maps.a_hi, bar, k0, m0);
        tma_load_2d_pair(sm.a_lo[s], &maps.a_lo, bar, k0, m0);
        tma_load_2d_pair(sm.b_hi[s], &maps.b_hi, bar, k0, n0 + (int)rank * C::kHalfN);
        tma_load_2d_pair(sm.b_lo[s], &maps.b_lo, bar, k0, n0 + (int)rank * C::kHalfN);
      }
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    if (lane == 0 && rank == 0) {
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % kStages, b = kb & 1;
        if (kb >= 2 && !mamba_scan::mbar_wait(&sm.acc_empty[b], (uint32_t)((kb >> 1) - 1) & 1u,
                                              &g_gemm_device_error))
          break;
        if (!mamba_scan::mbar_wait(&sm.full[s], (uint32_t)(kb / kStages) & 1u,
                                   &g_gemm_device_error))
          break;
        tc_fence_after();
        const uint32_t t = tmem + (uint32_t)(b * BN);
        const uint64_t ah = sw128_desc(sm.a_hi[s]), al = sw128_desc(sm.a_lo[s]);
        const uint64_t bh = sw128_desc(sm.b_hi[s]), bl = sw128_desc(sm.b_lo[s]);
#pragma unroll
        for (int k = 0; k < BK / 8; ++k) {
          const uint64_t off = (uint64_t)(k * 32) >> 4;
          mma_tf32_pair<BN>(t, al + off, bh + off, k > 0 ? 1u : 0u);
          mma_tf32_pair<BN>(t, ah + off, bl + off, 1u);
        }
#pragma unroll
        for (int k = 0; k < BK / 8; ++k) {
          const uint64_t off = (uint64_t)(k * 32) >> 4;
          mma_tf32_pair<BN>(t, ah + off, bh + off, 1u);
        }
        mma_commit_pair(&sm.empty[s]);     // both CTAs may refill the stage
        mma_commit_pair(&sm.acc_full[b]);  // both CTAs' sums of the block are ready
      }
    }
    __syncwarp();
  } else {
    const int quarter = warp & 3, col0 = (warp >> 2) * kAccCols;
    float2 acc[kAccCols / 2];
#pragma unroll
    for (int j = 0; j < kAccCols / 2; ++j) acc[j] = make_float2(0.f, 0.f);
    bool ok = true;
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)col0;
    const uint32_t leader_empty0 = map_to_rank(&sm.acc_empty[0], 0);
    const uint32_t leader_empty1 = map_to_rank(&sm.acc_empty[1], 0);
    for (int kb = 0; kb < nk; ++kb) {
      const int b = kb & 1;
      ok = mamba_scan::mbar_wait(&sm.acc_full[b], (uint32_t)(kb >> 1) & 1u, &g_gemm_device_error);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const uint32_t t = lane_base + (uint32_t)(b * BN);
      constexpr int kMax = 32;
#pragma unroll
      for (int c0 = 0; c0 < kAccCols; c0 += kMax) {
        uint32_t v[kMax];
        tmem_ld32(t + (uint32_t)c0, v);
        tmem_wait();
#pragma unroll
        for (int j = 0; j < kMax / 2; ++j)
          acc[c0 / 2 + j] = __fadd2_rn(acc[c0 / 2 + j], make_float2(__uint_as_float(v[2 * j]),
                                                                    __uint_as_float(v[2 * j + 1])));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(b ? leader_empty1 : leader_empty0);
    }
    // the last block's commit reached this CTA after every MMA of the pair
    // completed: both CTAs' stages have landed and been read
    if (__all_sync(0xffffffffu, ok))
      store_sums<kAccCols>(p, p.c + (int64_t)blockIdx.z * p.slice, acc,
                           (int64_t)m0 + quarter * 32, (int64_t)n0 + col0,
                           reinterpret_cast<float*>(&sm) + warp * kStoreScratch<kAccCols>, lane);
  }
  tc_fence_before();
  cluster_sync_all();  // the pair is done with TMEM and with each other's barriers
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(C::kTmemCols)
                 : "memory");
  }
}

// ------------------------------------------------------- split-K reduction

// C = (C_in +) the sum of the `splits` partial products in ws, added in split
// order (ws[0] + ws[1] + ...; fixed, so results do not depend on which CTA
// finished first). The partials are compact M x N slices `slice` floats
// apart, laid out like C: element (m, n) at m + n * M when C is column-major
// (col_major), m * N + n otherwise. `dense`: C and C_in (when given) are that
// same compact layout, 16-byte aligned, and M * N is a multiple of 4, so
// whole float4s go at once.
__global__ void __launch_bounds__(256)
    split_reduce_kernel(const float* __restrict__ ws, int splits, int64_t slice, int M, int N,
                        int col_major, int dense, float* c, const float* c_in, int64_t ldc_m,
                        int64_t ldc_n) {
  mamba_scan::pdl_wait();  // the partial products are complete and visible
  mamba_scan::pdl_trigger();
  const int64_t total = (int64_t)M * N;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if (dense) {
    for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < total / 4; v += stride) {
      float4 s = reinterpret_cast<const float4*>(ws)[v];
      for (int z = 1; z < splits; ++z) {
        const float4 t = reinterpret_cast<const float4*>(ws + z * slice)[v];
        s.x += t.x;
        s.y += t.y;
        s.z += t.z;
        s.w += t.w;
      }
      if (c_in) {
        const float4 t = reinterpret_cast<const float4*>(c_in)[v];
        s = make_float4(t.x + s.x, t.y + s.y, t.z + s.z, t.w + s.w);
      }
      reinterpret_cast<float4*>(c)[v] = s;
    }
    return;
  }
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    float s = ws[i];
    for (int z = 1; z < splits; ++z) s += ws[z * slice + i];
    const int64_t m = col_major ? i % M : i / N, n = col_major ? i / M : i % N;
    const int64_t o = m * ldc_m + n * ldc_n;
    c[o] = c_in ? c_in[o] + s : s;
  }
}

// --------------------------------------------------------- tf32 hi/lo split

__device__ __forceinline__ float to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// hi = tf32(x), lo = tf32(x - hi) (x - hi is exact in fp32).
__device__ __forceinline__ void split1(float x, float& hi, float& lo) {
  hi = to_tf32(x);
  lo = to_tf32(x - hi);
}

// Row-contiguous source: grid (column blocks, rows); each thread splits 4
// consecutive elements of one row (vector loads and stores when the row
// starts and strides allow it).
__global__ void split_rows_kernel(const float* __restrict__ x, int cols, int64_t ldx,
                                  float* __restrict__ hi, float* __restrict__ lo, int64_t ld,
                                  bool vec) {
  mamba_scan::pdl_trigger();
  mamba_scan::pdl_wait();
  const int64_t r = blockIdx.y;
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (c >= cols) return;
  const float* xr = x + r * ldx;
  float* hr = hi + r * ld;
  float* lr = lo + r * ld;
  if (vec && c + 4 <= cols) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(xr + c));
    float4 h, l;
    split1(v.x, h.x, l.x);
    split1(v.y, h.y, l.y);
    split1(v.z, h.z, l.z);
    split1(v.w, h.w, l.w);
    *reinterpret_cast<float4*>(hr + c) = h;
    *reinterpret_cast<float4*>(lr + c) = l;
  } else {
    for (int j = c; j < c + 4 && j < cols; ++j) split1(__ldg(xr + j), hr[j], lr[j]);
  }
}

// Transposing source (out[r][c] = x[c][r], x rows of length ldx): 32 x 32
// tiles through shared memory, coalesced on both sides.
__global__ void split_transpose_kernel(const float* __restrict__ x, int rows, int cols,
                                       int64_t ldx, float* __restrict__ hi,
                                       float* __restrict__ lo, int64_t ld) {
  mamba_scan::pdl_trigger();
  mamba_scan::pdl_wait();
  __shared__ float t[32][33];
  const int r0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
#pragma unroll
  for (int j = ty; j < 32; j += 8) {
    const int c = c0 + j, r = r0 + tx;  // x[c][r]
    t[j][tx] = (c < cols && r < rows) ? __ldg(x + (int64_t)c * ldx + r) : 0.f;
  }
  __syncthreads();
#pragma unroll
  for (int j = ty; j < 32; j += 8) {
    const int r = r0 + j, c = c0 + tx;
    if (r < rows && c < cols) {
      float h, l;
      split1(t[tx][j], h, l);
      hi[(int64_t)r * ld + c] = h;
      lo[(int64_t)r * ld + c] = l;
    }
  }
}

int read_and_clear_error() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemm_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_gemm_device_error, &zero, sizeof(int));
  }
  return v;
}

}  // namespace mamba_gemm

namespace {

PFN_cuTensorMapEncodeTiled_v12000 gemm_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// [rows][K] fp32, row stride ld floats, boxes of 32 K x box_rows rows, 128-byte swizzle.
bool encode_operand(PFN_cuTensorMapEncodeTiled_v12000 enc, CUtensorMap* m, const float* ptr,
                    int64_t rows, int64_t K, int64_t ld, int box_rows) {
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  const cuuint32_t box[2] = {mamba_gemm::BK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int device_sms() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int v = cache[dev].load(std::memory_order_relaxed);
  if (v > 0) return v;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
    v = 148;
  cache[dev].store(v, std::memory_order_relaxed);
  return v;
}

// Tile width with the fewest waves x (128 + BN) (one CTA per SM; a CTA
// streams (2 * 128 + 2 * BN) x 32 x 4 bytes per K block); ties go wider.
int tile_width(int64_t M, int64_t N, int sms) {
  const int64_t m_tiles = (M + mamba_gemm::BM - 1) / mamba_gemm::BM;
  auto cost = [&](int64_t bn) {
    const int64_t tiles = m_tiles * ((N + bn - 1) / bn);
    return (tiles + sms - 1) / sms * (mamba_gemm::BM + bn);
  };
  int best = 192;
  for (int bn : {128, 64})
    if (cost(bn) < cost(best)) best = bn;
  return best;
}

template <class C>
cudaError_t launch_gemm(const mamba_gemm::GemmMaps& maps, const mamba_gemm::GemmParams& p,
                        int64_t m_tiles, int splits, cudaStream_t st) {
  static std::once_flag attr_once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(attr_once, [] {
    attr_err = cudaFuncSetAttribute(mamba_gemm::gemm_tf32x3_kernel<C>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)C::kSmemBytes);
  });
  if (attr_err != cudaSuccess) return attr_err;
  const int64_t n_tiles = (p.N + C::BN - 1) / C::BN;
  return mamba_scan::launch_pdl(mamba_gemm::gemm_tf32x3_kernel<C>,
                                dim3((unsigned)m_tiles, (unsigned)n_tiles, (unsigned)splits),
                                dim3(C::kThreads), C::kSmemBytes, st, maps, p);
}

// CTA pairs (gemm_tf32x3_pair_kernel): the pair tile width with the fewest
// waves x (128 + BN/2) (per CTA and K block it streams (2 * 128 + 2 * BN/2)
// rows of 128 bytes), or 0 when single CTAs cost less ((128 + BN) per CTA);
// ties go to pairs.
int pair_width(int64_t M, int64_t N, int sms, int single_bn) {
  const int64_t m_tiles = (M + mamba_gemm::BM - 1) / mamba_gemm::BM;
  const int64_t single = (m_tiles * ((N + single_bn - 1) / single_bn) + sms - 1) / sms *
                         (mamba_gemm::BM + single_bn);
  const int64_t pairs_m = (M + 255) / 256;
  int best = 0;
  int64_t best_cost = single;
  for (int bn : {256, 192, 128, 64}) {
    const int64_t ctas = 2 * pairs_m * ((N + bn - 1) / bn);
    const int64_t cost = (ctas + sms - 1) / sms * (mamba_gemm::BM + bn / 2);
    if (cost <= best_cost) {
      best = bn;
      best_cost = cost;
    }
  }
  return best;
}

// Tiling of one product: CTA pairs of width pair_bn (0: single CTAs of
// width bn), K split `splits` ways (1: unsplit) with kb_per_split K blocks
// each and partial slices `slice` floats apart.
struct GemmPlan {
  int pair_bn, bn, splits, kb_per_split;
  int64_t slice;
  size_t workspace_bytes() const { return splits > 1 ? (size_t)splits * slice * 4 : 0; }
};

// Modelled SM cycles of a tiling, for choosing whether to split K: a K block
// costs a CTA the larger of its MMAs (12 x 128 x BN x 8 tf32 FMAs at ~1925
// per cycle) and its operand delivery ((2 * 128 + 2 * B rows) x 128 bytes at
// ~50 bytes per cycle per SM with every SM streaming); a tile adds ~10k
// cycles (start-up, pipeline fill and drain, stores); a split adds the
// reduction (one launch, then the partials and C through L2 at ~8 KB per
// cycle).
double plan_cycles(int64_t M, int64_t N, int64_t K, int sms, int pair_bn, int bn, int splits) {
  const int64_t nk = (K + mamba_gemm::BK - 1) / mamba_gemm::BK;
  const int64_t kbs = (nk + splits - 1) / splits;
  const int w = pair_bn ? pair_bn : bn;
  const int b_rows = pair_bn ? pair_bn / 2 : bn;
  const double block = std::max(6.4 * w, (2.0 * mamba_gemm::BM + 2.0 * b_rows) * 128.0 / 50.0);
  const int64_t ctas = (pair_bn ? 2 * ((M + 255) / 256) : (M + mamba_gemm::BM - 1) / mamba_gemm::BM) *
                       ((N + w - 1) / w) * splits;
  const int64_t waves = (ctas + sms - 1) / sms;
  double t = (double)waves * ((double)kbs * block + 10000.0);
  if (splits > 1) t += 2000.0 + (double)M * N * (splits + 2) * 4.0 / 8192.0;
  return t;
}

// The tiling of an M x N x K product: the unsplit choice of tile_width and
// pair_width, or, when the output has too few tiles to keep the SMs busy,
// the split of K (2..16 ways, every split at least one K block) that the
// model makes at least 25% faster.
GemmPlan plan_gemm(int64_t M, int64_t N, int64_t K, int sms, bool allow_split) {
  GemmPlan plan;
  plan.bn = tile_width(M, N, sms);
  plan.pair_bn = pair_width(M, N, sms, plan.bn);
  plan.splits = 1;
  plan.kb_per_split = (int)((K + mamba_gemm::BK - 1) / mamba_gemm::BK);
  plan.slice = 0;
  if (!allow_split) return plan;
  const int64_t nk = plan.kb_per_split;
  const double unsplit = plan_cycles(M, N, K, sms, plan.pair_bn, plan.bn, 1);
  double best = 0.75 * unsplit;
  for (int pair_bn : {256, 192, 128, 64, 0})
    for (int bn : {192, 128, 64}) {
      if (pair_bn && bn != 192) continue;  // bn is unused with pairs
      for (int splits = 2; splits <= 16; ++splits) {
        const int64_t kbs = (nk + splits - 1) / splits;
        if (kbs * (splits - 1) >= nk) break;  // the last split would be empty
        const double t = plan_cycles(M, N, K, sms, pair_bn, bn, splits);
        if (t < best) {
          best = t;
          plan.pair_bn = pair_bn;
          plan.bn = bn;
          plan.splits = splits;
          plan.kb_per_split = (int)kbs;
        }
      }
    }
  if (plan.splits > 1) plan.slice = (M * N + 3) / 4 * 4;  // 16-byte aligned slices
  return plan;
}

template <class C>
cudaError_t launch_gemm_pair(const mamba_gemm::GemmMaps& maps, const mamba_gemm::GemmParams& p,
                             int splits, cudaStream_t st) {
  static std::once_flag attr_once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(attr_once, [] {
    attr_err = cudaFuncSetAttribute(mamba_gemm::gemm_tf32x3_pair_kernel<C>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)C::kSmemBytes);
  });
  if (attr_err != cudaSuccess) return attr_err;
  const int64_t pairs_m = (p.M + 255) / 256, n_tiles = (p.N + C::BN - 1) / C::BN;
  return mamba_scan::launch_pdl(mamba_gemm::gemm_tf32x3_pair_kernel<C>,
                                dim3((unsigned)(2 * pairs_m), (unsigned)n_tiles, (unsigned)splits),
                                dim3(C::kThreads), C::kSmemBytes, st, maps, p);
}

bool overlap(const void* a, int64_t abytes, const void* b, int64_t bbytes) {
  const auto a0 = reinterpret_cast<uintptr_t>(a), b0 = reinterpret_cast<uintptr_t>(b);
  return a0 < b0 + (uintptr_t)bbytes && b0 < a0 + (uintptr_t)abytes;
}

}  // namespace

extern "C" {

int mamba_split_tf32(const float* x, int64_t rows, int64_t cols, int64_t ldx, int transpose,
                     float* hi, float* lo, int64_t ld, void* stream) {
  using mamba_scan::set_last_error;
  if (rows < 0 || cols < 0 || ld < cols)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "split_tf32: bad sizes");
  if (rows == 0 || cols == 0) return MAMBA_SCAN_OK;
  if (!x || !hi || !lo)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "split_tf32: NULL pointer");
  if (transpose ? ldx < rows : ldx < cols)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "split_tf32: ldx too small");
  if (rows > ((int64_t)1 << 31) || cols > ((int64_t)1 << 31) ||
      (!transpose && rows * cols > ((int64_t)1 << 40)))
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "split_tf32: too large");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (transpose) {
    const dim3 grid((unsigned)((rows + 31) / 32), (unsigned)((cols + 31) / 32));
    if (grid.y > 65535)
      return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "split_tf32: too many columns");
    const cudaError_t e = mamba_scan::launch_pdl(mamba_gemm::split_transpose_kernel, grid,
                                                 dim3(32, 8), 0, st, x, (int)rows, (int)cols,
                                                 ldx, hi, lo, ld);
    if (e != cudaSuccess) return set_last_error(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));
  } else {
    const bool vec = al16(x) && al16(hi) && al16(lo) && ldx % 4 == 0 && ld % 4 == 0;
    for (int64_t r0 = 0; r0 < rows; r0 += 65535) {  // grid.y holds at most 65535 rows
      const dim3 grid((unsigned)((cols + 4 * 128 - 1) / (4 * 128)),
                      (unsigned)std::min<int64_t>(65535, rows - r0));
      const cudaError_t e = mamba_scan::launch_pdl(mamba_gemm::split_rows_kernel, grid, dim3(128),
                                                   0, st, x + r0 * ldx, (int)cols, ldx,
                                                   hi + r0 * ld, lo + r0 * ld, ld, vec);
      if (e != cudaSuccess) return set_last_error(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));
    }
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_last_error(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));
  return MAMBA_SCAN_OK;
}

size_t mamba_gemm_tf32x3_workspace_size(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0 || M > ((int64_t)1 << 30) || N > ((int64_t)1 << 30) ||
      K > ((int64_t)1 << 30))
    return 0;
  return plan_gemm(M, N, K, device_sms(), true).workspace_bytes();
}

int mamba_gemm_tf32x3(const float* a_hi, const float* a_lo, int64_t lda, const float* b_hi,
                      const float* b_lo, int64_t ldb, const float* c_in, float* c,
                      int64_t ldc_m, int64_t ldc_n, int64_t M, int64_t N, int64_t K,
                      void* stream) {
  return mamba_gemm_tf32x3_ws(a_hi, a_lo, lda, b_hi, b_lo, ldb, c_in, c, ldc_m, ldc_n, M, N, K,
                              nullptr, 0, stream);
}

int mamba_gemm_tf32x3_ws(const float* a_hi, const float* a_lo, int64_t lda, const float* b_hi,
                         const float* b_lo, int64_t ldb, const float* c_in, float* c,
                         int64_t ldc_m, int64_t ldc_n, int64_t M, int64_t N, int64_t K,
                         void* workspace, size_t workspace_bytes, void* stream) {
  using mamba_scan::set_last_error;
  if (M < 0 || N < 0 || K < 0)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "gemm_tf32x3: negative size");
  if (M == 0 || N == 0) return MAMBA_SCAN_OK;
  if (K == 0)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "gemm_tf32x3: K must be positive");
  if (M > ((int64_t)1 << 30) || N > ((int64_t)1 << 30) || K > ((int64_t)1 << 30))
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "gemm_tf32x3: size exceeds 2^30");
  if (!a_hi || !a_lo || !b_hi || !b_lo || !c)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "gemm_tf32x3: NULL pointer");
  if (lda < K || ldb < K || lda % 4 != 0 || ldb % 4 != 0)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT,
                          "gemm_tf32x3: lda and ldb must be >= K and multiples of 4");
  if (!al16(a_hi) || !al16(a_lo) || !al16(b_hi) || !al16(b_lo))
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT,
                          "gemm_tf32x3: operands must be 16-byte aligned");
  if (ldc_m <= 0 || ldc_n <= 0)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "gemm_tf32x3: C strides must be positive");
  // C is written while the operands are read by other CTAs: no overlap.
  const int64_t c_bytes = ((M - 1) * ldc_m + (N - 1) * ldc_n + 1) * 4;
  const int64_t a_bytes = ((M - 1) * lda + K) * 4, b_bytes = ((N - 1) * ldb + K) * 4;
  const void* ops[4] = {a_hi, a_lo, b_hi, b_lo};
  const int64_t op_bytes[4] = {a_bytes, a_bytes, b_bytes, b_bytes};
  for (int i = 0; i < 4; ++i)
    if (overlap(c, c_bytes, ops[i], op_bytes[i]) ||
        (c_in && overlap(c_in, c_bytes, ops[i], op_bytes[i])))
      return set_last_error(MAMBA_SCAN_ERR_ALIASING, "gemm_tf32x3: C overlaps an operand");
  if (c_in && c_in != c && overlap(c_in, c_bytes, c, c_bytes))
    return set_last_error(MAMBA_SCAN_ERR_ALIASING,
                          "gemm_tf32x3: c_in must be C itself or not overlap it");
  const int64_t m_tiles = (M + mamba_gemm::BM - 1) / mamba_gemm::BM;
  if (m_tiles > 0x7FFFFFFF || (N + 63) / 64 > 65535)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "gemm_tf32x3: too many tiles");
  const GemmPlan plan = plan_gemm(M, N, K, device_sms(), workspace != nullptr);
  const bool split = plan.splits > 1;
  if (split) {
    if (workspace_bytes < plan.workspace_bytes())
      return set_last_error(MAMBA_SCAN_ERR_WORKSPACE,
                            "gemm_tf32x3: the workspace holds " + std::to_string(workspace_bytes) +
                                " bytes, this product needs " +
                                std::to_string(plan.workspace_bytes()) +
                                " (mamba_gemm_tf32x3_workspace_size)");
    if (!al16(workspace))
      return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT,
                            "gemm_tf32x3: the workspace must be 16-byte aligned");
    const int64_t ws_bytes = (int64_t)plan.workspace_bytes();
    for (int i = 0; i < 4; ++i)
      if (overlap(workspace, ws_bytes, ops[i], op_bytes[i]))
        return set_last_error(MAMBA_SCAN_ERR_ALIASING,
                              "gemm_tf32x3: the workspace overlaps an operand");
    if (overlap(workspace, ws_bytes, c, c_bytes) ||
        (c_in && overlap(workspace, ws_bytes, c_in, c_bytes)))
      return set_last_error(MAMBA_SCAN_ERR_ALIASING, "gemm_tf32x3: the workspace overlaps C");
  }
  auto enc = gemm_encode_fn();
  mamba_gemm::GemmMaps maps;
  std::memset(&maps, 0, sizeof maps);
  const int b_box = plan.pair_bn ? plan.pair_bn / 2 : plan.bn;  // a CTA of a pair holds half of B's tile
  if (!enc || !encode_operand(enc, &maps.a_hi, a_hi, M, K, lda, mamba_gemm::BM) ||
      !encode_operand(enc, &maps.a_lo, a_lo, M, K, lda, mamba_gemm::BM) ||
      !encode_operand(enc, &maps.b_hi, b_hi, N, K, ldb, b_box) ||
      !encode_operand(enc, &maps.b_lo, b_lo, N, K, ldb, b_box))
    return set_last_error(MAMBA_SCAN_ERR_CUDA, "gemm_tf32x3: tensor map encoding failed");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // a split writes compact partial slices laid out like C (column-major when
  // m is C's faster index), without C_in; the reduction then writes C
  const bool col_major = ldc_m < ldc_n;
  mamba_gemm::GemmParams p{c, c_in, ldc_m, ldc_n, (int)M, (int)N, (int)K,
                           plan.kb_per_split, 0};
  if (split) {
    p.c = static_cast<float*>(workspace);
    p.c_in = nullptr;
    p.ldc_m = col_major ? 1 : N;
    p.ldc_n = col_major ? M : 1;
    p.slice = plan.slice;
  }
  const int sp = plan.splits;
  cudaError_t e;
  if (plan.pair_bn == 256) e = launch_gemm_pair<mamba_gemm::Cfg2x256>(maps, p, sp, st);
  else if (plan.pair_bn == 192) e = launch_gemm_pair<mamba_gemm::Cfg2x192>(maps, p, sp, st);
  else if (plan.pair_bn == 128) e = launch_gemm_pair<mamba_gemm::Cfg2x128>(maps, p, sp, st);
  else if (plan.pair_bn == 64) e = launch_gemm_pair<mamba_gemm::Cfg2x64>(maps, p, sp, st);
  else if (plan.bn == 192) e = launch_gemm<mamba_gemm::Cfg192>(maps, p, m_tiles, sp, st);
  else if (plan.bn == 128) e = launch_gemm<mamba_gemm::Cfg128>(maps, p, m_tiles, sp, st);
  else e = launch_gemm<mamba_gemm::Cfg64>(maps, p, m_tiles, sp, st);
  if (e != cudaSuccess) return set_last_error(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));
  if (split) {
    const bool dense = (col_major ? (ldc_m == 1 && ldc_n == M) : (ldc_n == 1 && ldc_m == N)) &&
                       al16(c) && (!c_in || al16(c_in)) && (M * N) % 4 == 0;
    const int64_t items = dense ? M * N / 4 : M * N;
    const int64_t blocks = std::min<int64_t>((items + 255) / 256, (int64_t)device_sms() * 8);
    e = mamba_scan::launch_pdl(mamba_gemm::split_reduce_kernel, dim3((unsigned)blocks), dim3(256),
                               0, st, static_cast<const float*>(workspace), plan.splits,
                               plan.slice, (int)M, (int)N, (int)col_major, (int)dense, c, c_in,
                               ldc_m, ldc_n);
    if (e != cudaSuccess) return set_last_error(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));
  }
  return MAMBA_SCAN_OK;
}

}  // extern "C"
