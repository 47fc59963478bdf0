// Selective-scan kernels for sm_100a.
//
// Re-designs the reference plugin's compute loop
// (acmiyaguchi/mamba-onnx src/native/cpp/selective_scan.cc:232-305; Zig
// processOneDim, src/native/zig/selective_scan.zig:307-383) for a B200:
//
// * one CTA = one warp = 32 consecutive (b, d) rows of one batch entry; each
//   lane owns one row and keeps its 16 state values in registers (the
//   reference keeps them in two AVX registers, cc:241-242), so the C·h
//   contraction over d_state is a register reduction with no shuffles;
// * the sequence is streamed in tiles of 16 steps. u/delta/z tiles
//   ([32 rows][16 steps], L contiguous) and B/C tiles ([16 steps][16 states])
//   are fetched by TMA into a 2-stage shared-memory ring (mbarrier
//   completion), read back as float4 through the 64-byte swizzle so the
//   per-row reads are bank-conflict free, and B/C values are warp-wide
//   broadcasts; outputs go through a swizzled shared tile and a TMA store;
// * the per-state update runs on packed fp32x2 FMAs (FFMA2);
// * long sequences with few rows are split into chunks: an aggregate pass
//   computes, per (row, chunk), the chunk's end state from zero and its decay
//   prod(abar) (exp(A*sum(delta)) for the exact variants); the emit pass
//   folds the aggregates of the earlier chunks into its carry-in,
//   h_in = P*h_in + h_end, and re-runs its chunk from there.
//
// A plain-load tile path (no TMA) covers inputs that TMA cannot describe
// (seqlen not a multiple of 4, or pointers not 16-byte aligned); it uses the
// same shared-memory layout and the same math.
#include "scan_device.cuh"
#include "scan_kernels.h"

namespace mamba_scan {

// Device-wide error word (MAMBA_SCAN_ERR_* codes) set by a bounded wait that
// gave up; read and cleared by the host through mamba_scan_check_device_error().
__device__ int g_scan_device_error = 0;

#ifndef MAMBA_SCAN_ACC
#define MAMBA_SCAN_ACC 2
#endif
// Independent partial sums per step in the C.h contraction (2, 4 or 8).
constexpr int kAcc = MAMBA_SCAN_ACC;

// --------------------------------------------------------------- tile math

// One 16-step tile for the calling lane's row. Reads the swizzled u/delta/z
// tiles and the B/C tiles, updates h (and the decay product P, or the delta
// sum S, in aggregate mode) and, in emit mode, writes y into the swizzled
// output tile `os`. kPartial masks steps >= n_valid (the ragged last tile).
template <int V, int M, bool kPartial>
__device__ __forceinline__ void compute_tile(const float* us,
                                             const float* __restrict__ ds,
                                             const float* __restrict__ zs,
                                             const float* __restrict__ Bs,
                                             const float* __restrict__ Cs, float* os,
                                             int row, float2 (&h)[8], float2 (&P)[8], float& S,
                                             const float2 (&Ar)[8], float dskip, float bias,
                                             float bias_l2e, int n_valid) {
  using Tr = VariantTraits<V>;
  const float2 one2 = make_float2(1.f, 1.f);
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int off = row * kT + (((c ^ (row >> 1)) & 3) << 2);
    const float4 u4 = *reinterpret_cast<const float4*>(us + off);
    const float4 d4 = *reinterpret_cast<const float4*>(ds + off);
    float uu[4] = {u4.x, u4.y, u4.z, u4.w};
    float dd[4] = {d4.x, d4.y, d4.z, d4.w};
    float gate[4] = {1.f, 1.f, 1.f, 1.f};
    if (Tr::fused) {
#pragma unroll
      for (int j = 0; j < 4; ++j) dd[j] = softplus<Tr::exact>(dd[j], bias, bias_l2e);
      if (M == kEmit) {
        const float4 z4 = *reinterpret_cast<const float4*>(zs + off);
        gate[0] = silu<Tr::exact>(z4.x);
        gate[1] = silu<Tr::exact>(z4.y);
        gate[2] = silu<Tr::exact>(z4.z);
        gate[3] = silu<Tr::exact>(z4.w);
      }
    }
    if (kPartial) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (4 * c + j >= n_valid) dd[j] = 0.f;  // abar = 1, input term 0: h is held
    }
    float yy[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int t = 4 * c + j;
      const float dt = dd[j];
      const float du = dt * uu[j];
      const float2 dt2 = make_float2(dt, dt);
      const float2 du2 = make_float2(du, du);
      const float4* Bt = reinterpret_cast<const float4*>(Bs + t * kN);
      const float4* Ct = reinterpret_cast<const float4*>(Cs + t * kN);
      float2 a[8], bu[8];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 bq = Bt[q];
        if (Tr::exact) {
          // abar = exp(delta*A) = 2^(delta * A*log2(e)); Ar holds A*log2(e)
          const float2 x0 = mul2(dt2, Ar[2 * q]);
          const float2 x1 = mul2(dt2, Ar[2 * q + 1]);
          a[2 * q] = make_float2(ex2_approx(x0.x), ex2_approx(x0.y));
          a[2 * q + 1] = make_float2(ex2_approx(x1.x), ex2_approx(x1.y));
        } else {
          // abar = 1 + delta*A (cc:275-282 written as (1+dA)h + dBu)
          a[2 * q] = fma2(dt2, Ar[2 * q], one2);
          a[2 * q + 1] = fma2(dt2, Ar[2 * q + 1], one2);
        }
        bu[2 * q] = mul2(du2, make_float2(bq.x, bq.y));
        bu[2 * q + 1] = mul2(du2, make_float2(bq.z, bq.w));
      }
#pragma unroll
      for (int n = 0; n < 8; ++n) h[n] = fma2(a[n], h[n], bu[n]);
      if (M == kAggregate) {
        if (!Tr::exact) {
#pragma unroll
          for (int n = 0; n < 8; ++n) P[n] = mul2(P[n], a[n]);
        } else {
          S += dt;
        }
        yy[j] = 0.f;
      } else {
        float2 acc[kAcc];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 cq = Ct[q];
          const int i0 = (2 * q) % kAcc, i1 = (2 * q + 1) % kAcc;
          if (2 * q < kAcc) acc[i0] = mul2(make_float2(cq.x, cq.y), h[2 * q]);
          else acc[i0] = fma2(make_float2(cq.x, cq.y), h[2 * q], acc[i0]);
          if (2 * q + 1 < kAcc) acc[i1] = mul2(make_float2(cq.z, cq.w), h[2 * q + 1]);
          else acc[i1] = fma2(make_float2(cq.z, cq.w), h[2 * q + 1], acc[i1]);
        }
#pragma unroll
        for (int w = kAcc / 2; w >= 1; w /= 2)
#pragma unroll
          for (int i = 0; i < w; ++i) acc[i] = add2(acc[i], acc[i + w]);
        float y = acc[0].x + acc[0].y;                  // sum_n C*h (cc:285-296)
        y = fmaf(dskip, uu[j], y);                      // + D*u (cc:297)
        yy[j] = Tr::fused ? y * gate[j] : y;            // * silu(z) (cc:300-302)
      }
    }
    if (M == kEmit) *reinterpret_cast<float4*>(os + off) = make_float4(yy[0], yy[1], yy[2], yy[3]);
  }
}

// ------------------------------------------------- plain-load tile transfer

// Fill stage 0 of the ring with the tile starting at t0, using ordinary
// coalesced loads (two rows of 16 steps per warp instruction), zero-filling
// beyond seqlen / dim like the TMA path does.
template <int V, int M>
__device__ __forceinline__ void load_tile_plain(TileSmem& sm, const ScanParams& p, int b, int d0,
                                                int64_t t0, int lane) {
  using Tr = VariantTraits<V>;
  const int t = lane & (kT - 1);
  const bool t_ok = t0 + t < p.seqlen;
#pragma unroll 4
  for (int i = 0; i < kRows / 2; ++i) {
    const int row = 2 * i + (lane >> 4);
    const bool ok = t_ok && (d0 + row < p.dim);
    const int64_t g = ((int64_t)b * p.dim + d0 + row) * p.seqlen + t0 + t;
    const int s = swz(row, t);
    sm.u[0][s] = ok ? __ldg(p.u + g) : 0.f;
    sm.dl[0][s] = ok ? __ldg(p.delta + g) : 0.f;
    if (Tr::fused && M == kEmit) sm.z[0][s] = ok ? __ldg(p.z + g) : 0.f;
  }
#pragma unroll
  for (int i = 0; i < (kT * kN) / 32; ++i) {
    const int flat = i * 32 + lane;
    const int tt = flat / kN;
    const bool ok = t0 + tt < p.seqlen;
    const int64_t g = ((int64_t)b * p.seqlen + t0 + tt) * kN + (flat % kN);
    sm.B[0][flat] = ok ? __ldg(p.B + g) : 0.f;
    if (M == kEmit) sm.C[0][flat] = ok ? __ldg(p.C + g) : 0.f;
  }
}

__device__ __forceinline__ void store_tile_plain(const float* os, const ScanParams& p, int b,
                                                 int d0, int64_t t0, int lane) {
  const int t = lane & (kT - 1);
  if (t0 + t >= p.seqlen) return;
#pragma unroll 4
  for (int i = 0; i < kRows / 2; ++i) {
    const int row = 2 * i + (lane >> 4);
    if (d0 + row < p.dim) {
      const int64_t g = ((int64_t)b * p.dim + d0 + row) * p.seqlen + t0 + t;
      p.out[g] = os[swz(row, t)];
    }
  }
}

// ------------------------------------------------------------------ kernel

#ifndef MAMBA_SCAN_MIN_BLOCKS
#define MAMBA_SCAN_MIN_BLOCKS 8
#endif

template <int V, int M, bool kTma>
__global__ void __launch_bounds__(kRows, MAMBA_SCAN_MIN_BLOCKS)
    scan_kernel(const ScanParams p, const __grid_constant__ TmaMaps maps) {
  using Tr = VariantTraits<V>;
  __shared__ TileSmem sm;

  const int lane = threadIdx.x;
  // Which row tile and which part of the sequence this CTA owns.
  int rt, chunk, n_chunks;
  if (M == kEmit && (int)blockIdx.x < p.n_full) {
    rt = blockIdx.x;  // whole sequence in one pass
    chunk = 0;
    n_chunks = 1;
  } else {
    const int j = (int)blockIdx.x - (M == kEmit ? p.n_full : 0);
    const int per = (M == kEmit) ? p.n_chunks : p.n_chunks - 1;
    rt = p.n_full + j / per;
    chunk = j % per;
    n_chunks = p.n_chunks;
  }
  const int64_t l_begin = (int64_t)chunk * p.chunk_len;
  const int64_t l_end = (chunk == n_chunks - 1) ? p.seqlen : l_begin + p.chunk_len;
  const int n_tiles = (int)((l_end - l_begin + kT - 1) / kT);
  const int b = rt / p.tiles_per_batch;
  const int d0 = (rt - b * p.tiles_per_batch) * kRows;

  const int d = d0 + lane;
  const bool row_ok = d < p.dim;
  const int64_t dc = row_ok ? d : p.dim - 1;  // clamped: parameter loads stay in bounds
  const int64_t row = (int64_t)b * p.dim + dc;
  // this lane's slot among the split rows' aggregates
  const int64_t ws_row = (int64_t)(rt - p.n_full) * kRows + lane;

  // Per-row constants: A (scaled by log2(e) for the exp2-based exact
  // variants), the D skip weight, the optional delta bias.
  float2 Ar[8];
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    float a0 = __ldg(p.A + dc * kN + 2 * n), a1 = __ldg(p.A + dc * kN + 2 * n + 1);
    if (Tr::exact) {
      a0 *= 1.4426950408889634f;
      a1 *= 1.4426950408889634f;
    }
    Ar[n] = make_float2(a0, a1);
  }
  const float dskip = __ldg(p.D + dc);
  const float bias = (Tr::fused && p.delta_bias != nullptr) ? __ldg(p.delta_bias + dc) : 0.f;
  const float bias_l2e = bias * 1.4426950408889634f;

  // Initial state: zeros (cc:241-242) or h0; emit chunks > 0 fold in the
  // aggregates of the chunks before them.
  float2 h[8], P[8];
  float S = 0.f;
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    h[n] = make_float2(0.f, 0.f);
    P[n] = make_float2(1.f, 1.f);
  }
  if (M == kEmit) {
    if (p.h0 != nullptr) {
#pragma unroll
      for (int n = 0; n < 8; ++n)
        h[n] = make_float2(__ldg(p.h0 + row * kN + 2 * n), __ldg(p.h0 + row * kN + 2 * n + 1));
    }
    if (chunk > 0) {
      const float* w = p.ws + ws_row * (int64_t)(n_chunks - 1) * 2 * kN;
      for (int cc = 0; cc < chunk; ++cc) {
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          const float2 he = make_float2(w[cc * 2 * kN + 2 * n], w[cc * 2 * kN + 2 * n + 1]);
          const float2 pe =
              make_float2(w[cc * 2 * kN + kN + 2 * n], w[cc * 2 * kN + kN + 2 * n + 1]);
          h[n] = fma2(pe, h[n], he);
        }
      }
    }
  }

  if (kTma) {
    // bytes landing per stage: full boxes, out-of-range elements included
    constexpr uint32_t kRowTile = kRows * kT * 4, kBCTile = kT * kN * 4;
    constexpr uint32_t kStageBytes = 2 * kRowTile + kBCTile +
                                     (M == kEmit ? kBCTile : 0) +
                                     ((Tr::fused && M == kEmit) ? kRowTile : 0);
    // The swizzled tiles assume 1 KiB-aligned arrays; refuse to issue any TMA
    // otherwise (the same decision in every lane).
    if ((smem_u32(&sm) & 1023u) != 0) {
      if (lane == 0) atomicExch(&g_scan_device_error, 5);
      return;
    }
    if (lane == 0) {
#pragma unroll
      for (int s = 0; s < kStages; ++s) mbar_init(&sm.full[s], 1);
      fence_mbarrier_init();
    }
    __syncwarp();
    auto issue = [&](int k, int s) {
      const int t0 = (int)(l_begin + (int64_t)k * kT);
      mbar_arrive_expect_tx(&sm.full[s], kStageBytes);
      tma_load_3d(sm.u[s], &maps.u, &sm.full[s], t0, d0, b);
      tma_load_3d(sm.dl[s], &maps.delta, &sm.full[s], t0, d0, b);
      if (Tr::fused && M == kEmit) tma_load_3d(sm.z[s], &maps.z, &sm.full[s], t0, d0, b);
      tma_load_3d(sm.B[s], &maps.B, &sm.full[s], 0, t0, b);
      if (M == kEmit) tma_load_3d(sm.C[s], &maps.C, &sm.full[s], 0, t0, b);
    };
    if (lane == 0) {
      for (int k = 0; k < kStages && k < n_tiles; ++k) issue(k, k);
    }
    for (int k = 0; k < n_tiles; ++k) {
      const int s = k % kStages;
      const bool ok = mbar_wait(&sm.full[s], (uint32_t)(k / kStages) & 1u, &g_scan_device_error);
      if (!__all_sync(0xffffffffu, ok)) {  // timeout recorded; all lanes leave together
        if (M == kEmit && lane == 0) bulk_wait_all<0>();  // no store may still read smem
        return;
      }
      const int64_t t0 = l_begin + (int64_t)k * kT;
      const int n_valid = (l_end - t0 < kT) ? (int)(l_end - t0) : kT;
      float* os = sm.u[s];  // outputs overwrite this tile's u
      if (n_valid == kT)
        compute_tile<V, M, false>(sm.u[s], sm.dl[s], sm.z[s], sm.B[s], sm.C[s], os, lane, h, P, S,
                                  Ar, dskip, bias, bias_l2e, n_valid);
      else
        compute_tile<V, M, true>(sm.u[s], sm.dl[s], sm.z[s], sm.B[s], sm.C[s], os, lane, h, P, S,
                                 Ar, dskip, bias, bias_l2e, n_valid);
      if (M == kEmit) {
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_3d(&maps.out, os, (int)t0, d0, b);
          bulk_commit();
          bulk_wait_read<1>();  // the store of tile k-1 has left its stage
        }
        __syncwarp();
        // refill the stage of tile k-1 with tile k-1+kStages
        if (lane == 0 && k >= 1 && k - 1 + kStages < n_tiles)
          issue(k - 1 + kStages, (k - 1) % kStages);
      } else {
        __syncwarp();
        if (lane == 0 && k + kStages < n_tiles) issue(k + kStages, s);
      }
    }
    if (M == kEmit && lane == 0) bulk_wait_all<0>();
  } else {
    for (int k = 0; k < n_tiles; ++k) {
      const int64_t t0 = l_begin + (int64_t)k * kT;
      load_tile_plain<V, M>(sm, p, b, d0, t0, lane);
      __syncwarp();
      const int n_valid = (l_end - t0 < kT) ? (int)(l_end - t0) : kT;
      float* os = sm.u[0];
      if (n_valid == kT)
        compute_tile<V, M, false>(sm.u[0], sm.dl[0], sm.z[0], sm.B[0], sm.C[0], os, lane,
                                  h, P, S, Ar, dskip, bias, bias_l2e, n_valid);
      else
        compute_tile<V, M, true>(sm.u[0], sm.dl[0], sm.z[0], sm.B[0], sm.C[0], os, lane,
                                 h, P, S, Ar, dskip, bias, bias_l2e, n_valid);
      __syncwarp();
      if (M == kEmit) store_tile_plain(os, p, b, d0, t0, lane);
      __syncwarp();
    }
  }

  if (!row_ok) return;
  if (M == kEmit) {
    if (p.h_last != nullptr && chunk == n_chunks - 1) {
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        p.h_last[row * kN + 2 * n] = h[n].x;
        p.h_last[row * kN + 2 * n + 1] = h[n].y;
      }
    }
  } else {
    float* w = p.ws + (ws_row * (int64_t)(n_chunks - 1) + chunk) * 2 * kN;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      float2 pn = P[n];
      if (Tr::exact) pn = make_float2(ex2_approx(Ar[n].x * S), ex2_approx(Ar[n].y * S));
      w[2 * n] = h[n].x;
      w[2 * n + 1] = h[n].y;
      w[kN + 2 * n] = pn.x;
      w[kN + 2 * n + 1] = pn.y;
    }
  }
}

// ------------------------------------------------------------------ launch

template <int V>
static cudaError_t launch_v(int mode, bool tma, const ScanParams& p, const TmaMaps& maps,
                            unsigned blocks, cudaStream_t st) {
  const dim3 grid(blocks);
  const dim3 block(kRows);
  if (mode == kLaunchEmit) {
    if (tma)
      scan_kernel<V, kEmit, true><<<grid, block, 0, st>>>(p, maps);
    else
      scan_kernel<V, kEmit, false><<<grid, block, 0, st>>>(p, maps);
  } else {
    if (tma)
      scan_kernel<V, kAggregate, true><<<grid, block, 0, st>>>(p, maps);
    else
      scan_kernel<V, kAggregate, false><<<grid, block, 0, st>>>(p, maps);
  }
  return cudaGetLastError();
}

cudaError_t launch_scan_kernel(int variant, int mode, bool tma, const ScanParams& p,
                               const TmaMaps& maps, unsigned grid, cudaStream_t stream) {
  switch (variant) {
    case kLinear: return launch_v<kLinear>(mode, tma, p, maps, grid, stream);
    case kExact: return launch_v<kExact>(mode, tma, p, maps, grid, stream);
    case kFused: return launch_v<kFused>(mode, tma, p, maps, grid, stream);
    case kFusedExact: return launch_v<kFusedExact>(mode, tma, p, maps, grid, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <int V>
static cudaError_t occupancy_v(int mode, bool tma, int* blocks) {
  if (mode == kLaunchEmit)
    return tma ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks, scan_kernel<V, kEmit, true>,
                                                               kRows, 0)
               : cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks, scan_kernel<V, kEmit, false>,
                                                               kRows, 0);
  return tma ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                   blocks, scan_kernel<V, kAggregate, true>, kRows, 0)
             : cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                   blocks, scan_kernel<V, kAggregate, false>, kRows, 0);
}

cudaError_t max_blocks_per_sm(int variant, int mode, bool tma, int* blocks) {
  switch (variant) {
    case kLinear: return occupancy_v<kLinear>(mode, tma, blocks);
    case kExact: return occupancy_v<kExact>(mode, tma, blocks);
    case kFused: return occupancy_v<kFused>(mode, tma, blocks);
    case kFusedExact: return occupancy_v<kFusedExact>(mode, tma, blocks);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t read_and_clear_device_error(int* code) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return e;
  int v = 0;
  e = cudaMemcpyFromSymbol(&v, g_scan_device_error, sizeof(int));
  if (e != cudaSuccess) return e;
  if (v != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_scan_device_error, &zero, sizeof(int));
  }
  *code = v;
  return e;
}

}  // namespace mamba_scan
