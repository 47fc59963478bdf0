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

// --------------------------------------------------------------- tile math

// One 16-step tile for the calling lane's row. Reads the swizzled u/delta/z
// tiles and the B/C tiles, updates h (and the decay product P, or the delta
// sum S, in aggregate mode) and, in emit mode, writes y into the swizzled
// output tile. kPartial masks steps >= n_valid (the ragged last tile).
template <int V, int M, bool kPartial>
__device__ __forceinline__ void compute_tile(const float* __restrict__ us,
                                             const float* __restrict__ ds,
                                             const float* __restrict__ zs,
                                             const float* __restrict__ Bs,
                                             const float* __restrict__ Cs, float* __restrict__ os,
                                             int row, float2 (&h)[8], float2 (&P)[8], float& S,
                                             const float2 (&Ar)[8], float dskip, float bias,
                                             int n_valid) {
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
      for (int j = 0; j < 4; ++j) dd[j] = softplus<Tr::exact>(dd[j] + bias);
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
      float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 bq = Bt[q];
        float2 a0, a1;
        if (Tr::exact) {
          // abar = exp(delta*A) = 2^(delta * A*log2(e)); Ar holds A*log2(e)
          const float2 x0 = mul2(dt2, Ar[2 * q]);
          const float2 x1 = mul2(dt2, Ar[2 * q + 1]);
          a0 = make_float2(ex2_approx(x0.x), ex2_approx(x0.y));
          a1 = make_float2(ex2_approx(x1.x), ex2_approx(x1.y));
        } else {
          // abar = 1 + delta*A (cc:275-282 in the form (1+dA)h + dBu)
          a0 = fma2(dt2, Ar[2 * q], one2);
          a1 = fma2(dt2, Ar[2 * q + 1], one2);
        }
        h[2 * q] = fma2(a0, h[2 * q], mul2(du2, make_float2(bq.x, bq.y)));
        h[2 * q + 1] = fma2(a1, h[2 * q + 1], mul2(du2, make_float2(bq.z, bq.w)));
        if (M == kAggregate) {
          if (!Tr::exact) {
            P[2 * q] = mul2(P[2 * q], a0);
            P[2 * q + 1] = mul2(P[2 * q + 1], a1);
          }
        } else {
          const float4 cq = Ct[q];
          acc0 = fma2(make_float2(cq.x, cq.y), h[2 * q], acc0);
          acc1 = fma2(make_float2(cq.z, cq.w), h[2 * q + 1], acc1);
        }
      }
      if (M == kAggregate) {
        if (Tr::exact) S += dt;
        yy[j] = 0.f;
      } else {
        float y = (acc0.x + acc1.x) + (acc0.y + acc1.y);
        y = fmaf(dskip, uu[j], y);  // + D*u (cc:297)
        yy[j] = Tr::fused ? y * gate[j] : y;  // * silu(z) (cc:300-302)
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

template <int V, int M, bool kTma>
__global__ void __launch_bounds__(kRows, 8)
    scan_kernel(const ScanParams p, const __grid_constant__ TmaMaps maps) {
  using Tr = VariantTraits<V>;
  __shared__ TileSmem sm;

  const int lane = threadIdx.x;
  const int b = blockIdx.x / p.tiles_per_batch;
  const int d0 = (blockIdx.x - b * p.tiles_per_batch) * kRows;
  const int chunk = blockIdx.y;
  const int64_t l_begin = (int64_t)chunk * p.chunk_len;
  const int64_t l_end = (chunk == p.n_chunks - 1) ? p.seqlen : l_begin + p.chunk_len;
  const int n_tiles = (int)((l_end - l_begin + kT - 1) / kT);

  const int d = d0 + lane;
  const bool row_ok = d < p.dim;
  const int64_t dc = row_ok ? d : p.dim - 1;  // clamped: parameter loads stay in bounds
  const int64_t row = (int64_t)b * p.dim + dc;

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
      const float* w = p.ws + row * (int64_t)(p.n_chunks - 1) * 2 * kN;
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
    if (lane == 0) {
      if ((smem_u32(&sm) & 1023u) != 0) atomicExch(&g_scan_device_error, 5);
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
      if (!__all_sync(0xffffffffu, ok)) return;  // timeout recorded; all lanes leave together
      if (M == kEmit) {
        if (lane == 0) bulk_wait_read<1>();  // the store of tile k-2 has left out[k&1]
        __syncwarp();
      }
      const int64_t t0 = l_begin + (int64_t)k * kT;
      const int n_valid = (l_end - t0 < kT) ? (int)(l_end - t0) : kT;
      float* os = sm.out[k & 1];
      if (n_valid == kT)
        compute_tile<V, M, false>(sm.u[s], sm.dl[s], sm.z[s], sm.B[s], sm.C[s], os, lane, h, P, S,
                                  Ar, dskip, bias, n_valid);
      else
        compute_tile<V, M, true>(sm.u[s], sm.dl[s], sm.z[s], sm.B[s], sm.C[s], os, lane, h, P, S,
                                 Ar, dskip, bias, n_valid);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        if (M == kEmit) {
          tma_store_3d(&maps.out, os, (int)t0, d0, b);
          bulk_commit();
        }
        if (k + kStages < n_tiles) issue(k + kStages, s);
      }
    }
    if (M == kEmit && lane == 0) bulk_wait_all<0>();
  } else {
    for (int k = 0; k < n_tiles; ++k) {
      const int64_t t0 = l_begin + (int64_t)k * kT;
      load_tile_plain<V, M>(sm, p, b, d0, t0, lane);
      __syncwarp();
      const int n_valid = (l_end - t0 < kT) ? (int)(l_end - t0) : kT;
      if (n_valid == kT)
        compute_tile<V, M, false>(sm.u[0], sm.dl[0], sm.z[0], sm.B[0], sm.C[0], sm.out[0], lane,
                                  h, P, S, Ar, dskip, bias, n_valid);
      else
        compute_tile<V, M, true>(sm.u[0], sm.dl[0], sm.z[0], sm.B[0], sm.C[0], sm.out[0], lane,
                                 h, P, S, Ar, dskip, bias, n_valid);
      __syncwarp();
      if (M == kEmit) store_tile_plain(sm.out[0], p, b, d0, t0, lane);
      __syncwarp();
    }
  }

  if (!row_ok) return;
  if (M == kEmit) {
    if (p.h_last != nullptr && chunk == p.n_chunks - 1) {
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        p.h_last[row * kN + 2 * n] = h[n].x;
        p.h_last[row * kN + 2 * n + 1] = h[n].y;
      }
    }
  } else {
    float* w = p.ws + (row * (int64_t)(p.n_chunks - 1) + chunk) * 2 * kN;
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
                            dim3 grid, cudaStream_t st) {
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
                               const TmaMaps& maps, dim3 grid, cudaStream_t stream) {
  switch (variant) {
    case kLinear: return launch_v<kLinear>(mode, tma, p, maps, grid, stream);
    case kExact: return launch_v<kExact>(mode, tma, p, maps, grid, stream);
    case kFused: return launch_v<kFused>(mode, tma, p, maps, grid, stream);
    case kFusedExact: return launch_v<kFusedExact>(mode, tma, p, maps, grid, stream);
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
