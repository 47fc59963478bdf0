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
//   are fetched by TMA into a 3-stage shared-memory ring (mbarrier
//   completion), read back as float4 through the 64-byte swizzle so the
//   per-row reads are bank-conflict free, and B/C values are warp-wide
//   broadcasts; outputs are written over the tile's u values and leave by a
//   TMA store, and the stage is refilled once that store has read it;
// * the per-state update runs on packed fp32x2 FMAs (FFMA2);
// * long sequences with few rows are split into chunks: an aggregate pass
//   computes, per (row, chunk), the chunk's end state from zero and its decay
//   prod(abar) (exp(A*sum(delta)) for the exact variants); a carry kernel
//   folds them in order into the state entering each chunk,
//   h_in = P*h_in + h_end; the emit pass re-runs each chunk from its h_in.
//   Carry and emit are programmatic dependent launches: the emit pass's
//   whole row tiles start while the aggregate pass still runs.
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
#define MAMBA_SCAN_ACC 1
#endif
// Independent partial sums per step in the C.h contraction (1, 2, 4 or 8).
// One chain measured best: the contraction of step t overlaps the state
// update of step t+1, and the single chain saves the FADD2 that joins two
// partial sums (SelectiveScanFused 1x1536x1024: 26.0 -> 25.2 us).
constexpr int kAcc = MAMBA_SCAN_ACC;

// --------------------------------------------------------------- tile math

#ifndef MAMBA_SCAN_POLY_EMIT
#define MAMBA_SCAN_POLY_EMIT 0
#endif
#ifndef MAMBA_SCAN_POLY_AGG
#define MAMBA_SCAN_POLY_AGG 1
#endif
// Exact variants: of the 8 state pairs of a step, this many take abar =
// 2^(delta*A*log2 e) from exp2_fma2 (FMA pipe), the rest from the SFU. The
// aggregate pass has FMA capacity to spare (no C.h contraction) and its 16
// SFU exponentials per step bound it, so one pair moves there (Exact
// 1x2048x16384: 312 -> 295 us); the emit pass is not SFU-bound and keeps all
// of them on the SFU.
template <int M, int E> struct PolyPairs {
  static constexpr int value =
      E != kExpSfu ? 0 : ((M == kEmit) ? MAMBA_SCAN_POLY_EMIT : MAMBA_SCAN_POLY_AGG);
};

#ifndef MAMBA_SCAN_WSCALE
#define MAMBA_SCAN_WSCALE 1
#endif

// Linear variants (SelectiveScan, SelectiveScanFused) run the recurrence on
// a rescaled state. With w_t = delta_t * u_t,
//
//   h_t = (1 + delta_t A) h_{t-1} + w_t B_t
//
// becomes, for g_t = h_t / w_t and r_t = w_{t-1} / w_t,
//
//   g_t = r_t (1 + delta_t A) g_{t-1} + B_t,   y_t = w_t (C_t . g_t) + D u_t,
//
// so B enters unscaled and the per-state multiply delta*u*B disappears: the
// state update costs abar' = fma(r*delta, A, r) and one FMA, three FP32
// operations per (row, step, state) with the contraction instead of four.
// w is kept away from zero: |w| < kWMin takes kWMin (the input term then
// differs from w*B by at most 2*kWMin*|B|). At the start of a pass w_{-1} = 1
// (g = h), and the state leaves as h = w_last * g. The padding steps of a
// ragged last tile (delta = 0, B = 0) keep w and g as they are.
//
// g = h / w has a smaller range than h: where |w| is tiny against |h| (a
// u = 0 step in a state that has grown past ~1e26) g overflows although the
// reference's h stays finite. An overflow cannot heal (inf times r*abar stays
// inf or turns NaN), so each pass checks its final state (and decay product)
// once: if any lane's is not finite, the warp runs the whole pass again on h
// itself, exactly the reference's form (abar = 1 + delta*A, input term
// delta*u*B, no division), and that result replaces the first one. The hot
// loop pays nothing for this; a pass that overflows pays a second, slower
// pass.
//
// The exact variants keep abar = exp(delta*A) and the product delta*u*B (a
// positive w is not guaranteed, so r cannot be folded into the exponent).
constexpr float kWMin = 1e-12f;

__device__ __forceinline__ float safe_w(float w) { return fabsf(w) < kWMin ? kWMin : w; }

template <int V> struct Scaled {
  static constexpr bool value = MAMBA_SCAN_WSCALE && !VariantTraits<V>::exact;
};

template <bool B> struct BoolTag {
  static constexpr bool value = B;
};

// True when all 16 values of a lane's state are finite (their sum is: an
// infinite or NaN element makes it so, and a sum that overflows only sends a
// finite state to the slower pass).
__device__ __forceinline__ bool finite16(const float2 (&x)[8]) {
  float2 s = add2(x[0], x[1]);
#pragma unroll
  for (int n = 2; n < 8; ++n) s = add2(s, x[n]);
  return isfinite(s.x + s.y);
}

// abar and the input term of one step, for the lane's 16 states.
// Exact variants: (x0, x1) = (delta, delta*u); a = exp(delta*A) formed as the
// exp mode E says, bu = delta*u*B.
// Linear variants, rescaled (kScaled): (x0, x1) = (r*delta, r),
// a = r*(1 + delta*A), bu = B; on h itself: (x0, x1) = (delta, delta*u),
// a = 1 + delta*A, bu = delta*u*B.
template <int V, int M, bool kScaled, int E>
__device__ __forceinline__ void step_prep(const float* __restrict__ Bt_, float x0_, float x1_,
                                          const float2 (&Ar)[8], float2 (&a)[8], float2 (&bu)[8]) {
  using Tr = VariantTraits<V>;
  const float2 one2 = make_float2(1.f, 1.f);
  const float2 dt2 = make_float2(x0_, x0_);
  const float2 du2 = make_float2(x1_, x1_);
  const float4* Bt = reinterpret_cast<const float4*>(Bt_);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 bq = Bt[q];
    if (Tr::exact && E == kExpSfu) {
      // abar = exp(delta*A) = 2^(delta * A*log2(e)); Ar holds A*log2(e)
      const float2 x0 = mul2(dt2, Ar[2 * q]);
      const float2 x1 = mul2(dt2, Ar[2 * q + 1]);
      a[2 * q] = (2 * q < PolyPairs<M, E>::value)
                     ? exp2_fma2(x0)
                     : make_float2(ex2_approx(x0.x), ex2_approx(x0.y));
      a[2 * q + 1] = (2 * q + 1 < PolyPairs<M, E>::value)
                         ? exp2_fma2(x1)
                         : make_float2(ex2_approx(x1.x), ex2_approx(x1.y));
    } else if (Tr::exact && E == kExpIeee) {
      const float2 x0 = mul2(dt2, Ar[2 * q]);  // Ar holds A
      const float2 x1 = mul2(dt2, Ar[2 * q + 1]);
      a[2 * q] = make_float2(expf(x0.x), expf(x0.y));
      a[2 * q + 1] = make_float2(expf(x1.x), expf(x1.y));
    } else if (Tr::exact) {
      // the reference's 8-lane exp (cc:265-268: delta*A, then fast_exp_avx2)
      const float2 x0 = mul2(dt2, Ar[2 * q]);
      const float2 x1 = mul2(dt2, Ar[2 * q + 1]);
      a[2 * q] = make_float2(reference_exp<false>(x0.x), reference_exp<false>(x0.y));
      a[2 * q + 1] = make_float2(reference_exp<false>(x1.x), reference_exp<false>(x1.y));
    } else if (kScaled) {
      // abar' = r*(1 + delta*A) = fma(r*delta, A, r)
      a[2 * q] = fma2(dt2, Ar[2 * q], du2);
      a[2 * q + 1] = fma2(dt2, Ar[2 * q + 1], du2);
    } else {
      // abar = 1 + delta*A (cc:275-282 written as (1+dA)h + dBu)
      a[2 * q] = fma2(dt2, Ar[2 * q], one2);
      a[2 * q + 1] = fma2(dt2, Ar[2 * q + 1], one2);
    }
    if (kScaled) {
      bu[2 * q] = make_float2(bq.x, bq.y);
      bu[2 * q + 1] = make_float2(bq.z, bq.w);
    } else {
      bu[2 * q] = mul2(du2, make_float2(bq.x, bq.y));
      bu[2 * q + 1] = mul2(du2, make_float2(bq.z, bq.w));
    }
  }
}

// sum_n C[n]*h[n] (cc:285-296) as two partial sums (x, y lanes of a pair).
__device__ __forceinline__ float2 contract(const float* __restrict__ Ct_, const float2 (&h)[8]) {
  const float4* Ct = reinterpret_cast<const float4*>(Ct_);
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
  return acc[0];
}

// Per-step scalar work of one 16-step tile for the calling lane's row, on
// packed pairs of consecutive steps (entry k holds steps 2k and 2k+1):
//   dt, du  (delta, delta*u); on the rescaled state of the linear variants
//           (r*delta, r) with r_t = w_{t-1} / w_t;
//   ww      w = delta*u kept away from zero (rescaled state);
//   dsk     D*u (rescaled state, emit); uu: u; gate: silu(z) (fused, emit).
// Softplus (fused variants) is applied to delta first; kPartial zeroes delta
// of the steps >= n_valid (the ragged last tile).
struct TileScalars {
  float2 uu[8], dt[8], du[8], gate[8], ww[8], dsk[8];
};

template <int V, int M, bool kPartial, int E, bool kScaled>
__device__ __forceinline__ void tile_scalars(const float* us, const float* __restrict__ ds,
                                             const float* __restrict__ zs, int row, float dskip,
                                             float bias, float bias_l2e, int n_valid,
                                             float& w_prev, TileScalars& ts) {
  using Tr = VariantTraits<V>;
  const float2 bias_l2e2 = make_float2(bias_l2e, bias_l2e);
  const float2 dskip2 = make_float2(dskip, dskip);
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int off = row * kT + (((c ^ (row >> 1)) & 3) << 2);
    const float4 u4 = *reinterpret_cast<const float4*>(us + off);
    const float4 d4 = *reinterpret_cast<const float4*>(ds + off);
    ts.uu[2 * c] = make_float2(u4.x, u4.y);
    ts.uu[2 * c + 1] = make_float2(u4.z, u4.w);
    ts.dt[2 * c] = make_float2(d4.x, d4.y);
    ts.dt[2 * c + 1] = make_float2(d4.z, d4.w);
    if (Tr::fused && E == kExpReference) {
      // the reference backend's softplus and SiLU (cc:137-148)
      ts.dt[2 * c] = make_float2(softplus_reference(d4.x + bias), softplus_reference(d4.y + bias));
      ts.dt[2 * c + 1] =
          make_float2(softplus_reference(d4.z + bias), softplus_reference(d4.w + bias));
      if (M == kEmit) {
        const float4 z4 = *reinterpret_cast<const float4*>(zs + off);
        ts.gate[2 * c] = make_float2(silu_reference(z4.x), silu_reference(z4.y));
        ts.gate[2 * c + 1] = make_float2(silu_reference(z4.z), silu_reference(z4.w));
      }
    } else if (Tr::fused) {
      ts.dt[2 * c] = softplus2<Tr::exact>(ts.dt[2 * c], bias, bias_l2e2);
      ts.dt[2 * c + 1] = softplus2<Tr::exact>(ts.dt[2 * c + 1], bias, bias_l2e2);
      if (M == kEmit) {
        const float4 z4 = *reinterpret_cast<const float4*>(zs + off);
        ts.gate[2 * c] = silu2<Tr::exact>(make_float2(z4.x, z4.y));
        ts.gate[2 * c + 1] = silu2<Tr::exact>(make_float2(z4.z, z4.w));
      }
    }
  }
  if (kPartial) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (2 * k >= n_valid) ts.dt[k].x = 0.f;
      if (2 * k + 1 >= n_valid) ts.dt[k].y = 0.f;
    }
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) ts.du[k] = mul2(ts.dt[k], ts.uu[k]);
  // Linear variants on the rescaled state: from here dt holds r*delta, du
  // holds r, and ww holds w = delta*u (kept away from zero). A padding step
  // gets w = w_{t-1}, r = 1 and r*delta = 0: abar' = 1 and its B is zero.
  if (kScaled) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      ts.ww[k] = make_float2(safe_w(ts.du[k].x), safe_w(ts.du[k].y));
      const float2 inv = make_float2(rcp_approx(ts.ww[k].x), rcp_approx(ts.ww[k].y));
      ts.du[k] = make_float2(w_prev * inv.x, ts.ww[k].x * inv.y);  // r = w_{t-1} / w_t
      if (kPartial) {
        if (2 * k >= n_valid) {
          ts.ww[k].x = w_prev;
          ts.du[k].x = 1.f;
        }
        if (2 * k + 1 >= n_valid) {
          ts.ww[k].y = ts.ww[k].x;
          ts.du[k].y = 1.f;
        }
      }
      w_prev = ts.ww[k].y;
      ts.dt[k] = mul2(ts.du[k], ts.dt[k]);
      if (M == kEmit) ts.dsk[k] = mul2(dskip2, ts.uu[k]);
    }
  }
}

// y of steps (2k, 2k+1) from their contractions (s0, s1) = (C.h of step 2k,
// C.h of step 2k+1): + D*u (cc:297), * silu(z) (cc:300-302); on the rescaled
// state y = w*(C.g) + D*u.
template <int V, bool kScaled>
__device__ __forceinline__ float2 step_pair_output(const TileScalars& ts, int k, float s0, float s1,
                                                   float dskip) {
  using Tr = VariantTraits<V>;
  float2 y = make_float2(s0, s1);
  if (kScaled)
    y = fma2(ts.ww[k], y, ts.dsk[k]);
  else
    y = fma2(make_float2(dskip, dskip), ts.uu[k], y);
  return Tr::fused ? mul2(y, ts.gate[k]) : y;
}

// One 16-step tile for the calling lane's row (row-per-lane layout: the lane
// keeps all 16 states of its row in h[0..7]). Reads the swizzled u/delta/z
// tiles and the B/C tiles, updates h (and the decay product P, or the delta
// sum S, in aggregate mode) and, in emit mode, writes y into the swizzled
// output tile `os` (which may be the u tile itself: every u value is read
// before the first output is written). kScaled: the linear variants'
// rescaled state (false: h itself).
//
// The per-step scalar work is done first for all 16 steps (tile_scalars).
// The state loop then computes abar and the input term of step t+1 before
// the C.h contraction of step t, so the contraction overlaps the next step's
// independent work.
template <int V, int M, bool kPartial, int E, bool kScaled>
__device__ __forceinline__ void compute_tile(const float* us,
                                             const float* __restrict__ ds,
                                             const float* __restrict__ zs,
                                             const float* __restrict__ Bs,
                                             const float* __restrict__ Cs, float* os,
                                             int row, float2 (&h)[8], float2 (&P)[8], float& S,
                                             const float2 (&Ar)[8], float dskip, float bias,
                                             float bias_l2e, int n_valid, float& w_prev) {
  using Tr = VariantTraits<V>;
  TileScalars ts;
  tile_scalars<V, M, kPartial, E, kScaled>(us, ds, zs, row, dskip, bias, bias_l2e, n_valid,
                                           w_prev, ts);
  float2 a[8], bu[8];
  step_prep<V, M, kScaled, E>(Bs, ts.dt[0].x, ts.du[0].x, Ar, a, bu);
  float2 s_prev = make_float2(0.f, 0.f);
  float2 yy[8];
#pragma unroll
  for (int t = 0; t < kT; ++t) {
#pragma unroll
    for (int n = 0; n < 8; ++n) h[n] = fma2(a[n], h[n], bu[n]);
    if (M == kAggregate) {
      // the chunk's decay: the product of the abar (linear variants, and the
      // reference exp, whose product is what the backend's recurrence
      // applies), else exp(A * sum(delta)) at the chunk's end
      if (!Tr::exact || E == kExpReference) {
#pragma unroll
        for (int n = 0; n < 8; ++n) P[n] = mul2(P[n], a[n]);
      } else {
        S += (t & 1) ? ts.dt[t >> 1].y : ts.dt[t >> 1].x;
      }
    }
    if (t + 1 < kT) {
      const int k = (t + 1) >> 1;
      step_prep<V, M, kScaled, E>(Bs + (t + 1) * kN, ((t + 1) & 1) ? ts.dt[k].y : ts.dt[k].x,
                                  ((t + 1) & 1) ? ts.du[k].y : ts.du[k].x, Ar, a, bu);
    }
    if (M == kEmit) {
      const float2 s = contract(Cs + t * kN, h);
      if (t & 1)
        yy[t >> 1] = step_pair_output<V, kScaled>(ts, t >> 1, s_prev.x + s_prev.y, s.x + s.y,
                                                   dskip);
      else
        s_prev = s;
    }
  }
  if (M == kEmit) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int off = row * kT + (((c ^ (row >> 1)) & 3) << 2);
      *reinterpret_cast<float4*>(os + off) =
          make_float4(yy[2 * c].x, yy[2 * c].y, yy[2 * c + 1].x, yy[2 * c + 1].y);
    }
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

// Which row tile and which part of the sequence a CTA owns.
struct CtaWork {
  int rt, chunk, n_chunks, n_tiles, b, d0;
  int64_t l_begin, l_end;
};

template <int M> __device__ __forceinline__ CtaWork cta_work(const ScanParams& p) {
  CtaWork w;
  if (M == kEmit && (int)blockIdx.x < p.n_full) {
    w.rt = blockIdx.x;  // whole sequence in one pass
    w.chunk = 0;
    w.n_chunks = 1;
  } else {
    const int j = (int)blockIdx.x - (M == kEmit ? p.n_full : 0);
    const int per = (M == kEmit) ? p.n_chunks : p.n_chunks - 1;
    w.rt = p.n_full + j / per;
    w.chunk = j % per;
    w.n_chunks = p.n_chunks;
  }
  w.l_begin = (int64_t)w.chunk * p.chunk_len;
  w.l_end = (w.chunk == w.n_chunks - 1) ? p.seqlen : w.l_begin + p.chunk_len;
  w.n_tiles = (int)((w.l_end - w.l_begin + kT - 1) / kT);
  w.b = w.rt / p.tiles_per_batch;
  w.d0 = (w.rt - w.b * p.tiles_per_batch) * kRows;
  return w;
}

// The calling lane's row and its constants: A (scaled by log2(e) for the
// exact variants' SFU exp2), the D skip weight, the optional delta bias.
struct RowConsts {
  float2 Ar[8];
  float dskip, bias, bias_l2e;
  int64_t row;     // b*dim + d (d clamped to the last row for padding lanes)
  int64_t ws_row;  // this lane's slot among the split rows' aggregates
  bool row_ok;     // d < dim
};

template <int V, int E>
__device__ __forceinline__ void row_consts(const ScanParams& p, const CtaWork& w, int lane,
                                           RowConsts& rc) {
  using Tr = VariantTraits<V>;
  const int d = w.d0 + lane;
  rc.row_ok = d < p.dim;
  const int64_t dc = rc.row_ok ? d : p.dim - 1;  // clamped: parameter loads stay in bounds
  rc.row = (int64_t)w.b * p.dim + dc;
  rc.ws_row = (int64_t)(w.rt - p.n_full) * kRows + lane;
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    float a0 = __ldg(p.A + dc * kN + 2 * n), a1 = __ldg(p.A + dc * kN + 2 * n + 1);
    if (Tr::exact && E == kExpSfu) {
      a0 *= 1.4426950408889634f;
      a1 *= 1.4426950408889634f;
    }
    rc.Ar[n] = make_float2(a0, a1);
  }
  rc.dskip = __ldg(p.D + dc);
  rc.bias = (Tr::fused && p.delta_bias != nullptr) ? __ldg(p.delta_bias + dc) : 0.f;
  rc.bias_l2e = rc.bias * 1.4426950408889634f;
}

// Initial state: zeros (cc:241-242) or h0; emit chunks > 0 start from the
// carry-in state of the chunks before them. w_prev = 1: g = h at the start.
template <int M>
__device__ __forceinline__ void init_state(const ScanParams& p, const CtaWork& w,
                                           const RowConsts& rc, float2 (&h)[8], float2 (&P)[8],
                                           float& S, float& w_prev) {
  S = 0.f;
  w_prev = 1.f;
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    h[n] = make_float2(0.f, 0.f);
    P[n] = make_float2(1.f, 1.f);
  }
  if (M == kEmit) {
    if (w.chunk > 0) {
      // The state entering this chunk, folded by carry_kernel (launched
      // between the two passes; wait for it and, through it, the aggregate
      // pass). Whole row tiles and first chunks do not wait.
      pdl_wait();
      const float4* ws = reinterpret_cast<const float4*>(
          p.ws + (rc.ws_row * (int64_t)(w.n_chunks - 1) + w.chunk - 1) * 2 * kN);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 e = __ldcg(ws + q);
        h[2 * q] = make_float2(e.x, e.y);
        h[2 * q + 1] = make_float2(e.z, e.w);
      }
    } else if (p.h0 != nullptr) {
#pragma unroll
      for (int n = 0; n < 8; ++n)
        h[n] = make_float2(__ldg(p.h0 + rc.row * kN + 2 * n),
                           __ldg(p.h0 + rc.row * kN + 2 * n + 1));
    }
  }
}

// One pass over a CTA's tiles with plain loads and stores (stage 0 of the
// ring). kScaled: the linear variants' rescaled state, or h itself.
// kOneForm: every tile through the ragged-tile code (less code for a pass
// that runs rarely).
template <int V, int M, int E, bool kScaled, bool kOneForm = false>
__device__ __forceinline__ void plain_pass(TileSmem& sm, const ScanParams& p, const CtaWork& w,
                                           int lane, const RowConsts& rc, float2 (&h)[8],
                                           float2 (&P)[8], float& S, float& w_prev) {
  for (int k = 0; k < w.n_tiles; ++k) {
    const int64_t t0 = w.l_begin + (int64_t)k * kT;
    load_tile_plain<V, M>(sm, p, w.b, w.d0, t0, lane);
    __syncwarp();
    const int n_valid = (w.l_end - t0 < kT) ? (int)(w.l_end - t0) : kT;
    float* os = sm.u[0];
    if (n_valid == kT && !kOneForm)
      compute_tile<V, M, false, E, kScaled>(sm.u[0], sm.dl[0], sm.z[0], sm.B[0], sm.C[0], os,
                                            lane, h, P, S, rc.Ar, rc.dskip, rc.bias, rc.bias_l2e,
                                            n_valid, w_prev);
    else
      compute_tile<V, M, true, E, kScaled>(sm.u[0], sm.dl[0], sm.z[0], sm.B[0], sm.C[0], os,
                                           lane, h, P, S, rc.Ar, rc.dskip, rc.bias, rc.bias_l2e,
                                           n_valid, w_prev);
    __syncwarp();
    if (M == kEmit) store_tile_plain(os, p, w.b, w.d0, t0, lane);
    __syncwarp();
  }
}

// End of a pass: the state back to h (and, for the aggregates, prod(abar));
// the final state to h_last (emit, last chunk) or the chunk's end state and
// decay to the workspace (aggregate).
template <int V, int M, int E>
__device__ __forceinline__ void finish_pass(const ScanParams& p, const CtaWork& w,
                                            const RowConsts& rc, float2 (&h)[8], float2 (&P)[8],
                                            float S, float w_prev) {
  using Tr = VariantTraits<V>;
  if (!rc.row_ok) return;
  if (Scaled<V>::value) {
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      h[n] = mul2(h[n], make_float2(w_prev, w_prev));
      P[n] = mul2(P[n], make_float2(w_prev, w_prev));
    }
  }
  if (M == kEmit) {
    if (p.h_last != nullptr && w.chunk == w.n_chunks - 1) {
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        p.h_last[rc.row * kN + 2 * n] = h[n].x;
        p.h_last[rc.row * kN + 2 * n + 1] = h[n].y;
      }
    }
  } else {
    // 32 floats per (row, chunk): the end state, then the decay.
    float4* ws = reinterpret_cast<float4*>(
        p.ws + (rc.ws_row * (int64_t)(w.n_chunks - 1) + w.chunk) * 2 * kN);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float2 p0 = P[2 * q], p1 = P[2 * q + 1];
      if (Tr::exact && E == kExpSfu) {
        p0 = make_float2(ex2_approx(rc.Ar[2 * q].x * S), ex2_approx(rc.Ar[2 * q].y * S));
        p1 = make_float2(ex2_approx(rc.Ar[2 * q + 1].x * S),
                         ex2_approx(rc.Ar[2 * q + 1].y * S));
      } else if (Tr::exact && E == kExpIeee) {
        p0 = make_float2(expf(rc.Ar[2 * q].x * S), expf(rc.Ar[2 * q].y * S));
        p1 = make_float2(expf(rc.Ar[2 * q + 1].x * S), expf(rc.Ar[2 * q + 1].y * S));
      }
      ws[q] = make_float4(h[2 * q].x, h[2 * q].y, h[2 * q + 1].x, h[2 * q + 1].y);
      ws[4 + q] = make_float4(p0.x, p0.y, p1.x, p1.y);
    }
  }
}

// The CTA's whole pass again, on h itself (the reference's form), for a warp
// whose rescaled state overflowed; writes every output of the pass again and
// finishes it. (Kept inline: an out-of-line call made the hot loop slower.)
template <int V, int M, int E>
__device__ __forceinline__ void rerun_on_h(const ScanParams& p, TileSmem& sm, int lane) {
  const CtaWork w = cta_work<M>(p);
  RowConsts rc;
  row_consts<V, E>(p, w, lane, rc);
  float2 h[8], P[8];
  float S, w_prev;
  init_state<M>(p, w, rc, h, P, S, w_prev);
  plain_pass<V, M, E, false, true>(sm, p, w, lane, rc, h, P, S, w_prev);
  finish_pass<V, M, E>(p, w, rc, h, P, S, 1.f);
}

template <int V, int M, bool kTma, int E>
__global__ void __launch_bounds__(kRows, MAMBA_SCAN_MIN_BLOCKS)
    scan_kernel(const __grid_constant__ ScanParams p, const __grid_constant__ TmaMaps maps) {
  using Tr = VariantTraits<V>;
  constexpr bool kScaled = Scaled<V>::value;
  __shared__ TileSmem sm;
  // The carry kernel (launched next, programmatic dependent launch) may be
  // scheduled right away; it waits for this grid to finish before reading.
  if (M == kAggregate) pdl_trigger();

  const int lane = threadIdx.x;
  const CtaWork w = cta_work<M>(p);
  RowConsts rc;
  row_consts<V, E>(p, w, lane, rc);
  float2 h[8], P[8];
  float S, w_prev;  // w_prev: linear variants run the state as g = h / w
  init_state<M>(p, w, rc, h, P, S, w_prev);
  const int b = w.b, d0 = w.d0;
  const int64_t l_begin = w.l_begin, l_end = w.l_end;
  const int n_tiles = w.n_tiles;

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
    int issued = 0;  // tiles whose loads lane 0 has issued
    auto issue = [&](int k, int s) {
      ++issued;
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
        if (lane == 0) {
          // Before the CTA's shared memory can go to another CTA: give the
          // loads already issued for later tiles up to 100 ms each to land
          // (a lost one never will; its wait gives up too), and let no
          // store still read shared memory.
          for (int j = k + 1; j < issued; ++j)
            mbar_wait(&sm.full[j % kStages], (uint32_t)(j / kStages) & 1u, &g_scan_device_error,
                      100000000ull);
          if (M == kEmit) bulk_wait_all<0>();
        }
        __syncwarp();
        return;
      }
      const int64_t t0 = l_begin + (int64_t)k * kT;
      const int n_valid = (l_end - t0 < kT) ? (int)(l_end - t0) : kT;
      float* os = sm.u[s];  // outputs overwrite this tile's u
      if (n_valid == kT)
        compute_tile<V, M, false, E, kScaled>(sm.u[s], sm.dl[s], sm.z[s], sm.B[s], sm.C[s], os,
                                              lane, h, P, S, rc.Ar, rc.dskip, rc.bias,
                                              rc.bias_l2e, n_valid, w_prev);
      else
        compute_tile<V, M, true, E, kScaled>(sm.u[s], sm.dl[s], sm.z[s], sm.B[s], sm.C[s], os,
                                             lane, h, P, S, rc.Ar, rc.dskip, rc.bias,
                                             rc.bias_l2e, n_valid, w_prev);
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
    plain_pass<V, M, E, kScaled>(sm, p, w, lane, rc, h, P, S, w_prev);
  }

  // The rescaled state overflows only where the reference's h is large and
  // |delta*u| tiny (see Scaled): then this warp's whole pass runs again on h.
  if (kScaled) {
    const bool bad = rc.row_ok && !(finite16(h) && (M == kEmit || finite16(P)));
    if (__any_sync(0xffffffffu, bad)) {
      if (kTma && M == kEmit) {
        // the first pass's TMA stores are complete (waited for above): order
        // them before the second pass's stores of the same outputs
        if (lane == 0) fence_proxy_async();
        __syncwarp();
      }
      rerun_on_h<V, M, E>(p, sm, lane);
      return;
    }
  }
  finish_pass<V, M, E>(p, w, rc, h, P, S, w_prev);
}

// ------------------------------------------------------------ carry kernel

// Turns the chunk aggregates of the split row tiles into the states entering
// each chunk: h_in(0) = h0 (or 0) and h_in(c) = P(c-1) * h_in(c-1) +
// h_end(c-1), folded over the chunks in order. One thread per (row, state);
// h_in(c) overwrites h_end(c-1) in the workspace, where the emit pass of
// chunk c reads it. Launched after the aggregate pass as a programmatic
// dependent launch: it lets the emit pass be scheduled at once, then waits
// for the aggregate pass.
template <int kAhead>  // chunks whose loads are in flight together
__global__ void __launch_bounds__(kCarryThreads) carry_kernel(const ScanParams p) {
  pdl_trigger();
  const int64_t gid = (int64_t)blockIdx.x * kCarryThreads + threadIdx.x;
  const int s = (int)(gid % kN);
  const int64_t ws_row = gid / kN;
  if (ws_row >= (int64_t)p.n_tail * kRows) return;
  const int rt = p.n_full + (int)(ws_row / kRows);
  const int b = rt / p.tiles_per_batch;
  const int64_t d = (int64_t)(rt - b * p.tiles_per_batch) * kRows + ws_row % kRows;
  if (d >= p.dim) return;  // padding rows of the last tile: nothing to carry
  float h = (p.h0 != nullptr) ? __ldg(p.h0 + ((int64_t)b * p.dim + d) * kN + s) : 0.f;
  pdl_wait();
  const int n = p.n_chunks - 1;
  float* w = p.ws + ws_row * (int64_t)n * 2 * kN + s;
  for (int c = 0; c < n; c += kAhead) {
    float he[kAhead], pe[kAhead];
#pragma unroll
    for (int f = 0; f < kAhead; ++f) {
      he[f] = 0.f;
      pe[f] = 1.f;
      if (c + f < n) {
        he[f] = __ldcg(w + (c + f) * 2 * kN);
        pe[f] = __ldcg(w + (c + f) * 2 * kN + kN);
      }
    }
#pragma unroll
    for (int f = 0; f < kAhead; ++f) {
      if (c + f < n) {
        h = fmaf(pe[f], h, he[f]);
        w[(c + f) * 2 * kN] = h;
      }
    }
  }
}

// ------------------------------------------------------- wait self-test

// Exercises the bounded wait's give-up path without any fault: one arrival
// announces 16 bytes of transaction that no copy will ever deliver, so the
// phase cannot complete; mbar_wait gives up after limit_ns and records
// MAMBA_SCAN_ERR_DEVICE_TIMEOUT. No asynchronous copy is issued, so nothing
// is in flight when the CTA exits.
__global__ void __launch_bounds__(32) wait_selftest_kernel(uint64_t limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbarrier_init();
  }
  __syncwarp();
  if (threadIdx.x == 0) mbar_arrive_expect_tx(&bar, 16);
  __syncwarp();
  mbar_wait(&bar, 0, &g_scan_device_error, limit_ns);
}

cudaError_t launch_wait_selftest(uint64_t limit_ns, cudaStream_t stream) {
  wait_selftest_kernel<<<1, 32, 0, stream>>>(limit_ns);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ launch

// Launch `kernel` on `st`; with `pdl` as a programmatic dependent launch (the
// grid may start before the previous kernel in the stream has finished; it
// orders itself with griddepcontrol.wait).
template <typename... Args>
static cudaError_t launch(void (*kernel)(Args...), unsigned blocks, unsigned threads,
                          cudaStream_t st, bool pdl, const Args&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

template <int V, int E>
static cudaError_t launch_ve(int mode, bool tma, const ScanParams& p, const TmaMaps& maps,
                             unsigned blocks, cudaStream_t st, bool pdl) {
  if (mode == kLaunchEmit)
    return tma ? launch(scan_kernel<V, kEmit, true, E>, blocks, kRows, st, pdl, p, maps)
               : launch(scan_kernel<V, kEmit, false, E>, blocks, kRows, st, pdl, p, maps);
  return tma ? launch(scan_kernel<V, kAggregate, true, E>, blocks, kRows, st, pdl, p, maps)
             : launch(scan_kernel<V, kAggregate, false, E>, blocks, kRows, st, pdl, p, maps);
}

template <int V>
static cudaError_t launch_v(int mode, bool tma, int exp_mode, const ScanParams& p,
                            const TmaMaps& maps, unsigned blocks, cudaStream_t st, bool pdl) {
  if constexpr (!VariantTraits<V>::exact) {
    return launch_ve<V, kExpSfu>(mode, tma, p, maps, blocks, st, pdl);
  } else {
    if (exp_mode == kExpIeee) return launch_ve<V, kExpIeee>(mode, tma, p, maps, blocks, st, pdl);
    if (exp_mode == kExpReference)
      return launch_ve<V, kExpReference>(mode, tma, p, maps, blocks, st, pdl);
    return launch_ve<V, kExpSfu>(mode, tma, p, maps, blocks, st, pdl);
  }
}

cudaError_t launch_scan_kernel(int variant, int exp_mode, int mode, bool tma,
                               const ScanParams& p, const TmaMaps& maps, unsigned grid,
                               cudaStream_t stream, bool pdl) {
  switch (variant) {
    case kLinear: return launch_v<kLinear>(mode, tma, exp_mode, p, maps, grid, stream, pdl);
    case kExact: return launch_v<kExact>(mode, tma, exp_mode, p, maps, grid, stream, pdl);
    case kFused: return launch_v<kFused>(mode, tma, exp_mode, p, maps, grid, stream, pdl);
    case kFusedExact:
      return launch_v<kFusedExact>(mode, tma, exp_mode, p, maps, grid, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_carry_kernel(const ScanParams& p, cudaStream_t stream) {
  const int64_t threads = (int64_t)p.n_tail * kRows * kN;
  const unsigned blocks = (unsigned)((threads + kCarryThreads - 1) / kCarryThreads);
  // Up to 8 chunk aggregates per row: a small kernel (its CTAs wait resident
  // beside the emit pass's whole row tiles, so they must stay light); more:
  // 32 in flight, one load round trip for up to 33 chunks.
  if (p.n_chunks - 1 <= 8) return launch(carry_kernel<8>, blocks, kCarryThreads, stream, true, p);
  return launch(carry_kernel<32>, blocks, kCarryThreads, stream, true, p);
}

template <int V, int E>
static cudaError_t occupancy_ve(int mode, bool tma, int* blocks) {
  if (mode == kLaunchEmit)
    return tma ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                     blocks, scan_kernel<V, kEmit, true, E>, kRows, 0)
               : cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                     blocks, scan_kernel<V, kEmit, false, E>, kRows, 0);
  return tma ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                   blocks, scan_kernel<V, kAggregate, true, E>, kRows, 0)
             : cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                   blocks, scan_kernel<V, kAggregate, false, E>, kRows, 0);
}

template <int V>
static cudaError_t occupancy_v(int mode, bool tma, int exp_mode, int* blocks) {
  if constexpr (!VariantTraits<V>::exact) {
    return occupancy_ve<V, kExpSfu>(mode, tma, blocks);
  } else {
    if (exp_mode == kExpIeee) return occupancy_ve<V, kExpIeee>(mode, tma, blocks);
    if (exp_mode == kExpReference) return occupancy_ve<V, kExpReference>(mode, tma, blocks);
    return occupancy_ve<V, kExpSfu>(mode, tma, blocks);
  }
}

cudaError_t max_blocks_per_sm(int variant, int exp_mode, int mode, bool tma, int* blocks) {
  switch (variant) {
    case kLinear: return occupancy_v<kLinear>(mode, tma, exp_mode, blocks);
    case kExact: return occupancy_v<kExact>(mode, tma, exp_mode, blocks);
    case kFused: return occupancy_v<kFused>(mode, tma, exp_mode, blocks);
    case kFusedExact: return occupancy_v<kFusedExact>(mode, tma, exp_mode, blocks);
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
