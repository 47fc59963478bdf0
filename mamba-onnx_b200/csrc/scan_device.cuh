// Device-side building blocks of the selective-scan kernels (sm_100a).
//
// PTX wrappers for mbarriers, TMA tensor copies and bulk-group waits, the
// per-element math of the four reference variants, and the shared-memory tile
// layout. The kernels themselves are in scan_kernels.cu.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mamba_scan {

constexpr int kN = 16;     // d_state; the reference kernels support only 16 (cc:228-230)
constexpr int kRows = 32;  // (b, d) rows per CTA: one warp, one row per lane
constexpr int kT = 16;     // time steps per tile: 64-byte rows in shared memory
constexpr int kStages = 3;  // tiles in the shared-memory ring
constexpr int kCarryThreads = 256;  // threads per CTA of the carry kernel
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // a tile wait gives up after 2 s

enum Variant { kLinear = 0, kExact = 1, kFused = 2, kFusedExact = 3 };

// How the Exact variants form exp (abar = exp(delta*A), the chunk decay, and
// in reference mode the exps inside softplus and SiLU):
//   kExpSfu       2^(x*log2 e) on the SFU (ex2.approx), softplus/SiLU with
//                 CUDA's expf/log1pf;
//   kExpIeee      CUDA's expf everywhere;
//   kExpReference the reference C++ backend's own exp, its published Taylor-5
//                 plus 2^n method, in softplus and SiLU too, so the output
//                 follows that backend's (float64-inexact) numbers.
enum ExpMode { kExpSfu = 0, kExpIeee = 1, kExpReference = 2 };
enum Mode { kEmit = 0, kAggregate = 1 };

template <int V> struct VariantTraits {
  static constexpr bool fused = (V == kFused || V == kFusedExact);
  static constexpr bool exact = (V == kExact || V == kFusedExact);
};

// ---------------------------------------------------------------- PTX wrappers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's generic-proxy shared-memory accesses against later
// async-proxy (TMA) accesses.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Orders this thread's async-proxy (TMA) accesses, in every state space,
// against its later generic-proxy accesses.
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n"
      "  .reg .pred p;\n"
      "  mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "  selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait on an mbarrier phase. Gives up after limit_ns of wall time
// (2 s for the scan kernels), records MAMBA_SCAN_ERR_DEVICE_TIMEOUT (6) in
// *err and returns false, so a lost transaction can never hang the GPU.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err,
                                          uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = globaltimer_ns();
  // the iteration cap backs up the clock check (each try_wait already
  // suspends for a while before it fails)
  for (uint32_t spins = 0; spins < (1u << 26); ++spins) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((spins & 255u) == 255u && globaltimer_ns() - start > limit_ns) break;
  }
  atomicExch(err, 6);  // MAMBA_SCAN_ERR_DEVICE_TIMEOUT
  return false;
}

// 3-D tiled TMA load into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// 3-D tiled TMA store from shared memory (out-of-range elements are clipped).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int c0,
                                             int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until at most N committed bulk groups still read shared memory.
template <int N> __device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Wait until at most N committed bulk groups are still in flight.
template <int N> __device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// Programmatic dependent launch: let the next grid in the stream be
// scheduled now (it still orders itself with pdl_wait) ...
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ... and wait until the previous grid in the stream has finished and its
// writes are visible (returns at once when this grid was launched normally).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ------------------------------------------------------------------ the math

// 2^x on the SFU (PTX ex2.approx.ftz.f32).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32x2 arithmetic (sm_100 FFMA2/FMUL2).
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }

// 2^x for a pair, on the FMA pipe instead of the SFU: x = j + f with j =
// round(x) (adding 1.5*2^23 rounds to an integer in the low mantissa bits)
// and f in [-1/2, 1/2]; 2^f by a degree-6 polynomial (relative-error
// near-minimax fit on [-1/2, 1/2], coefficients fitted for this code; max
// relative error 7.9e-8 in float32 Horner form, under one ulp); then j is
// added to the exponent field. x is clamped to [-125, 127] so the result is
// always a normal float: 2^x below 2^-125 comes out as ~2^-125 instead of
// 0 (an absolute difference under 3e-38), above 2^127 as 2^127.
__device__ __forceinline__ float2 exp2_fma2(float2 x) {
  x = make_float2(fminf(fmaxf(x.x, -125.f), 127.f), fminf(fmaxf(x.y, -125.f), 127.f));
  const float2 t = add2(x, make_float2(12582912.f, 12582912.f));
  const float2 j = add2(t, make_float2(-12582912.f, -12582912.f));
  const float2 f = fma2(j, make_float2(-1.f, -1.f), x);  // x - j, exact
  float2 p = make_float2(1.534580806037411e-4f, 1.534580806037411e-4f);
  p = fma2(p, f, make_float2(1.3399930903688073e-3f, 1.3399930903688073e-3f));
  p = fma2(p, f, make_float2(9.618489071726799e-3f, 9.618489071726799e-3f));
  p = fma2(p, f, make_float2(5.550328642129898e-2f, 5.550328642129898e-2f));
  p = fma2(p, f, make_float2(0.24022646248340607f, 0.24022646248340607f));
  p = fma2(p, f, make_float2(0.6931471824645996f, 0.6931471824645996f));
  p = fma2(p, f, make_float2(1.f, 1.f));
  // bits(t) = bits(1.5*2^23) + j, and bits(1.5*2^23) << 23 wraps to 0
  return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23)));
}

__device__ __forceinline__ float lg2_approx(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// exp(x) as the reference C++ backend computes it (selective_scan.cc:33-69,
// method published in docs/optimization_notes.md:60-100): x clamped to
// +-88.3762626647949, n = floor(x * 1.44269504089), f = x - n*ln2 in [0, ln2),
// e^f by the degree-5 Taylor polynomial 1 + f + f^2/2 + ... + f^5/120 in Horner
// form with FMAs, times 2^n formed as the bit pattern (n + 127) << 23. Every
// step is a correctly rounded fp32 operation, so the result equals the
// backend's bit for bit (denormal inputs aside: the backend runs with FTZ/DAZ).
// For n = -128 (x below about -88.03) that pattern is the one of -inf, and the
// backend's exp returns -inf there; so does this one.
// kFmaReduction: f as one FMA (the backend's scalar copies, which its compiler
// contracts) or as a multiply and a subtract (its 8-lane copy in the scan loop).
template <bool kFmaReduction> __device__ __forceinline__ float reference_exp(float x) {
  x = fmaxf(fminf(x, 88.3762626647949f), -88.3762626647949f);
  const float t = __fmul_rn(x, 1.44269504089f);
  const float tf = floorf(t);
  const float f = kFmaReduction ? __fmaf_rn(-tf, 0.6931471805599453f, x)
                                : __fsub_rn(x, __fmul_rn(tf, 0.6931471805599453f));
  float p = __fmaf_rn(0.008333333333f, f, 0.041666666666f);
  p = __fmaf_rn(p, f, 0.166666666666f);
  p = __fmaf_rn(p, f, 0.5f);
  p = __fmaf_rn(p, f, 1.0f);
  p = __fmaf_rn(p, f, 1.0f);
  const unsigned bits = static_cast<unsigned>(static_cast<int>(tf) + 127) << 23;
  return __fmul_rn(p, __uint_as_float(bits));
}

// softplus(x + bias) = log(1 + e^(x+bias)).
// Exact variants: IEEE expf/log1pf with the reference's branches
// (cc:137-143: x > 20 -> x, x < -20 -> e^x).
// Approximate variants: SFU 2^x and log2 on s = (x + bias) * log2(e), formed
// by one FMA with bias_l2e = bias * log2(e); s > 20*log2(e) returns x + bias.
// Below x = -20 this gives log(1 + e^x) rounded in fp32 (0 once e^x < 2^-24)
// instead of e^x: an absolute difference under 2.1e-9.
template <bool kExactMath>
__device__ __forceinline__ float softplus(float x, float bias, float bias_l2e) {
  if (kExactMath) {
    // Both candidates are computed and one is selected (no divergent
    // branches, so the steps of a tile can be interleaved); for x > 88.7,
    // e = inf and l = inf are computed but not selected.
    x += bias;
    const float e = expf(x);
    const float l = log1pf(e);
    return x > 20.f ? x : (x < -20.f ? e : l);
  } else {
    const float s = fmaf(x, 1.4426950408889634f, bias_l2e);
    const float l = lg2_approx(1.f + ex2_approx(s));
    return (s > 28.853900817779268f ? s : l) * 0.6931471805599453f;
  }
}

// silu(x) = x / (1 + e^-x) (cc:145-148); approximate variants use the SFU
// 2^x and reciprocal.
template <bool kExactMath> __device__ __forceinline__ float silu(float x) {
  if (kExactMath) return x / (1.f + expf(-x));
  return x * rcp_approx(1.f + ex2_approx(x * -1.4426950408889634f));
}

// The reference backend's softplus and SiLU (cc:137-148): its own exp (the
// scalar, FMA-reduced copy), then log1pf, or 1 + e and an IEEE division.
__device__ __forceinline__ float softplus_reference(float x) {
  const float e = reference_exp<true>(x);
  const float l = log1pf(e);
  return x > 20.f ? x : (x < -20.f ? e : l);
}
__device__ __forceinline__ float silu_reference(float x) {
  return __fdiv_rn(x, __fadd_rn(1.f, reference_exp<true>(-x)));
}

// Two consecutive steps at once: the FMA/add/multiply parts of softplus and
// silu run as packed fp32x2 operations (each lane of the pair rounds exactly
// like the scalar forms above); the SFU calls stay scalar.
template <bool kExactMath>
__device__ __forceinline__ float2 softplus2(float2 x, float bias, float2 bias_l2e) {
  if (kExactMath) return make_float2(softplus<true>(x.x, bias, 0.f), softplus<true>(x.y, bias, 0.f));
  const float2 s = fma2(x, make_float2(1.4426950408889634f, 1.4426950408889634f), bias_l2e);
  float2 l = add2(make_float2(1.f, 1.f), make_float2(ex2_approx(s.x), ex2_approx(s.y)));
  l = make_float2(s.x > 28.853900817779268f ? s.x : lg2_approx(l.x),
                  s.y > 28.853900817779268f ? s.y : lg2_approx(l.y));
  return mul2(l, make_float2(0.6931471805599453f, 0.6931471805599453f));
}

template <bool kExactMath> __device__ __forceinline__ float2 silu2(float2 x) {
  if (kExactMath) return make_float2(silu<true>(x.x), silu<true>(x.y));
  const float2 t = mul2(x, make_float2(-1.4426950408889634f, -1.4426950408889634f));
  const float2 d = add2(make_float2(1.f, 1.f), make_float2(ex2_approx(t.x), ex2_approx(t.y)));
  return mul2(x, make_float2(rcp_approx(d.x), rcp_approx(d.y)));
}

// Offset (in floats) of element (row, t) of a [kRows][kT] tile stored with the
// TMA 64-byte swizzle: 16-byte chunk index t/4 XOR bits 7..8 of the row's byte
// offset (64*row), i.e. (row >> 1) & 3.
__device__ __forceinline__ int swz(int row, int t) {
  return row * kT + ((((t >> 2) ^ (row >> 1)) & 3) << 2) + (t & 3);
}

// Shared memory of one CTA: a ring of kStages tiles. The outputs of a tile
// are written over its u tile, which the TMA store then reads; the stage is
// refilled one tile later, once that store has left shared memory. Every
// array starts on a 1 KiB boundary so the swizzle is anchored at its start.
struct __align__(1024) TileSmem {
  float u[kStages][kRows * kT];
  float dl[kStages][kRows * kT];
  float z[kStages][kRows * kT];
  float B[kStages][kT * kN];
  float C[kStages][kT * kN];
  uint64_t full[kStages];
};

}  // namespace mamba_scan
