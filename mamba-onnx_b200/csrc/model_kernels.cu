// Kernels of the Mamba block around the selective-scan op (sm_100a).
//
// The reference ships only the scan op; the block that feeds it (its dataflow
// is benchmarks/profiler.py:18-150 of acmiyaguchi/mamba-onnx) is the caller's.
// mamba_onnx/model.py is that caller, and these two kernels replace the
// chains of small torch kernels it would otherwise launch per block:
//
// * RMSNorm over the model dimension, y = x * rsqrt(mean(x^2) + eps) * w:
//   one warp per row, float4 loads, shuffle reduction;
// * the causal depthwise convolution over the sequence followed by SiLU,
//   y[b,d,t] = silu(bias[d] + sum_k w[d,k] * x[b,d,t-(K-1)+k]) with zeros
//   before t = 0 (torch's conv1d with padding K-1, sliced to the first L
//   outputs): one thread per four consecutive steps of one channel.
//
// * x_proj, [dt | B | C][t] = W_x x[:, t], for every token: a thread-block
//   cluster of 8 CTAs per 32 tokens, each CTA summing 1/8 of d_inner (in
//   96-row steps) into a 32 x P partial tile in shared memory (4 tokens x
//   P/32 outputs per thread in registers), then each CTA adds 4 token rows
//   of all 8 partials in cluster-rank order through distributed shared
//   memory (deterministic, no
//   global scratch) and writes them straight into the three outputs the scan
//   takes (dt [L][rank], B and C [L][dstate] contiguous);
//
// The first two are memory-bound (two HBM passes over their tensor); x_proj
// replaces a cuBLAS fp32 GEMM that its skinny shape leaves at a few CTAs,
// plus the copies of the B and C slices out of its output. The C entry
// points are declared in include/mamba_model_ops.h.
#include <cooperative_groups.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <string>

#include "../../include/mamba_model_ops.h"
#include "../../include/mamba_scan.h"
#include "scan_device.cuh"
#include "scan_kernels.h"

namespace cg = cooperative_groups;

namespace {

using mamba_scan::launch_pdl;

// Every kernel here is launched as a programmatic dependent launch: it lets
// the next kernel be scheduled at once, then waits for the previous one
// before its first global access.
__device__ __forceinline__ void pdl_enter() {
  mamba_scan::pdl_trigger();
  mamba_scan::pdl_wait();
}

constexpr int kNormWarps = 8;        // rows per CTA of the RMSNorm kernel
constexpr int kConvThreads = 256;    // threads per CTA of the convolution kernel
constexpr int kConvMaxWidth = 8;     // widest convolution supported

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// tf32(v) rounded to nearest (ties away), as mamba_split_tf32 forms its hi
// part; the lo part is tf32(v - hi).
__device__ __forceinline__ float round_tf32(float v) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
  return __uint_as_float(r);
}

// Stores four normalised values of a row: y itself, or (kSplit) its tf32
// parts hi = tf32(y), lo = tf32(y - hi), the operand form of the tensor-core
// GEMM (mamba_split_tf32's output for the same y).
template <bool kSplit>
__device__ __forceinline__ void store_norm4(float* y, float* hi, float* lo, const float4 v) {
  if (!kSplit) {
    *reinterpret_cast<float4*>(y) = v;
    return;
  }
  const float4 h = make_float4(round_tf32(v.x), round_tf32(v.y), round_tf32(v.z), round_tf32(v.w));
  *reinterpret_cast<float4*>(hi) = h;
  *reinterpret_cast<float4*>(lo) = make_float4(round_tf32(v.x - h.x), round_tf32(v.y - h.y),
                                               round_tf32(v.z - h.z), round_tf32(v.w - h.w));
}

// kVec: rows of cols % 4 == 0 floats with 16-byte aligned bases.
// kSplit: y is not written; hi and lo (rows of ld floats, ld % 4 == 0)
// receive the tf32 parts of each normalised value (kVec only).
template <bool kVec, bool kSplit = false>
__global__ void __launch_bounds__(kNormWarps * 32)
    rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                   float* __restrict__ y, int64_t rows, int cols, float eps,
                   float* __restrict__ hi = nullptr, float* __restrict__ lo = nullptr,
                   int64_t ld = 0) {
  static_assert(kVec || !kSplit, "the split form stores float4s");
  pdl_enter();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * kNormWarps + warp;
  if (r >= rows) return;
  const float* xr = x + r * cols;
  float* yr = kSplit ? nullptr : y + r * cols;
  float* hr = kSplit ? hi + r * ld : nullptr;
  float* lr = kSplit ? lo + r * ld : nullptr;
  float ss = 0.f;
  if (kVec) {
    for (int c = lane * 4; c < cols; c += 128) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(xr + c));
      ss = fmaf(v.x, v.x, ss);
      ss = fmaf(v.y, v.y, ss);
      ss = fmaf(v.z, v.z, ss);
      ss = fmaf(v.w, v.w, ss);
    }
  } else {
    for (int c = lane; c < cols; c += 32) ss = fmaf(xr[c], xr[c], ss);
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / (float)cols + eps);
  if (kVec) {
    for (int c = lane * 4; c < cols; c += 128) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(xr + c));
      const float4 g = __ldg(reinterpret_cast<const float4*>(w + c));
      store_norm4<kSplit>(yr + c, hr + c, lr + c,
                          make_float4(v.x * inv * g.x, v.y * inv * g.y, v.z * inv * g.z,
                                      v.w * inv * g.w));
    }
  } else {
    for (int c = lane; c < cols; c += 32) yr[c] = xr[c] * inv * w[c];
  }
}

__device__ __forceinline__ float silu_exact(float v) { return v / (1.f + expf(-v)); }

// One thread: steps [t0, t0+4) of row (b, d); its width+3 inputs are read
// through the read-only cache (neighbouring threads share most of them).
// kVec: seqlen % 4 == 0 and 16-byte aligned rows (one float4 store).
template <bool kVec>
__global__ void __launch_bounds__(kConvThreads)
    conv_silu_kernel(const float* __restrict__ x, int64_t x_bstride,
                     const float* __restrict__ w, const float* __restrict__ bias,
                     float* __restrict__ y, int64_t dim, int64_t seqlen, int64_t blocks_per_row,
                     int64_t n_items, int width) {
  pdl_enter();
  const int64_t i = (int64_t)blockIdx.x * kConvThreads + threadIdx.x;
  if (i >= n_items) return;
  const int64_t row = i / blocks_per_row;  // b * dim + d
  const int64_t t0 = (i - row * blocks_per_row) * 4;
  const int64_t b = row / dim, d = row - b * dim;
  const float* xr = x + b * x_bstride + d * seqlen;
  float* yr = y + row * seqlen;
  // inputs t0-(width-1) .. t0+3; window[j] = x[t0 - (width-1) + j], 0 before t = 0
  float win[kConvMaxWidth + 3];
  const int64_t base = t0 - (width - 1);
#pragma unroll
  for (int j = 0; j < kConvMaxWidth + 3; ++j) {
    const int64_t t = base + j;
    win[j] = (j < width + 3 && t >= 0 && t < seqlen) ? __ldg(xr + t) : 0.f;
  }
  float wk[kConvMaxWidth];
#pragma unroll
  for (int k = 0; k < kConvMaxWidth; ++k) wk[k] = k < width ? __ldg(w + d * width + k) : 0.f;
  const float bd = bias ? __ldg(bias + d) : 0.f;
  float o[4];
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    float acc = bd;
#pragma unroll
    for (int k = 0; k < kConvMaxWidth; ++k)
      if (k < width) acc = fmaf(wk[k], win[s + k], acc);
    o[s] = silu_exact(acc);
  }
  if (kVec) {
    *reinterpret_cast<float4*>(yr + t0) = make_float4(o[0], o[1], o[2], o[3]);
  } else {
#pragma unroll
    for (int s = 0; s < 4; ++s)
      if (t0 + s < seqlen) yr[t0 + s] = o[s];
  }
}

// The same for the width-4 convolution of Mamba models on 16-byte aligned
// rows with seqlen % 4 == 0: CTA (row, blockIdx.y) covers 1024 steps of one
// (b, d) row, each thread reading its inputs as two float4s (steps t0-4.. and
// t0..) and the row's 4 weights as one; the same sums in the same order.
__global__ void __launch_bounds__(kConvThreads)
    conv4_silu_kernel(const float* __restrict__ x, int64_t x_bstride,
                      const float* __restrict__ w, const float* __restrict__ bias,
                      float* __restrict__ y, unsigned dim, int64_t seqlen) {
  pdl_enter();
  const int64_t t0 = ((int64_t)blockIdx.y * kConvThreads + threadIdx.x) * 4;
  if (t0 >= seqlen) return;
  const unsigned row = blockIdx.x, b = row / dim, d = row - b * dim;  // row = b * dim + d
  const float* xr = x + (int64_t)b * x_bstride + (int64_t)d * seqlen;
  const float4 cur = __ldg(reinterpret_cast<const float4*>(xr + t0));
  const float4 prev = t0 > 0 ? __ldg(reinterpret_cast<const float4*>(xr + t0 - 4))
                             : make_float4(0.f, 0.f, 0.f, 0.f);
  const float win[7] = {prev.y, prev.z, prev.w, cur.x, cur.y, cur.z, cur.w};  // t0-3 .. t0+3
  const float4 w4 = __ldg(reinterpret_cast<const float4*>(w + (int64_t)d * 4));
  const float wk[4] = {w4.x, w4.y, w4.z, w4.w};
  const float bd = bias ? __ldg(bias + d) : 0.f;
  float o[4];
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    float acc = bd;
#pragma unroll
    for (int k = 0; k < 4; ++k) acc = fmaf(wk[k], win[s + k], acc);
    o[s] = silu_exact(acc);
  }
  *reinterpret_cast<float4*>(y + (int64_t)row * seqlen + t0) = make_float4(o[0], o[1], o[2], o[3]);
}

// ------------------------------------------------------ convolution step

// One decoding step of the causal convolution, one thread per (b, d): the
// window state[b, d, :] (oldest first) shifts by one and takes the new input,
// y[b, d] = silu(bias[d] + sum_k w[d, k] * state[b, d, k]).
__global__ void __launch_bounds__(kConvThreads)
    conv_step_kernel(float* __restrict__ state, const float* __restrict__ x, int64_t x_bstride,
                     const float* __restrict__ w, const float* __restrict__ bias,
                     float* __restrict__ y, int64_t batch, int64_t dim, int width) {
  pdl_enter();
  const int64_t i = (int64_t)blockIdx.x * kConvThreads + threadIdx.x;
  if (i >= batch * dim) return;
  const int64_t b = i / dim, d = i - b * dim;
  float* st = state + i * width;
  float acc = bias ? __ldg(bias + d) : 0.f;
  float prev = __ldg(x + b * x_bstride + d);  // the newest input goes last
#pragma unroll
  for (int k = kConvMaxWidth - 1; k >= 0; --k) {
    if (k >= width) continue;
    const float cur = st[k];
    st[k] = prev;
    acc = fmaf(__ldg(w + d * width + k), prev, acc);
    prev = cur;
  }
  y[i] = silu_exact(acc);
}

// ---------------------------------------------------- RMSNorm + GEMV step

constexpr int kNgThreads = 256;  // 8 warps, one output row each per pass
constexpr int kNgMaxCols = 4096;

// out[b, j] = weight[j] . (x[b] * rsqrt(mean(x[b]^2) + eps) * norm_w), for
// a few tokens (decoding): every CTA normalises its token's row into shared
// memory (cols <= 4096), then each warp takes output rows j with float4
// loads of weight[j] and a fixed shuffle tree (deterministic).
__global__ void __launch_bounds__(kNgThreads)
    norm_gemv_kernel(const float* __restrict__ x, const float* __restrict__ norm_w,
                     const float* __restrict__ weight, float* __restrict__ out, int cols,
                     int rows_out, float eps) {
  pdl_enter();
  __shared__ __align__(16) float xn[kNgMaxCols];
  __shared__ float red[kNgThreads / 32];
  const int b = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* xr = x + (int64_t)b * cols;
  float ss = 0.f;
  for (int c = threadIdx.x; c < cols; c += kNgThreads) {
    const float v = __ldg(xr + c);
    xn[c] = v;
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kNgThreads / 32; ++w) tot += red[w];
  const float inv = rsqrtf(tot / (float)cols + eps);
  for (int c = threadIdx.x; c < cols; c += kNgThreads) xn[c] = xn[c] * inv * __ldg(norm_w + c);
  __syncthreads();
  const int j = blockIdx.x * (kNgThreads / 32) + warp;
  if (j >= rows_out) return;
  const float* wr = weight + (int64_t)j * cols;
  float acc = 0.f;
  for (int c = lane * 4; c < cols; c += 128) {
    const float4 wv = __ldg(reinterpret_cast<const float4*>(wr + c));
    const float4 xv = *reinterpret_cast<const float4*>(&xn[c]);
    acc = fmaf(wv.x, xv.x, acc);
    acc = fmaf(wv.y, xv.y, acc);
    acc = fmaf(wv.z, xv.z, acc);
    acc = fmaf(wv.w, xv.w, acc);
  }
  acc = warp_sum(acc);
  if (lane == 0) out[(int64_t)b * rows_out + j] = acc;
}

// out[b, j] = (residual[b, j] +) weight[j] . x[b], for a few tokens: each
// CTA stages its token's x in shared memory, each warp takes output rows j
// (float4 loads of weight[j], a fixed shuffle tree: deterministic).
// residual may be out itself (the residual stream updated in place), so
// neither is declared __restrict__: each output element's residual is read by
// the lane that then writes it.
__global__ void __launch_bounds__(kNgThreads)
    gemv_kernel(const float* __restrict__ x, const float* __restrict__ weight,
                const float* residual, float* out, int cols, int rows_out) {
  pdl_enter();
  __shared__ __align__(16) float xs[kNgMaxCols];
  const int b = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int c = threadIdx.x; c < cols; c += kNgThreads) xs[c] = __ldg(x + (int64_t)b * cols + c);
  __syncthreads();
  const int j = blockIdx.x * (kNgThreads / 32) + warp;
  if (j >= rows_out) return;
  const float* wr = weight + (int64_t)j * cols;
  float acc = 0.f;
  for (int c = lane * 4; c < cols; c += 128) {
    const float4 wv = __ldg(reinterpret_cast<const float4*>(wr + c));
    const float4 xv = *reinterpret_cast<const float4*>(&xs[c]);
    acc = fmaf(wv.x, xv.x, acc);
    acc = fmaf(wv.y, xv.y, acc);
    acc = fmaf(wv.z, xv.z, acc);
    acc = fmaf(wv.w, xv.w, acc);
  }
  acc = warp_sum(acc);
  if (lane == 0) {
    const int64_t o = (int64_t)b * rows_out + j;
    out[o] = residual ? residual[o] + acc : acc;
  }
}

// ------------------------------------------------------- SSM decode step

constexpr int kSsmThreads = 128;  // channels per CTA
constexpr int kSsmMaxRank = 256;
constexpr int kSsmN = 16;         // d_state (as the scan op)

// One decoding step of a SelectiveScanFusedExact block for channel (b, d),
// with dt_proj fused in front and the state updated in place:
//   delta = softplus(W_dt[d] . dt[b] + bias[d])   (the op's branches: > 20 -> x,
//                                                  < -20 -> e^x, else log1p(e^x))
//   h[n]  = exp(delta A[d,n]) h[n] + delta u B[b,n]
//   y     = (sum_n C[b,n] h[n] + D[d] u) * silu(z)
// dt, B and C of the CTA's batch entry are staged in shared memory.
__global__ void __launch_bounds__(kSsmThreads)
    ssm_step_kernel(const float* __restrict__ u, const float* __restrict__ z, int64_t z_bstride,
                    const float* __restrict__ dt, const float* __restrict__ Bm,
                    const float* __restrict__ Cm, const float* __restrict__ w_dt,
                    const float* __restrict__ dt_bias, const float* __restrict__ A,
                    const float* __restrict__ Dskip, float* __restrict__ state,
                    float* __restrict__ y, int dim, int rank) {
  pdl_enter();
  __shared__ float sdt[kSsmMaxRank];
  __shared__ float sB[kSsmN], sC[kSsmN];
  const int b = blockIdx.y;
  for (int r = threadIdx.x; r < rank; r += kSsmThreads) sdt[r] = __ldg(dt + (int64_t)b * rank + r);
  if (threadIdx.x < kSsmN) {
    sB[threadIdx.x] = __ldg(Bm + b * kSsmN + threadIdx.x);
    sC[threadIdx.x] = __ldg(Cm + b * kSsmN + threadIdx.x);
  }
  __syncthreads();
  const int d = blockIdx.x * kSsmThreads + threadIdx.x;
  if (d >= dim) return;
  const float* wr = w_dt + (int64_t)d * rank;
  // W_dt[d] . dt: float4 loads of the row (all in flight), four partial sums
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  int r = 0;
  if ((rank & 3) == 0 && (reinterpret_cast<uintptr_t>(w_dt) & 15u) == 0) {
    const float4* w4 = reinterpret_cast<const float4*>(wr);
#pragma unroll 4
    for (int q = 0; q < rank / 4; ++q) {
      const float4 wv = __ldg(w4 + q);
      a0 = fmaf(wv.x, sdt[4 * q], a0);
      a1 = fmaf(wv.y, sdt[4 * q + 1], a1);
      a2 = fmaf(wv.z, sdt[4 * q + 2], a2);
      a3 = fmaf(wv.w, sdt[4 * q + 3], a3);
    }
    r = rank;
  }
  for (; r < rank; ++r) a0 = fmaf(__ldg(wr + r), sdt[r], a0);
  const float xd = (dt_bias ? __ldg(dt_bias + d) : 0.f) + ((a0 + a1) + (a2 + a3));
  const float e = expf(xd);
  const float delta = xd > 20.f ? xd : (xd < -20.f ? e : log1pf(e));
  const int64_t row = (int64_t)b * dim + d;
  const float uv = __ldg(u + row);
  const float du = delta * uv;
  float* h = state + row * kSsmN;
  const float* a = A + (int64_t)d * kSsmN;
  float acc = 0.f;
#pragma unroll
  for (int n = 0; n < kSsmN; ++n) {
    const float hn = fmaf(expf(delta * __ldg(a + n)), h[n], du * sB[n]);
    h[n] = hn;
    acc = fmaf(sC[n], hn, acc);
  }
  const float zv = __ldg(z + (int64_t)b * z_bstride + d);
  y[row] = fmaf(__ldg(Dskip + d), uv, acc) * (zv / (1.f + expf(-zv)));
}

// ------------------------------------------------------------------ x_proj

constexpr int kXpCluster = 8;    // CTAs per token block, each 1/8 of d_inner
constexpr int kXpTokens = 32;    // tokens per block: 8 groups of 4
constexpr int kXpThreads = 256;  // 8 token groups x 32 groups of 4 outputs
constexpr int kXpDChunk = 96;    // d_inner rows staged per step (2 steps at d_inner 1536)
constexpr int kXpMaxOut = 128;   // rank + 2 * dstate
constexpr int kXpRow = kXpMaxOut + 1;  // padded rows of the partial tile
// Row stride of the staged weights: 16-byte aligned rows for the float4
// reads, and 132 = 4 (mod 32) so the float4 stores of 32 consecutive rows
// spread over all banks.
constexpr int kXpWRow = kXpMaxOut + 4;

struct XpStage {
  float x[kXpDChunk][kXpTokens];  // x[d][t] of the chunk
  float w[kXpDChunk][kXpWRow];    // W_x[j][d], transposed to [d][j]
};
union XpSmem {
  XpStage stage;
  float part[kXpTokens][kXpRow];  // this CTA's partial sums, [t][j]
};
// x_proj with dt_proj fused (kDelta): up to this dt_rank. After the partial
// sums are added, the union holds dt of the cluster's 32 tokens as [k][t]
// (row stride 33) and then a chunk of dt_proj's weight as [k][96 d].
constexpr int kXpDtMaxRank = 96;
constexpr int kXpDtRow = kXpTokens + 1;
static_assert(kXpDtMaxRank * (kXpDtRow + kXpDChunk) * 4 <= sizeof(XpSmem), "fused dt_proj smem");
// ... plus, outside the union, this CTA's 4 finished token rows of dt, [k][4]
constexpr size_t kXpDtlBytes = (size_t)kXpMaxOut * (kXpTokens / kXpCluster) * 4;
constexpr size_t kXpSmemBytes = sizeof(XpSmem) + kXpDtlBytes;

// Thread (og, tg) = (tid / 8, tid % 8) sums outputs 4 og .. 4 og + 3 of
// tokens 4 tg .. 4 tg + 3 over its CTA's d_inner range: per d one float4 of
// x and one of W, and 8 packed FMAs over token pairs (each output's sum runs
// over d in order, as a scalar loop would). Warps whose outputs all lie past
// P (rank + 2 * dstate) only stage.
// kDelta: dt_proj fused, delta[b, d, t] = sum_k w_dt[d, k] dt[b, t, k]
// written instead of dt (rank <= kXpDtMaxRank): each CTA of the cluster
// forms delta for its own d_inner range and the cluster's 32 tokens.
template <bool kDelta>
__global__ void __cluster_dims__(kXpCluster, 1, 1) __launch_bounds__(kXpThreads, 2)
    xproj_kernel(const float* __restrict__ x, const float* __restrict__ w, float* __restrict__ dt,
                 float* __restrict__ Bm, float* __restrict__ Cm, int dim, int seqlen, int rank,
                 int dstate, const float* __restrict__ w_dt, float* __restrict__ delta) {
  pdl_enter();
  extern __shared__ __align__(16) uint8_t xp_raw[];
  XpSmem& sm = *reinterpret_cast<XpSmem*>(xp_raw);
  float* dtl = reinterpret_cast<float*>(xp_raw + sizeof(XpSmem));  // kDelta: [k][4]
  cg::cluster_group cluster = cg::this_cluster();
  const int crank = (int)cluster.block_rank();
  const int b = blockIdx.y;
  const int t0 = (blockIdx.x / kXpCluster) * kXpTokens;
  const int P = rank + 2 * dstate;
  const int per = (dim + kXpCluster - 1) / kXpCluster;
  const int d_lo = min(dim, crank * per), d_hi = min(dim, d_lo + per);
  const float* xb = x + (int64_t)b * dim * seqlen;
  const int tid = threadIdx.x, tg = tid & 7, og = tid >> 3;
  const bool computes = 4 * (og & ~3) < P;  // warp-uniform: the warp's 16 outputs start below P

  float2 acc[2][4];  // [token pair][output]: .x token 4 tg + 2 p, .y the next
#pragma unroll
  for (int p2 = 0; p2 < 2; ++p2)
#pragma unroll
    for (int o = 0; o < 4; ++o) acc[p2][o] = make_float2(0.f, 0.f);

  // Loads of a 96-row chunk go to registers first, all issued before any is
  // stored (x: 12 per thread, rows of 32 tokens; W: 12 x 4 per thread, four
  // outputs of one d_inner row, zeros past P): one load round trip per chunk.
  constexpr int kXq = kXpDChunk * kXpTokens / kXpThreads;         // 12
  constexpr int kWq = kXpDChunk * (kXpMaxOut / 4) / kXpThreads;   // 12
  float xr[kXq];
  float4 wr[kWq];
  auto fetch = [&](int dc) {
#pragma unroll
    for (int q = 0; q < kXq; ++q) {
      const int d = dc + (tid >> 5) + 8 * q, t = t0 + (tid & 31);
      xr[q] = (d < d_hi && t < seqlen) ? __ldg(xb + (int64_t)d * seqlen + t) : 0.f;
    }
#pragma unroll
    for (int q = 0; q < kWq; ++q) {
      const int i = tid + kXpThreads * q, j = 4 * (i / kXpDChunk), d = dc + i % kXpDChunk;
      const bool dok = d < d_hi;
      const float* wc = w + (int64_t)j * dim + d;
      wr[q] = make_float4((dok && j < P) ? __ldg(wc) : 0.f,
                          (dok && j + 1 < P) ? __ldg(wc + dim) : 0.f,
                          (dok && j + 2 < P) ? __ldg(wc + 2 * dim) : 0.f,
                          (dok && j + 3 < P) ? __ldg(wc + 3 * dim) : 0.f);
    }
  };
  for (int dc = d_lo; dc < d_hi; dc += kXpDChunk) {
    fetch(dc);
    __syncthreads();  // the previous chunk has been read
#pragma unroll
    for (int q = 0; q < kXq; ++q) sm.stage.x[(tid >> 5) + 8 * q][tid & 31] = xr[q];
#pragma unroll
    for (int q = 0; q < kWq; ++q) {
      const int i = tid + kXpThreads * q;
      *reinterpret_cast<float4*>(&sm.stage.w[i % kXpDChunk][4 * (i / kXpDChunk)]) = wr[q];
    }
    __syncthreads();
    const int n = min(kXpDChunk, d_hi - dc);
    if (computes) {
#pragma unroll 4
      for (int dd = 0; dd < n; ++dd) {
        const float4 xv = *reinterpret_cast<const float4*>(&sm.stage.x[dd][4 * tg]);
        const float4 wv = *reinterpret_cast<const float4*>(&sm.stage.w[dd][4 * og]);
        const float2 x01 = make_float2(xv.x, xv.y), x23 = make_float2(xv.z, xv.w);
        const float wo[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int o = 0; o < 4; ++o) {
          const float2 w2 = make_float2(wo[o], wo[o]);
          acc[0][o] = mamba_scan::fma2(x01, w2, acc[0][o]);
          acc[1][o] = mamba_scan::fma2(x23, w2, acc[1][o]);
        }
      }
    }
  }
  __syncthreads();  // the staging area becomes the partial tile
#pragma unroll
  for (int p2 = 0; p2 < 2; ++p2)
#pragma unroll
    for (int o = 0; o < 4; ++o) {
      sm.part[4 * tg + 2 * p2][4 * og + o] = acc[p2][o].x;
      sm.part[4 * tg + 2 * p2 + 1][4 * og + o] = acc[p2][o].y;
    }
  cluster.sync();  // every CTA's partial tile is complete and visible
  // this CTA completes token rows [4 crank, 4 crank + 4): the 8 partials
  // added in rank order
  constexpr int kRows = kXpTokens / kXpCluster;
  const float* parts[kXpCluster];  // every CTA's partial tile, mapped once
#pragma unroll
  for (int r = 0; r < kXpCluster; ++r) parts[r] = cluster.map_shared_rank(&sm.part[0][0], r);
  for (int i = tid; i < kRows * P; i += kXpThreads) {
    const int tt = crank * kRows + i / P, j = i % P;
    float sum = 0.f;
#pragma unroll
    for (int r = 0; r < kXpCluster; ++r) sum += parts[r][tt * kXpRow + j];
    const int t = t0 + tt;
    if (kDelta && j < rank) dtl[j * kRows + (tt - crank * kRows)] = sum;
    if (t < seqlen) {
      const int64_t row = (int64_t)b * seqlen + t;
      if (j < rank) {
        if (!kDelta) dt[row * rank + j] = sum;
      } else if (j < rank + dstate) {
        Bm[row * dstate + (j - rank)] = sum;
      } else {
        Cm[row * dstate + (j - rank - dstate)] = sum;
      }
    }
  }
  if constexpr (kDelta) {
    // every CTA's 4 rows of dt are final, and no CTA reads the partial tiles
    // any more: the union is free
    cluster.sync();
    float* dtf = &sm.part[0][0];                 // dt of the 32 tokens, [k][t]
    float* wdt = dtf + kXpDtMaxRank * kXpDtRow;  // w_dt of 96 d_inner rows, [k][d]
    for (int i = tid; i < kXpTokens * rank; i += kXpThreads) {
      const int k = i / kXpTokens, tt = i % kXpTokens;
      const float* src = cluster.map_shared_rank(dtl, tt / kRows);
      dtf[k * kXpDtRow + tt] = src[k * kRows + tt % kRows];
    }
    const int warp = tid >> 5, lane = tid & 31;  // lane = token, warp = 12 rows of the chunk
    constexpr int kWq = kXpDtMaxRank * kXpDChunk / kXpThreads;  // 36 loads per thread
    for (int dc = d_lo; dc < d_hi; dc += kXpDChunk) {
      float r[kWq];
#pragma unroll
      for (int q = 0; q < kWq; ++q) {
        const int i = tid + kXpThreads * q, dd = i % kXpDChunk, k = i / kXpDChunk;
        r[q] = (k < rank && dc + dd < d_hi) ? __ldg(w_dt + (int64_t)(dc + dd) * rank + k) : 0.f;
      }
      __syncthreads();  // dtf is complete; the previous chunk's weights have been read
#pragma unroll
      for (int q = 0; q < kWq; ++q) {
        const int i = tid + kXpThreads * q;
        wdt[(i / kXpDChunk) * kXpDChunk + i % kXpDChunk] = r[q];
      }
      __syncthreads();
      float2 a2[6];
#pragma unroll
      for (int i = 0; i < 6; ++i) a2[i] = make_float2(0.f, 0.f);
      const float* wrow = wdt + 12 * warp;
#pragma unroll 4
      for (int k = 0; k < rank; ++k) {
        const float dv = dtf[k * kXpDtRow + lane];
        const float2 d2 = make_float2(dv, dv);
        const float4 w0 = *reinterpret_cast<const float4*>(wrow + k * kXpDChunk);
        const float4 w1 = *reinterpret_cast<const float4*>(wrow + k * kXpDChunk + 4);
        const float4 w2 = *reinterpret_cast<const float4*>(wrow + k * kXpDChunk + 8);
        a2[0] = mamba_scan::fma2(make_float2(w0.x, w0.y), d2, a2[0]);
        a2[1] = mamba_scan::fma2(make_float2(w0.z, w0.w), d2, a2[1]);
        a2[2] = mamba_scan::fma2(make_float2(w1.x, w1.y), d2, a2[2]);
        a2[3] = mamba_scan::fma2(make_float2(w1.z, w1.w), d2, a2[3]);
        a2[4] = mamba_scan::fma2(make_float2(w2.x, w2.y), d2, a2[4]);
        a2[5] = mamba_scan::fma2(make_float2(w2.z, w2.w), d2, a2[5]);
      }
      const int t = t0 + lane;
      if (t < seqlen) {
#pragma unroll
        for (int i = 0; i < 6; ++i) {
          const int d = dc + 12 * warp + 2 * i;
          float* o = delta + ((int64_t)b * dim + d) * seqlen + t;
          if (d < d_hi) o[0] = a2[i].x;
          if (d + 1 < d_hi) o[seqlen] = a2[i].y;
        }
      }
    }
  }
  cluster.sync();  // no CTA leaves while another still reads its shared memory
}

// x_proj for a few tokens (decoding): 4 warps per (token, output), each
// summing a quarter of d_inner with 8 independent partial sums per lane
// (loads in flight together), then a fixed shuffle tree and a fixed-order
// sum of the 4 warps' results through shared memory (deterministic).
constexpr int kXpFewTokens = 16;  // batch * seqlen up to this take this kernel
__global__ void __launch_bounds__(256)
    xproj_few_kernel(const float* __restrict__ x, const float* __restrict__ w,
                     float* __restrict__ dt, float* __restrict__ Bm, float* __restrict__ Cm,
                     int dim, int seqlen, int rank, int dstate) {
  pdl_enter();
  __shared__ float part[2][4];
  const int P = rank + 2 * dstate;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int jj = warp >> 2, q = warp & 3;  // 2 outputs per CTA, 4 warps each
  const int j = blockIdx.x * 2 + jj;
  const int tok = blockIdx.y, b = tok / seqlen, t = tok - b * seqlen;
  const int per = (dim + 3) / 4, d_lo = min(dim, q * per), d_hi = min(dim, d_lo + per);
  float acc = 0.f;
  if (j < P) {
    const float* xr = x + (int64_t)b * dim * seqlen + t;
    const float* wr = w + (int64_t)j * dim;
    float a[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) a[u] = 0.f;
    for (int d0 = d_lo + lane; d0 < d_hi; d0 += 32 * 8) {
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int d = d0 + 32 * u;
        if (d < d_hi) a[u] = fmaf(__ldg(wr + d), __ldg(xr + (int64_t)d * seqlen), a[u]);
      }
    }
    acc = ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
  }
  acc = warp_sum(acc);
  if (lane == 0) part[jj][q] = acc;
  __syncthreads();
  if (threadIdx.x < 2) {
    const int jo = blockIdx.x * 2 + threadIdx.x;
    if (jo < P) {
      const float sum = (part[threadIdx.x][0] + part[threadIdx.x][1]) +
                        (part[threadIdx.x][2] + part[threadIdx.x][3]);
      const int64_t row = (int64_t)b * seqlen + t;
      if (jo < rank)
        dt[row * rank + jo] = sum;
      else if (jo < rank + dstate)
        Bm[row * dstate + (jo - rank)] = sum;
      else
        Cm[row * dstate + (jo - rank - dstate)] = sum;
    }
  }
}

cudaError_t launch_xproj(dim3 grid, cudaStream_t st, const float* x, const float* w, float* dt,
                         float* Bm, float* Cm, int dim, int seqlen, int rank, int dstate,
                         const float* w_dt = nullptr, float* delta = nullptr) {
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [] {
    attr = cudaFuncSetAttribute(xproj_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)kXpSmemBytes);
    if (attr == cudaSuccess)
      attr = cudaFuncSetAttribute(xproj_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)kXpSmemBytes);
  });
  if (attr != cudaSuccess) return attr;
  if (delta != nullptr)
    return launch_pdl(xproj_kernel<true>, grid, dim3(kXpThreads), kXpSmemBytes, st, x, w, dt, Bm,
                      Cm, dim, seqlen, rank, dstate, w_dt, delta);
  return launch_pdl(xproj_kernel<false>, grid, dim3(kXpThreads), kXpSmemBytes, st, x, w, dt, Bm,
                    Cm, dim, seqlen, rank, dstate, w_dt, delta);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool overlap(const void* a, size_t abytes, const void* b, size_t bbytes) {
  const auto a0 = reinterpret_cast<uintptr_t>(a), b0 = reinterpret_cast<uintptr_t>(b);
  return a0 < b0 + bbytes && b0 < a0 + abytes;
}

// ----------------------------------------------------------------- dt_proj

// delta[b, d, l] = sum_k W[d, k] * dt[b, l, k]: the block's dt_proj (its bias
// is added inside the scan op, through delta_bias), written as the [B, D, L]
// delta the scan reads. A GEMM with K = dt_rank (48 for Mamba-130m), far too
// shallow for tensor-core tiles to pay. One CTA of 128 threads per 64 (d) x
// 64 (l) tile (Mamba-130m: 384 CTAs, all resident at once), K in steps of up
// to 64 held whole in shared memory, stored k-major so that each thread
// reads its 4 d and 8 l values as float4s; each thread keeps 4 x 8 outputs
// (packed FFMA2 over l pairs) summed in k order, and stores float4 runs
// along l. The weight tile is loaded before waiting for the previous kernel.
//
// Both operands are [rows][rank] in memory (k contiguous): kVec (rank % 4 ==
// 0, 16-byte aligned bases) loads them as float4 runs along k, coalesced,
// and scatters each into 4 k-rows of the tile. Columns are swizzled in
// groups of 4 (group g of k-row k sits at g ^ ((k / 4) % 8)), so those
// scattered stores spread over the banks while the float4 reads of 4
// consecutive columns stay whole and aligned.
constexpr int kDtBM = 64, kDtBN = 64, kDtBK = 64, kDtThreads = 128;

__device__ __forceinline__ int dt_swz(int c, int k) {
  return ((((c >> 2) ^ (k >> 2)) & 7) | ((c >> 2) & 8)) << 2 | (c & 3);
}

template <bool kVec>
__global__ void __launch_bounds__(kDtThreads)
    dt_proj_kernel(const float* __restrict__ dt, const float* __restrict__ w,
                   float* __restrict__ delta, int dim, int seqlen, int rank) {
  __shared__ __align__(16) float ws[kDtBK][kDtBM];
  __shared__ __align__(16) float xs[kDtBK][kDtBN];
  const int tid = threadIdx.x;
  const int b = blockIdx.z, d0 = blockIdx.y * kDtBM, l0 = blockIdx.x * kDtBN;
  const float* dtb = dt + (int64_t)b * seqlen * rank;
  const int ty = tid >> 3, tx = tid & 7;  // outputs: d0 + 4ty + i, l0 + 4tx + {0..3, 32..35}
  float2 acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = make_float2(0.f, 0.f);
  // kVec loaders: float4 q = tid + 128 j of a 64 x 64 tile is (row q / 16,
  // k = 4 (q % 16)); otherwise element i = tid + 128 j is (row i % 64,
  // k = i / 64). Every load of a tile is issued before any is stored.
  constexpr int kLd = kDtBM * kDtBK / kDtThreads;  // 32 elements per thread and tile
  constexpr int kLd4 = kLd / 4;
  float r[kLd];
  // a tile of a [rows][rank] operand (rows from row0, K step k0, kn wide)
  // into registers
  auto load = [&](const float* src, int row0, int nrows, int k0, int kn) {
    if (kVec) {
#pragma unroll
      for (int j = 0; j < kLd4; ++j) {
        const int q = tid + kDtThreads * j, row = q >> 4, k = 4 * (q & 15);
        const float4 v = (row0 + row < nrows && k < kn)
                             ? __ldg(reinterpret_cast<const float4*>(
                                   src + (int64_t)(row0 + row) * rank + k0 + k))
                             : make_float4(0.f, 0.f, 0.f, 0.f);
        r[4 * j] = v.x;
        r[4 * j + 1] = v.y;
        r[4 * j + 2] = v.z;
        r[4 * j + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < kLd; ++j) {
        const int row = tid & 63, k = (tid >> 6) + 2 * j;
        r[j] = (row0 + row < nrows && k < kn) ? src[(int64_t)(row0 + row) * rank + k0 + k] : 0.f;
      }
    }
  };
  auto store = [&](float (*tile)[64]) {
    if (kVec) {
#pragma unroll
      for (int j = 0; j < kLd4; ++j) {
        const int q = tid + kDtThreads * j, row = q >> 4, k = 4 * (q & 15);
#pragma unroll
        for (int e = 0; e < 4; ++e) tile[k + e][dt_swz(row, k + e)] = r[4 * j + e];
      }
    } else {
#pragma unroll
      for (int j = 0; j < kLd; ++j) {
        const int row = tid & 63, k = (tid >> 6) + 2 * j;
        tile[k][dt_swz(row, k)] = r[j];
      }
    }
  };
  for (int k0 = 0; k0 < rank; k0 += kDtBK) {
    const int kn = min(kDtBK, rank - k0);
    if (k0 > 0) __syncthreads();  // the previous K step has been read
    load(w, d0, dim, k0, kn);
    store(ws);
    // dt is the previous kernel's output (x_proj): wait for it (a no-op
    // unless launched as a programmatic dependent launch)
    if (k0 == 0) pdl_enter();
    load(dtb, l0, seqlen, k0, kn);
    store(xs);
    __syncthreads();
#pragma unroll 8
    for (int k = 0; k < kn; ++k) {
      // dt_swz of these 4-aligned columns: the group index XOR (k / 4) % 8
      const int f = (k >> 2) & 7;
      const float4 wv = *reinterpret_cast<const float4*>(&ws[k][4 * (ty ^ f)]);
      const float4 x0 = *reinterpret_cast<const float4*>(&xs[k][4 * (tx ^ f)]);
      const float4 x1 = *reinterpret_cast<const float4*>(&xs[k][4 * ((8 + tx) ^ f)]);
      const float wi[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 w2 = make_float2(wi[i], wi[i]);
        acc[i][0] = mamba_scan::fma2(w2, make_float2(x0.x, x0.y), acc[i][0]);
        acc[i][1] = mamba_scan::fma2(w2, make_float2(x0.z, x0.w), acc[i][1]);
        acc[i][2] = mamba_scan::fma2(w2, make_float2(x1.x, x1.y), acc[i][2]);
        acc[i][3] = mamba_scan::fma2(w2, make_float2(x1.z, x1.w), acc[i][3]);
      }
    }
  }
  const bool vec = (seqlen & 3) == 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int d = d0 + 4 * ty + i;
    if (d >= dim) break;
    float* row = delta + ((int64_t)b * dim + d) * seqlen;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int l = l0 + 32 * h + 4 * tx;
      const float2 a = acc[i][2 * h], c = acc[i][2 * h + 1];
      if (vec && l + 3 < seqlen) {
        *reinterpret_cast<float4*>(row + l) = make_float4(a.x, a.y, c.x, c.y);
      } else {
        const float v[4] = {a.x, a.y, c.x, c.y};
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (l + j < seqlen) row[l + j] = v[j];
      }
    }
  }
}

}  // namespace

extern "C" {

int mamba_rmsnorm(const float* x, const float* weight, float* y, int64_t rows, int64_t cols,
                  float eps, void* stream) {
  using mamba_scan::set_last_error;
  if (rows < 0 || cols <= 0 || cols > (1 << 20))
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "rmsnorm: bad rows/cols");
  if (rows == 0) return MAMBA_SCAN_OK;
  if (!x || !weight || !y)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "rmsnorm: NULL pointer");
  {
    const uintptr_t x0 = reinterpret_cast<uintptr_t>(x), y0 = reinterpret_cast<uintptr_t>(y);
    const uintptr_t n = (uintptr_t)rows * (uintptr_t)cols * 4;
    if (x0 < y0 + n && y0 < x0 + n)
      return set_last_error(MAMBA_SCAN_ERR_ALIASING, "rmsnorm: y overlaps x");
  }
  if (rows > ((int64_t)1 << 31) * kNormWarps)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "rmsnorm: too many rows");
  const unsigned grid = (unsigned)((rows + kNormWarps - 1) / kNormWarps);
  const bool vec = cols % 4 == 0 && aligned16(x) && aligned16(weight) && aligned16(y);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* const none = nullptr;
  const cudaError_t e =
      vec ? launch_pdl(rmsnorm_kernel<true>, dim3(grid), dim3(kNormWarps * 32), 0, st, x, weight,
                       y, rows, (int)cols, eps, none, none, (int64_t)0)
          : launch_pdl(rmsnorm_kernel<false>, dim3(grid), dim3(kNormWarps * 32), 0, st, x, weight,
                       y, rows, (int)cols, eps, none, none, (int64_t)0);
  if (e != cudaSuccess) return set_last_error(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));
  return MAMBA_SCAN_OK;
}

int mamba_rmsnorm_split_tf32(const float* x, const float* weight, int64_t rows, int64_t cols,
                             float eps, float* hi, float* lo, int64_t ld, void* stream) {
  using mamba_scan::set_last_error;
  if (rows < 0 || cols <= 0 || cols > (1 << 20))
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "rmsnorm_split_tf32: bad rows/cols");
  if (rows == 0) return MAMBA_SCAN_OK;
  if (!x || !weight || !hi || !lo)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "rmsnorm_split_tf32: NULL pointer");
  if (cols % 4 != 0 || ld < cols || ld % 4 != 0 || !aligned16(x) || !aligned16(weight) ||
      !aligned16(hi) || !aligned16(lo))
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT,
                          "rmsnorm_split_tf32: cols and ld must be multiples of 4 (ld >= cols) "
                          "and every pointer 16-byte aligned");
  {
    const uintptr_t x0 = reinterpret_cast<uintptr_t>(x), n = (uintptr_t)rows * (uintptr_t)cols * 4;
    const uintptr_t m = ((uintptr_t)(rows - 1) * (uintptr_t)ld + (uintptr_t)cols) * 4;
    const uintptr_t h0 = reinterpret_cast<uintptr_t>(hi), l0 = reinterpret_cast<uintptr_t>(lo);
    if ((x0 < h0 + m && h0 < x0 + n) || (x0 < l0 + m && l0 < x0 + n) ||
        (h0 < l0 + m && l0 < h0 + m))
      return set_last_error(MAMBA_SCAN_ERR_ALIASING,
                            "rmsnorm_split_tf32: x, hi and lo must not overlap");
  }
  if (rows > ((int64_t)1 << 31) * kNormWarps)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "rmsnorm_split_tf32: too many rows");
  const unsigned grid = (unsigned)((rows + kNormWarps - 1) / kNormWarps);
  float* const none = nullptr;
  const cudaError_t e = launch_pdl(rmsnorm_kernel<true, true>, dim3(grid), dim3(kNormWarps * 32), 0,
                                   static_cast<cudaStream_t>(stream), x, weight, none, rows,
                                   (int)cols, eps, hi, lo, ld);
  if (e != cudaSuccess) return set_last_error(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));
  return MAMBA_SCAN_OK;
}

int mamba_causal_conv1d_silu(const float* x, int64_t x_batch_stride, const float* weight,
                             const float* bias, float* y, int64_t batch, int64_t dim,
                             int64_t seqlen, int64_t width, void* stream) {
  using mamba_scan::set_last_error;
  if (batch < 0 || dim < 0 || seqlen < 0 || width < 1 || width > kConvMaxWidth)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT,
                          "causal_conv1d_silu: bad shape (width must be 1.." +
                              std::to_string(kConvMaxWidth) + ")");
  if (batch == 0 || dim == 0 || seqlen == 0) return MAMBA_SCAN_OK;
  if (!x || !weight || !y)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "causal_conv1d_silu: NULL pointer");
  if (x_batch_stride < dim * seqlen)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT,
                          "causal_conv1d_silu: batch stride below dim * seqlen");
  const int64_t blocks_per_row = (seqlen + 3) / 4;
  const int64_t n_items = batch * dim * blocks_per_row;
  if (n_items / kConvThreads >= ((int64_t)1 << 31))
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "causal_conv1d_silu: too large");
  // x and y must not overlap: other threads still read x where y is written
  const uintptr_t x0 = reinterpret_cast<uintptr_t>(x), y0 = reinterpret_cast<uintptr_t>(y);
  const uintptr_t x1 = x0 + (size_t)((batch - 1) * x_batch_stride + dim * seqlen) * 4;
  const uintptr_t y1 = y0 + (size_t)(batch * dim * seqlen) * 4;
  if (x0 < y1 && y0 < x1)
    return set_last_error(MAMBA_SCAN_ERR_ALIASING, "causal_conv1d_silu: y overlaps x");
  const unsigned grid = (unsigned)((n_items + kConvThreads - 1) / kConvThreads);
  const bool vec = seqlen % 4 == 0 && x_batch_stride % 4 == 0 && aligned16(x) && aligned16(y);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t t_blocks = (blocks_per_row + kConvThreads - 1) / kConvThreads;
  if (vec && width == 4 && aligned16(weight) && batch * dim < ((int64_t)1 << 31) &&
      t_blocks <= 65535) {
    const cudaError_t e =
        launch_pdl(conv4_silu_kernel, dim3((unsigned)(batch * dim), (unsigned)t_blocks),
                   dim3(kConvThreads), 0, st, x, x_batch_stride, weight, bias, y, (unsigned)dim,
                   seqlen);
    if (e != cudaSuccess) return set_last_error(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));
    return MAMBA_SCAN_OK;
  }
  const cudaError_t e =
      vec ? launch_pdl(conv_silu_kernel<true>, dim3(grid), dim3(kConvThreads), 0, st, x,
                       x_batch_stride, weight, bias, y, dim, seqlen, blocks_per_row, n_items,
                       (int)width)
          : launch_pdl(conv_silu_kernel<false>, dim3(grid), dim3(kConvThreads), 0, st, x,
                       x_batch_stride, weight, bias, y, dim, seqlen, blocks_per_row, n_items,
                       (int)width);
  if (e != cudaSuccess) return set_last_error(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));
  return MAMBA_SCAN_OK;
}

int mamba_x_proj(const float* x, const float* weight, float* dt, float* B, float* C,
                 int64_t batch, int64_t dim, int64_t seqlen, int64_t rank, int64_t dstate,
                 void* stream) {
  using mamba_scan::set_last_error;
  if (batch < 0 || dim < 0 || seqlen < 0 || rank < 1 || dstate < 1 ||
      rank + 2 * dstate > kXpMaxOut)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT,
                          "x_proj: bad shape (rank + 2 * dstate must be 3.." +
                              std::to_string(kXpMaxOut) + ")");
  if (batch == 0 || seqlen == 0) return MAMBA_SCAN_OK;
  if (!x || !weight || !dt || !B || !C || dim == 0)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "x_proj: NULL pointer or dim 0");
  if (batch > 65535 || dim > ((int64_t)1 << 30) || seqlen > ((int64_t)1 << 30) ||
      (seqlen + kXpTokens - 1) / kXpTokens * kXpCluster > 0x7FFFFFFF)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "x_proj: too large");
  const size_t xb = (size_t)(batch * dim * seqlen) * 4, wb = (size_t)((rank + 2 * dstate) * dim) * 4;
  const size_t dtb = (size_t)(batch * seqlen * rank) * 4, bcb = (size_t)(batch * seqlen * dstate) * 4;
  const void* outs[3] = {dt, B, C};
  const size_t out_bytes[3] = {dtb, bcb, bcb};
  for (int i = 0; i < 3; ++i) {
    if (overlap(outs[i], out_bytes[i], x, xb) || overlap(outs[i], out_bytes[i], weight, wb))
      return set_last_error(MAMBA_SCAN_ERR_ALIASING, "x_proj: an output overlaps an input");
    for (int k = i + 1; k < 3; ++k)
      if (overlap(outs[i], out_bytes[i], outs[k], out_bytes[k]))
        return set_last_error(MAMBA_SCAN_ERR_ALIASING, "x_proj: outputs overlap");
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (batch * seqlen <= kXpFewTokens) {
    const dim3 few((unsigned)((rank + 2 * dstate + 1) / 2), (unsigned)(batch * seqlen));
    const cudaError_t e = launch_pdl(xproj_few_kernel, few, dim3(256), 0, st, x, weight, dt, B, C,
                                     (int)dim, (int)seqlen, (int)rank, (int)dstate);
    if (e != cudaSuccess) return set_last_error(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));
    return MAMBA_SCAN_OK;
  }
  const dim3 grid((unsigned)((seqlen + kXpTokens - 1) / kXpTokens * kXpCluster), (unsigned)batch);
  const cudaError_t e = launch_xproj(grid, st, x, weight, dt, B, C, (int)dim, (int)seqlen,
                                     (int)rank, (int)dstate);
  if (e != cudaSuccess) return set_last_error(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));
  return MAMBA_SCAN_OK;
}

int mamba_x_proj_delta(const float* x, const float* weight, const float* dt_weight, float* delta,
                       float* B, float* C, int64_t batch, int64_t dim, int64_t seqlen,
                       int64_t rank, int64_t dstate, void* stream) {
  using mamba_scan::set_last_error;
  if (batch < 0 || dim < 0 || seqlen < 0 || rank < 1 || dstate < 1 || rank > kXpDtMaxRank ||
      rank + 2 * dstate > kXpMaxOut)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT,
                          "x_proj_delta: bad shape (rank 1.." + std::to_string(kXpDtMaxRank) +
                              ", rank + 2 * dstate <= " + std::to_string(kXpMaxOut) + ")");
  if (batch == 0 || seqlen == 0 || dim == 0) return MAMBA_SCAN_OK;
  if (!x || !weight || !dt_weight || !delta || !B || !C)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "x_proj_delta: NULL pointer");
  if (batch > 65535 || dim > ((int64_t)1 << 30) || seqlen > ((int64_t)1 << 30) ||
      (seqlen + kXpTokens - 1) / kXpTokens * kXpCluster > 0x7FFFFFFF)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "x_proj_delta: too large");
  const size_t xb = (size_t)(batch * dim * seqlen) * 4, wb = (size_t)((rank + 2 * dstate) * dim) * 4;
  const size_t wdb = (size_t)(dim * rank) * 4, bcb = (size_t)(batch * seqlen * dstate) * 4;
  const void* outs[3] = {delta, B, C};
  const size_t out_bytes[3] = {xb, bcb, bcb};
  for (int i = 0; i < 3; ++i) {
    if (overlap(outs[i], out_bytes[i], x, xb) || overlap(outs[i], out_bytes[i], weight, wb) ||
        overlap(outs[i], out_bytes[i], dt_weight, wdb))
      return set_last_error(MAMBA_SCAN_ERR_ALIASING, "x_proj_delta: an output overlaps an input");
    for (int k = i + 1; k < 3; ++k)
      if (overlap(outs[i], out_bytes[i], outs[k], out_bytes[k]))
        return set_last_error(MAMBA_SCAN_ERR_ALIASING, "x_proj_delta: outputs overlap");
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)((seqlen + kXpTokens - 1) / kXpTokens * kXpCluster), (unsigned)batch);
  const cudaError_t e = launch_xproj(grid, st, x, weight, nullptr, B, C, (int)dim, (int)seqlen,
                                     (int)rank, (int)dstate, dt_weight, delta);
  if (e != cudaSuccess) return set_last_error(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));
  return MAMBA_SCAN_OK;
}

int mamba_dt_proj(const float* dt, const float* weight, float* delta, int64_t batch, int64_t dim,
                  int64_t seqlen, int64_t rank, void* stream) {
  using mamba_scan::set_last_error;
  if (batch < 0 || dim < 0 || seqlen < 0 || rank < 1)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "dt_proj: bad shape");
  if (batch == 0 || dim == 0 || seqlen == 0) return MAMBA_SCAN_OK;
  if (!dt || !weight || !delta)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "dt_proj: NULL pointer");
  if (batch > 65535 || dim > ((int64_t)1 << 30) || seqlen > ((int64_t)1 << 30) ||
      rank > ((int64_t)1 << 20) || (dim + kDtBM - 1) / kDtBM > 65535)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "dt_proj: too large");
  const size_t db = (size_t)(batch * dim * seqlen) * 4;
  if (overlap(delta, db, dt, (size_t)(batch * seqlen * rank) * 4) ||
      overlap(delta, db, weight, (size_t)(dim * rank) * 4))
    return set_last_error(MAMBA_SCAN_ERR_ALIASING, "dt_proj: delta overlaps an input");
  const dim3 grid((unsigned)((seqlen + kDtBN - 1) / kDtBN), (unsigned)((dim + kDtBM - 1) / kDtBM),
                  (unsigned)batch);
  if (rank % 4 == 0 && aligned16(dt) && aligned16(weight))
    dt_proj_kernel<true><<<grid, kDtThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        dt, weight, delta, (int)dim, (int)seqlen, (int)rank);
  else
    dt_proj_kernel<false><<<grid, kDtThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        dt, weight, delta, (int)dim, (int)seqlen, (int)rank);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_last_error(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));
  return MAMBA_SCAN_OK;
}

int mamba_causal_conv1d_step(float* state, const float* x, int64_t x_batch_stride,
                             const float* weight, const float* bias, float* y, int64_t batch,
                             int64_t dim, int64_t width, void* stream) {
  using mamba_scan::set_last_error;
  if (batch < 0 || dim < 0 || width < 1 || width > kConvMaxWidth)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT,
                          "causal_conv1d_step: bad shape (width must be 1.." +
                              std::to_string(kConvMaxWidth) + ")");
  if (batch == 0 || dim == 0) return MAMBA_SCAN_OK;
  if (!state || !x || !weight || !y)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "causal_conv1d_step: NULL pointer");
  if (x_batch_stride < dim || batch * dim / kConvThreads >= ((int64_t)1 << 31))
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT,
                          "causal_conv1d_step: bad batch stride or too large");
  const size_t sb = (size_t)(batch * dim * width) * 4, yb = (size_t)(batch * dim) * 4;
  const size_t xb = (size_t)((batch - 1) * x_batch_stride + dim) * 4;
  if (overlap(y, yb, state, sb) || overlap(y, yb, x, xb) || overlap(state, sb, x, xb))
    return set_last_error(MAMBA_SCAN_ERR_ALIASING, "causal_conv1d_step: buffers overlap");
  const unsigned grid = (unsigned)((batch * dim + kConvThreads - 1) / kConvThreads);
  const cudaError_t e =
      launch_pdl(conv_step_kernel, dim3(grid), dim3(kConvThreads), 0,
                 static_cast<cudaStream_t>(stream), state, x, x_batch_stride, weight, bias, y,
                 batch, dim, (int)width);
  if (e != cudaSuccess) return set_last_error(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));
  return MAMBA_SCAN_OK;
}

int mamba_ssm_decode_step(const float* u, const float* z, int64_t z_batch_stride,
                          const float* dt, const float* B, const float* C, const float* dt_weight,
                          const float* dt_bias, const float* A, const float* D, float* state,
                          float* y, int64_t batch, int64_t dim, int64_t rank, int64_t dstate,
                          void* stream) {
  using mamba_scan::set_last_error;
  if (dstate != kSsmN)
    return set_last_error(MAMBA_SCAN_ERR_UNSUPPORTED_DSTATE,
                          "ssm_decode_step: only dstate=16 is supported");
  if (batch < 0 || dim < 0 || rank < 1 || rank > kSsmMaxRank)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT,
                          "ssm_decode_step: bad shape (rank 1.." + std::to_string(kSsmMaxRank) + ")");
  if (batch == 0 || dim == 0) return MAMBA_SCAN_OK;
  if (!u || !z || !dt || !B || !C || !dt_weight || !A || !D || !state || !y)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "ssm_decode_step: NULL pointer");
  if (z_batch_stride < dim || batch > 65535 || dim > ((int64_t)1 << 30))
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT,
                          "ssm_decode_step: bad z batch stride or too large");
  const size_t yb = (size_t)(batch * dim) * 4, sb = yb * kSsmN;
  const void* ins[] = {u, z, dt, B, C, dt_weight, A, D};
  const size_t in_bytes[] = {yb, (size_t)((batch - 1) * z_batch_stride + dim) * 4,
                             (size_t)(batch * rank) * 4, (size_t)(batch * kSsmN) * 4,
                             (size_t)(batch * kSsmN) * 4, (size_t)(dim * rank) * 4,
                             (size_t)(dim * kSsmN) * 4, (size_t)dim * 4};
  for (int i = 0; i < 8; ++i)
    if (overlap(y, yb, ins[i], in_bytes[i]) || overlap(state, sb, ins[i], in_bytes[i]))
      return set_last_error(MAMBA_SCAN_ERR_ALIASING,
                            "ssm_decode_step: y or state overlaps an input");
  if (overlap(y, yb, state, sb))
    return set_last_error(MAMBA_SCAN_ERR_ALIASING, "ssm_decode_step: y overlaps state");
  const dim3 grid((unsigned)((dim + kSsmThreads - 1) / kSsmThreads), (unsigned)batch);
  const cudaError_t e =
      launch_pdl(ssm_step_kernel, grid, dim3(kSsmThreads), 0, static_cast<cudaStream_t>(stream),
                 u, z, z_batch_stride, dt, B, C, dt_weight, dt_bias, A, D, state, y, (int)dim,
                 (int)rank);
  if (e != cudaSuccess) return set_last_error(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));
  return MAMBA_SCAN_OK;
}

int mamba_rmsnorm_gemv(const float* x, const float* norm_weight, float eps, const float* weight,
                       float* out, int64_t batch, int64_t cols, int64_t rows_out, void* stream) {
  using mamba_scan::set_last_error;
  if (batch < 0 || cols < 1 || cols > kNgMaxCols || cols % 4 != 0 || rows_out < 0)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT,
                          "rmsnorm_gemv: cols must be a multiple of 4 in 4.." +
                              std::to_string(kNgMaxCols));
  if (batch == 0 || rows_out == 0) return MAMBA_SCAN_OK;
  if (!x || !norm_weight || !weight || !out)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "rmsnorm_gemv: NULL pointer");
  if (!aligned16(weight) || batch > 65535 || rows_out > ((int64_t)1 << 30))
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT,
                          "rmsnorm_gemv: weight must be 16-byte aligned; or too large");
  const size_t ob = (size_t)(batch * rows_out) * 4;
  if (overlap(out, ob, x, (size_t)(batch * cols) * 4) ||
      overlap(out, ob, weight, (size_t)(rows_out * cols) * 4) ||
      overlap(out, ob, norm_weight, (size_t)cols * 4))
    return set_last_error(MAMBA_SCAN_ERR_ALIASING, "rmsnorm_gemv: out overlaps an input");
  const dim3 grid((unsigned)((rows_out + kNgThreads / 32 - 1) / (kNgThreads / 32)), (unsigned)batch);
  const cudaError_t e =
      launch_pdl(norm_gemv_kernel, grid, dim3(kNgThreads), 0, static_cast<cudaStream_t>(stream),
                 x, norm_weight, weight, out, (int)cols, (int)rows_out, eps);
  if (e != cudaSuccess) return set_last_error(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));
  return MAMBA_SCAN_OK;
}

int mamba_gemv(const float* x, const float* weight, const float* residual, float* out,
               int64_t batch, int64_t cols, int64_t rows_out, void* stream) {
  using mamba_scan::set_last_error;
  if (batch < 0 || cols < 1 || cols > kNgMaxCols || cols % 4 != 0 || rows_out < 0)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT,
                          "gemv: cols must be a multiple of 4 in 4.." + std::to_string(kNgMaxCols));
  if (batch == 0 || rows_out == 0) return MAMBA_SCAN_OK;
  if (!x || !weight || !out)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "gemv: NULL pointer");
  if (!aligned16(weight) || batch > 65535 || rows_out > ((int64_t)1 << 30))
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT,
                          "gemv: weight must be 16-byte aligned; or too large");
  const size_t ob = (size_t)(batch * rows_out) * 4;
  if (overlap(out, ob, x, (size_t)(batch * cols) * 4) ||
      overlap(out, ob, weight, (size_t)(rows_out * cols) * 4) ||
      (residual && residual != out && overlap(out, ob, residual, ob)))
    return set_last_error(MAMBA_SCAN_ERR_ALIASING,
                          "gemv: out overlaps x or weight (residual may be out itself)");
  const dim3 grid((unsigned)((rows_out + kNgThreads / 32 - 1) / (kNgThreads / 32)), (unsigned)batch);
  const cudaError_t e =
      launch_pdl(gemv_kernel, grid, dim3(kNgThreads), 0, static_cast<cudaStream_t>(stream), x,
                 weight, residual, out, (int)cols, (int)rows_out);
  if (e != cudaSuccess) return set_last_error(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));
  return MAMBA_SCAN_OK;
}

}  // extern "C"
