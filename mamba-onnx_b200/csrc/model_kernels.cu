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
// Both are memory-bound (two HBM passes over their tensor); the C entry
// points are declared in include/mamba_model_ops.h.
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/mamba_model_ops.h"
#include "../../include/mamba_scan.h"
#include "scan_kernels.h"

namespace {

constexpr int kNormWarps = 8;        // rows per CTA of the RMSNorm kernel
constexpr int kConvThreads = 256;    // threads per CTA of the convolution kernel
constexpr int kConvMaxWidth = 8;     // widest convolution supported

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// kVec: rows of cols % 4 == 0 floats with 16-byte aligned bases.
template <bool kVec>
__global__ void __launch_bounds__(kNormWarps * 32)
    rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                   float* __restrict__ y, int64_t rows, int cols, float eps) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * kNormWarps + warp;
  if (r >= rows) return;
  const float* xr = x + r * cols;
  float* yr = y + r * cols;
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
      *reinterpret_cast<float4*>(yr + c) =
          make_float4(v.x * inv * g.x, v.y * inv * g.y, v.z * inv * g.z, v.w * inv * g.w);
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

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

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
  if (vec)
    rmsnorm_kernel<true><<<grid, kNormWarps * 32, 0, st>>>(x, weight, y, rows, (int)cols, eps);
  else
    rmsnorm_kernel<false><<<grid, kNormWarps * 32, 0, st>>>(x, weight, y, rows, (int)cols, eps);
  const cudaError_t e = cudaGetLastError();
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
  if (vec)
    conv_silu_kernel<true><<<grid, kConvThreads, 0, st>>>(x, x_batch_stride, weight, bias, y, dim,
                                                          seqlen, blocks_per_row, n_items,
                                                          (int)width);
  else
    conv_silu_kernel<false><<<grid, kConvThreads, 0, st>>>(x, x_batch_stride, weight, bias, y,
                                                           dim, seqlen, blocks_per_row, n_items,
                                                           (int)width);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_last_error(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));
  return MAMBA_SCAN_OK;
}

}  // extern "C"
