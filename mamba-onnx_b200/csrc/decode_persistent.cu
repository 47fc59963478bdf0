// One decoding step of a whole Mamba model in one persistent kernel (sm_100a).
//
// The reference ships only the scan op; decoding with it is the caller's
// business (its block dataflow: benchmarks/profiler.py:18-150 of
// acmiyaguchi/mamba-onnx). Per token and block, the chain of separate
// launches (RMSNorm + in_proj GEMV, convolution step, x_proj, the SSM step,
// out_proj GEMV) is latency-bound: every launch waits for the previous one,
// and none has enough work to fill the GPU. Here one cooperative launch
// (one CTA of 256 threads per SM, all resident) runs every block and the
// LM head, with a grid-wide barrier between the four phases of a block:
//
//   A  every CTA normalises h (the residual stream) into shared memory;
//      warps take in_proj rows; a row of the x half then runs the
//      convolution step of its channel (window shift, conv, SiLU) -> x;
//      a row of the z half is stored -> z
//   B  x_proj: 4 warps of one CTA per output (dt, B, C)
//   C  the SSM step, one thread per (token, channel): dt_proj, softplus,
//      exp(delta A) state update in place, C.h + D u, SiLU(z) gate -> y
//   D  out_proj: warps take rows, h += W_out y
//
// and, after the last block, the final RMSNorm and the tied LM head (phase
// A's pattern without the convolution). Every sum is formed in the same
// order as in the separate kernels (mamba_rmsnorm_gemv, the convolution
// step, mamba_x_proj's few-token path, mamba_ssm_decode_step, mamba_gemv),
// so the results equal that chain's bit for bit.
//
// What a phase reads that no earlier phase of the step writes (weights,
// biases, A, the states) is loaded into registers before the barrier that
// precedes it, so that after the barrier only activations are fetched. The
// barrier is a counter in the caller's scratch (zeroed by the entry point
// before the launch) that every CTA adds to with a release reduction and
// then waits on; every wait is bounded (2 s of wall time, then an abort flag that
// makes all CTAs leave at their next barrier, and the error code
// MAMBA_SCAN_ERR_DEVICE_TIMEOUT for mamba_scan_check_device_error). Data
// written during the launch is read through L2 (ld.global.cg), never through
// the non-coherent path.
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/mamba_model_ops.h"
#include "../../include/mamba_scan.h"
#include "scan_device.cuh"
#include "scan_kernels.h"

namespace mamba_decode {

__device__ int g_decode_device_error = 0;

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kNormThreads = 256;  // threads forming a norm's sum of squares (as mamba_rmsnorm_gemv)
constexpr int kMaxBatch = 4;
constexpr int kN = 16;  // d_state
constexpr uint64_t kBarrierLimitNs = 2000000000ull;

struct Args {
  const mamba_decode_layer* layers;
  int n_layer;
  float* h;  // [batch][d_model]
  const float* norm_f;
  const float* lm_head;  // [vocab][d_model]
  float* logits;         // [batch][vocab]
  unsigned int* ctl;     // [0] barrier count, [1] abort flag
  float* xbuf;           // [batch][d_inner]: convolution output (the scan's u)
  float* zbuf;           // [batch][d_inner]
  float* xdbl;           // [batch][rank + 2 dstate]
  float* ybuf;           // [batch][d_inner]
  int batch, d_model, d_inner, width, rank, vocab;
  float eps;
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float silu_exact(float v) { return v / (1.f + expf(-v)); }

__device__ __forceinline__ unsigned int ld_acquire(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// Prefetch `bytes` from `p` into L2, one 128-byte line per lane and step.
__device__ __forceinline__ void prefetch_row(const float* p, int64_t bytes, int lane) {
  const char* c = reinterpret_cast<const char*>(p);
  for (int64_t o = (int64_t)lane * 128; o < bytes; o += 32 * 128) prefetch_l2(c + o);
}

// Grid-wide barrier number `k` (1, 2, ...): every CTA adds one to a counter
// with a release reduction (no return value, so the additions of all CTAs
// pipeline at the counter's L2 slice) and waits for it to reach k times the
// grid size. ctl: [0] counter, [1] abort flag (the first 128 bytes are zeroed
// before every launch).
constexpr int kCtlWords = 32;

// Arrival at barrier k: the CTA's writes so far are released with it. Loads
// issued between arrival and barrier_wait (the next phase's preloads) overlap
// the wait.
__device__ __forceinline__ void barrier_arrive(unsigned int* ctl) {
  __syncthreads();
  if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctl) : "memory");
}

// Wait until every CTA has arrived at barrier k; false when the launch is
// being abandoned (a wait timed out here or in another CTA). Thread 0 polls
// the counter and the abort flag with one 8-byte acquire load (ctl is the
// 16-byte aligned scratch base). No fence follows: the acquire load that sees
// the count synchronises with every CTA's release reduction, and the
// __syncthreads after it orders the other threads' reads behind it; every
// read of another CTA's results goes to L2 (__ldcg), never to a stale L1
// line. (A __threadfence here cost 0.4 us per barrier, 39 us per token.)
__device__ __noinline__ bool barrier_wait(unsigned int* ctl, unsigned int k,
                                          uint64_t limit_ns = kBarrierLimitNs) {
  __shared__ int ok_s;
  if (threadIdx.x == 0) {
    int ok = 1;
    const unsigned int target = k * gridDim.x;
    if (ld_acquire(ctl) < target) {
      const uint64_t start = mamba_scan::globaltimer_ns();
      for (uint32_t spins = 0;; ++spins) {
        unsigned long long both;
        asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(both) : "l"(ctl) : "memory");
        if ((unsigned int)both >= target) break;
        if ((unsigned int)(both >> 32) != 0u || spins >= (1u << 28)) {
          ok = 0;
          break;
        }
        if ((spins & 63u) == 63u && mamba_scan::globaltimer_ns() - start > limit_ns) {
          atomicExch(ctl + 1, 1u);
          atomicExch(&g_decode_device_error, 6);  // MAMBA_SCAN_ERR_DEVICE_TIMEOUT
          ok = 0;
          break;
        }
      }
    }
    ok_s = ok;
  }
  __syncthreads();
  return ok_s != 0;
}

// acc[b] = weight_row . xs[b] for every token, in mamba_gemv's order (float4
// steps of 128 columns per lane, then the shuffle tree).
__device__ __forceinline__ void row_dot(const float* wr, const float* xs, int cols, int batch,
                                        int lane, float (&acc)[kMaxBatch]) {
#pragma unroll
  for (int b = 0; b < kMaxBatch; ++b) acc[b] = 0.f;
  for (int c = lane * 4; c < cols; c += 128) {
    const float4 wv = __ldg(reinterpret_cast<const float4*>(wr + c));
#pragma unroll
    for (int b = 0; b < kMaxBatch; ++b) {
      if (b >= batch) break;
      const float4 xv = *reinterpret_cast<const float4*>(xs + b * cols + c);
      acc[b] = fmaf(wv.x, xv.x, acc[b]);
      acc[b] = fmaf(wv.y, xv.y, acc[b]);
      acc[b] = fmaf(wv.z, xv.z, acc[b]);
      acc[b] = fmaf(wv.w, xv.w, acc[b]);
    }
  }
#pragma unroll
  for (int b = 0; b < kMaxBatch; ++b) acc[b] = warp_sum(acc[b]);
}

// Register preloads: what a phase reads that no earlier phase of the step
// writes (weights, biases, A, the two states) is loaded before the barrier
// that precedes the phase, so that after the barrier only the activations are
// fetched (one L2 round trip). Sizes below bound the models this kernel
// takes (Mamba-130m: d_model 768, d_inner 1536, dt_rank 48, d_conv 4).
constexpr int kMaxModel = 1024;            // d_model
constexpr int kMaxInner = 2048;            // d_inner
constexpr int kMaxRankPre = 64;            // dt_rank
constexpr int kMaxConv = 4;                // d_conv
constexpr int kAI = kMaxModel / 128;       // float4 per lane of an in_proj row
constexpr int kDI = kMaxInner / 128;       // float4 per lane of an out_proj row
constexpr int kXI = kMaxInner / 4 / 256;   // x_proj: steps of 256 over a quarter row

constexpr int kRowsA = 3;                  // in_proj rows preloaded per warp
struct PreA {  // kRowsA in_proj rows of this warp; the convolution of the x half
  float4 w[kRowsA][kAI];
  float cw[kRowsA][kMaxConv], cs[kRowsA][kMaxConv], cb[kRowsA];
  struct Row2 {  // two rows of d_model (the LM head)
    float4 w[2][kAI];
  };
};
struct PreB {  // a quarter row of x_proj (warps 0-3 of CTAs holding an output)
  float w[kXI][8];
};
struct PreC {  // this thread's channel
  float4 w[kMaxRankPre / 4];
  float an[kN], hs[kN], dsk, bias;
};
struct PreD {  // one out_proj row of this warp
  float4 w[kDI];
};

// Rows of phases A and D spread over CTAs first: row sw + k * n_gw with
// sw = warp * gridDim.x + blockIdx.x.
__device__ __forceinline__ void preload_A(const Args& a, const mamba_decode_layer& L, int sw,
                                          int n_gw, int lane, PreA& p) {
  const int dm = a.d_model, di = a.d_inner;
#pragma unroll
  for (int rr = 0; rr < kRowsA; ++rr) {
    const int r = sw + rr * n_gw;
#pragma unroll
    for (int i = 0; i < kAI; ++i) {
      const int c = lane * 4 + 128 * i;
      p.w[rr][i] = (r < 2 * di && c < dm)
                       ? __ldg(reinterpret_cast<const float4*>(L.in_proj_weight + (int64_t)r * dm + c))
                       : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const bool conv = r < di && lane < a.batch;
#pragma unroll
    for (int k = 0; k < kMaxConv; ++k) {
      p.cw[rr][k] = (conv && k < a.width) ? __ldg(L.conv_weight + (int64_t)r * a.width + k) : 0.f;
      p.cs[rr][k] = (conv && k < a.width)
                        ? __ldcg(L.conv_state + ((int64_t)lane * di + r) * a.width + k)
                        : 0.f;
    }
    p.cb[rr] = (conv && L.conv_bias) ? __ldg(L.conv_bias + r) : 0.f;
  }
}

__device__ __forceinline__ void preload_B(const Args& a, const mamba_decode_layer& L, int warp,
                                          int lane, PreB& p) {
  const int di = a.d_inner, P = a.rank + 2 * kN;
  const int per = (di + 3) / 4, d_lo = min(di, (warp & 3) * per), d_hi = min(di, d_lo + per);
  const int j = blockIdx.x;
#pragma unroll
  for (int it = 0; it < kXI; ++it)
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int d = d_lo + lane + 256 * it + 32 * u;
      p.w[it][u] = (warp < 4 && j < P && d < d_hi) ? __ldg(L.x_proj_weight + (int64_t)j * di + d)
                                                   : 0.f;
    }
}

__device__ __forceinline__ void preload_C(const Args& a, const mamba_decode_layer& L, int tid,
                                          PreC& p) {
  const int di = a.d_inner, R = a.rank;
  const int i = blockIdx.x + gridDim.x * tid;
  const bool ok = i < a.batch * di;
  const int d = ok ? i % di : 0;
#pragma unroll
  for (int q = 0; q < kMaxRankPre / 4; ++q)
    p.w[q] = (ok && 4 * q < R)
                 ? __ldg(reinterpret_cast<const float4*>(L.dt_proj_weight + (int64_t)d * R) + q)
                 : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int n = 0; n < kN; ++n) {
    p.an[n] = ok ? __ldg(L.A + (int64_t)d * kN + n) : 0.f;
    p.hs[n] = ok ? __ldcg(L.ssm_state + (int64_t)i * kN + n) : 0.f;
  }
  p.dsk = ok ? __ldg(L.D + d) : 0.f;
  p.bias = (ok && L.dt_proj_bias) ? __ldg(L.dt_proj_bias + d) : 0.f;
}

__device__ __forceinline__ void preload_D(const Args& a, const mamba_decode_layer& L, int sw,
                                          int lane, PreD& p) {
  const int dm = a.d_model, di = a.d_inner;
#pragma unroll
  for (int i = 0; i < kDI; ++i) {
    const int c = lane * 4 + 128 * i;
    p.w[i] = (sw < dm && c < di)
                 ? __ldg(reinterpret_cast<const float4*>(L.out_proj_weight + (int64_t)sw * di + c))
                 : make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// xn[b][c] = x[b][c] * rsqrt(mean(x[b]^2) + eps) * w[c] for every token, the
// sum of squares by the first 256 threads in mamba_rmsnorm_gemv's order; all
// of a token's loads are issued before the sum.
__device__ __forceinline__ void norm_rows_pre(const float* x, const float* w, float* xn,
                                              float* red, int batch, int cols, float eps) {
  constexpr int kIt = kMaxModel / kNormThreads;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float wv[kIt];
#pragma unroll
  for (int k = 0; k < kIt; ++k) {
    const int c = tid + kNormThreads * k;
    wv[k] = (tid < kNormThreads && c < cols) ? __ldg(w + c) : 0.f;
  }
  for (int b = 0; b < batch; ++b) {
    float v[kIt];
#pragma unroll
    for (int k = 0; k < kIt; ++k) {
      const int c = tid + kNormThreads * k;
      v[k] = (tid < kNormThreads && c < cols) ? __ldcg(x + (int64_t)b * cols + c) : 0.f;
    }
    if (tid < kNormThreads) {
      float ss = 0.f;
#pragma unroll
      for (int k = 0; k < kIt; ++k)
        if (tid + kNormThreads * k < cols) ss = fmaf(v[k], v[k], ss);
      ss = warp_sum(ss);
      if (lane == 0) red[warp] = ss;
    }
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < kNormThreads / 32; ++i) tot += red[i];
    const float inv = rsqrtf(tot / (float)cols + eps);
#pragma unroll
    for (int k = 0; k < kIt; ++k) {
      const int c = tid + kNormThreads * k;
      if (tid < kNormThreads && c < cols) xn[b * cols + c] = v[k] * inv * wv[k];
    }
    __syncthreads();
  }
}

// acc[b] = (preloaded row) . xs[b], in mamba_gemv's order.
template <int kI>
__device__ __forceinline__ void row_dot_pre(const float4 (&w)[kI], const float* xs, int cols,
                                            int batch, int lane, float (&acc)[kMaxBatch]) {
#pragma unroll
  for (int b = 0; b < kMaxBatch; ++b) acc[b] = 0.f;
#pragma unroll
  for (int i = 0; i < kI; ++i) {
    const int c = lane * 4 + 128 * i;
    if (c >= cols) break;
#pragma unroll
    for (int b = 0; b < kMaxBatch; ++b) {
      if (b >= batch) break;
      const float4 xv = *reinterpret_cast<const float4*>(xs + b * cols + c);
      acc[b] = fmaf(w[i].x, xv.x, acc[b]);
      acc[b] = fmaf(w[i].y, xv.y, acc[b]);
      acc[b] = fmaf(w[i].z, xv.z, acc[b]);
      acc[b] = fmaf(w[i].w, xv.w, acc[b]);
    }
  }
#pragma unroll
  for (int b = 0; b < kMaxBatch; ++b) acc[b] = warp_sum(acc[b]);
}

__device__ __forceinline__ float pick(const float (&acc)[kMaxBatch], int lane) {
  float v = acc[0];
#pragma unroll
  for (int b = 1; b < kMaxBatch; ++b)
    if (lane == b) v = acc[b];
  return v;
}

// in_proj row r's outputs (acc) to the convolution step (x half: conv state
// and weights preloaded in slot rr, or loaded here when rr < 0) or to z.
__device__ __forceinline__ void finish_in_proj_row(const Args& a, const mamba_decode_layer& L,
                                                   int r, const float (&acc)[kMaxBatch], int lane,
                                                   const PreA* p, int rr) {
  const int di = a.d_inner;
  if (lane >= a.batch) return;
  const float v = pick(acc, lane);
  if (r >= di) {
    a.zbuf[(int64_t)lane * di + (r - di)] = v;
    return;
  }
  // mamba_causal_conv1d_step for (b = lane, d = r)
  float* st = L.conv_state + ((int64_t)lane * di + r) * a.width;
  float cacc = p ? p->cb[rr] : (L.conv_bias ? __ldg(L.conv_bias + r) : 0.f);
  float prev = v;
#pragma unroll
  for (int k = kMaxConv - 1; k >= 0; --k) {
    if (k >= a.width) continue;
    const float cur = p ? p->cs[rr][k] : __ldcg(st + k);
    st[k] = prev;
    cacc = fmaf(p ? p->cw[rr][k] : __ldg(L.conv_weight + (int64_t)r * a.width + k), prev, cacc);
    prev = cur;
  }
  a.xbuf[(int64_t)lane * di + r] = silu_exact(cacc);
}

__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const Args a) {
  extern __shared__ __align__(16) float dsm[];  // [batch][max(d_model, d_inner)]
  __shared__ float red[kNormThreads / 32];
  __shared__ float part[kWarps];
  __shared__ float sdt[kMaxBatch][kMaxRankPre];
  __shared__ float sB[kMaxBatch][kN], sC[kMaxBatch][kN];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int sw = warp * gridDim.x + blockIdx.x, n_gw = gridDim.x * kWarps;
  const int B = a.batch, dm = a.d_model, di = a.d_inner, R = a.rank, P = a.rank + 2 * kN;
  unsigned int bar = 0;

  PreA pa;
  preload_A(a, a.layers[0], sw, n_gw, lane, pa);
  // lane b < batch of the warp owning out_proj row sw carries h[b][sw]
  float hrow = (sw < dm && lane < B) ? __ldcg(a.h + (int64_t)lane * dm + sw) : 0.f;
  for (int l = 0; l < a.n_layer; ++l) {
    const mamba_decode_layer L = a.layers[l];
    // ---- A: RMSNorm + in_proj; the x half through the convolution step
    norm_rows_pre(a.h, L.norm_weight, dsm, red, B, dm, a.eps);
#pragma unroll
    for (int rr = 0; rr < kRowsA; ++rr) {
      const int r = sw + rr * n_gw;
      if (r < 2 * di) {
        float acc[kMaxBatch];
        row_dot_pre(pa.w[rr], dsm, dm, B, lane, acc);
        finish_in_proj_row(a, L, r, acc, lane, &pa, rr);
      }
    }
    for (int r = sw + kRowsA * n_gw; r < 2 * di; r += n_gw) {  // rows beyond the preloaded
      float acc[kMaxBatch];
      row_dot(L.in_proj_weight + (int64_t)r * dm, dsm, dm, B, lane, acc);
      finish_in_proj_row(a, L, r, acc, lane, nullptr, -1);
    }
    barrier_arrive(a.ctl);
    ++bar;
    PreB pb;
    preload_B(a, L, warp, lane, pb);
    if (!barrier_wait(a.ctl, bar)) return;

    // ---- B: x_proj, output j on 4 warps of CTA j (mamba_x_proj's few-token order)
    for (int j = blockIdx.x; j < P; j += gridDim.x) {
      const int q = warp & 3;
      const int per = (di + 3) / 4, d_lo = min(di, q * per), d_hi = min(di, d_lo + per);
      float accb[kMaxBatch];
#pragma unroll
      for (int b = 0; b < kMaxBatch; ++b) accb[b] = 0.f;
      if (warp < 4) {
        const bool pre = j == (int)blockIdx.x;
#pragma unroll
        for (int b = 0; b < kMaxBatch; ++b) {
          if (b >= B) break;
          const float* xr = a.xbuf + (int64_t)b * di;
          float xv[kXI][8];
#pragma unroll
          for (int it = 0; it < kXI; ++it)
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              const int d = d_lo + lane + 256 * it + 32 * u;
              xv[it][u] = d < d_hi ? __ldcg(xr + d) : 0.f;
            }
          float s[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) s[u] = 0.f;
#pragma unroll
          for (int it = 0; it < kXI; ++it)
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              const int d = d_lo + lane + 256 * it + 32 * u;
              if (d < d_hi) {
                const float wv = pre ? pb.w[it][u] : __ldg(L.x_proj_weight + (int64_t)j * di + d);
                s[u] = fmaf(wv, xv[it][u], s[u]);
              }
            }
          accb[b] = warp_sum(((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7])));
        }
      }
      for (int b = 0; b < B; ++b) {
        if (warp < 4 && lane == 0) part[warp] = accb[b];
        __syncthreads();
        if (tid == 0) a.xdbl[(int64_t)b * P + j] = (part[0] + part[1]) + (part[2] + part[3]);
        __syncthreads();
      }
    }
    barrier_arrive(a.ctl);
    ++bar;
    PreC pc;
    preload_C(a, L, tid, pc);
    if (!barrier_wait(a.ctl, bar)) return;

    // ---- C: SSM step, thread per (b, d) (mamba_ssm_decode_step's arithmetic)
    for (int i = tid; i < B * R; i += kThreads) sdt[i / R][i % R] = __ldcg(a.xdbl + (int64_t)(i / R) * P + i % R);
    if (tid < B * kN) {
      const int b = tid / kN, n = tid % kN;
      sB[b][n] = __ldcg(a.xdbl + (int64_t)b * P + R + n);
      sC[b][n] = __ldcg(a.xdbl + (int64_t)b * P + R + kN + n);
    }
    {
      const int i = blockIdx.x + gridDim.x * tid;
      const bool ok = i < B * di;
      const float uv = ok ? __ldcg(a.xbuf + i) : 0.f;
      const float zv = ok ? __ldcg(a.zbuf + i) : 0.f;
      __syncthreads();
      if (ok) {
        const int b = i / di;
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
        if ((R & 3) == 0 && (reinterpret_cast<uintptr_t>(L.dt_proj_weight) & 15u) == 0) {
#pragma unroll
          for (int q = 0; q < kMaxRankPre / 4; ++q) {
            if (4 * q >= R) break;
            a0 = fmaf(pc.w[q].x, sdt[b][4 * q], a0);
            a1 = fmaf(pc.w[q].y, sdt[b][4 * q + 1], a1);
            a2 = fmaf(pc.w[q].z, sdt[b][4 * q + 2], a2);
            a3 = fmaf(pc.w[q].w, sdt[b][4 * q + 3], a3);
          }
        } else {
          const float* wr = L.dt_proj_weight + (int64_t)(i % di) * R;
          for (int r = 0; r < R; ++r) a0 = fmaf(__ldg(wr + r), sdt[b][r], a0);
        }
        const float xd = pc.bias + ((a0 + a1) + (a2 + a3));
        const float e = expf(xd);
        const float delta = xd > 20.f ? xd : (xd < -20.f ? e : log1pf(e));
        const float du = delta * uv;
        float* hs = L.ssm_state + (int64_t)i * kN;
        float acc = 0.f;
#pragma unroll
        for (int n = 0; n < kN; ++n) {
          const float hn = fmaf(expf(delta * pc.an[n]), pc.hs[n], du * sB[b][n]);
          hs[n] = hn;
          acc = fmaf(sC[b][n], hn, acc);
        }
        a.ybuf[i] = fmaf(pc.dsk, uv, acc) * (zv / (1.f + expf(-zv)));
      }
    }
    barrier_arrive(a.ctl);
    ++bar;
    PreD pd;
    preload_D(a, L, sw, lane, pd);
    if (!barrier_wait(a.ctl, bar)) return;

    // ---- D: out_proj + residual (mamba_gemv's order)
    for (int i = tid; i < B * di; i += kThreads) dsm[i] = __ldcg(a.ybuf + i);
    __syncthreads();
    for (int j = sw; j < dm; j += n_gw) {
      float acc[kMaxBatch];
      if (j == sw)
        row_dot_pre(pd.w, dsm, di, B, lane, acc);
      else
        row_dot(L.out_proj_weight + (int64_t)j * di, dsm, di, B, lane, acc);
      if (lane < B) {
        float* hp = a.h + (int64_t)lane * dm + j;
        if (j == sw) {  // this warp's row of the residual stream, kept in a register
          hrow = hrow + pick(acc, lane);
          *hp = hrow;
        } else {
          *hp = __ldcg(hp) + pick(acc, lane);
        }
      }
    }
    barrier_arrive(a.ctl);
    ++bar;
    if (l + 1 < a.n_layer) {
      preload_A(a, a.layers[l + 1], sw, n_gw, lane, pa);
    } else if (sw < a.vocab) {
      prefetch_row(a.lm_head + (int64_t)sw * dm, (int64_t)dm * 4, lane);
    }
    if (!barrier_wait(a.ctl, bar)) return;
  }

  // ---- final RMSNorm + tied LM head (mamba_rmsnorm_gemv's order)
  norm_rows_pre(a.h, a.norm_f, dsm, red, B, dm, a.eps);
  for (int j = sw; j < a.vocab; j += 2 * n_gw) {
    // two rows per step, their loads issued together
    PreA::Row2 w2;
    const int j1 = j + n_gw;
#pragma unroll
    for (int i = 0; i < kAI; ++i) {
      const int c = lane * 4 + 128 * i;
      w2.w[0][i] = c < dm ? __ldg(reinterpret_cast<const float4*>(a.lm_head + (int64_t)j * dm + c))
                          : make_float4(0.f, 0.f, 0.f, 0.f);
      w2.w[1][i] = (j1 < a.vocab && c < dm)
                       ? __ldg(reinterpret_cast<const float4*>(a.lm_head + (int64_t)j1 * dm + c))
                       : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float acc[kMaxBatch];
    row_dot_pre(w2.w[0], dsm, dm, B, lane, acc);
    if (lane < B) a.logits[(int64_t)lane * a.vocab + j] = pick(acc, lane);
    if (j1 < a.vocab) {
      row_dot_pre(w2.w[1], dsm, dm, B, lane, acc);
      if (lane < B) a.logits[(int64_t)lane * a.vocab + j1] = pick(acc, lane);
    }
  }
}

// The barrier's give-up path, without any fault: one CTA arrives at barrier
// 2 (count 1 of the 2 it waits for), so its wait cannot complete and gives up
// after limit_ns, recording the timeout.
__global__ void __launch_bounds__(32) barrier_selftest_kernel(unsigned int* ctl, uint64_t limit_ns) {
  barrier_arrive(ctl);
  barrier_wait(ctl, 2, limit_ns);
}

}  // namespace

int read_and_clear_error() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_decode_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_decode_device_error, &zero, sizeof(int));
  }
  return v;
}

}  // namespace mamba_decode

namespace {
int64_t round_up4(int64_t x) { return (x + 3) / 4 * 4; }
}  // namespace

extern "C" {

size_t mamba_decode_scratch_size(int64_t batch, int64_t d_inner, int64_t rank, int64_t dstate) {
  if (batch < 1 || d_inner < 1 || rank < 1 || dstate < 1) return 0;
  // the barrier's control words, then x, z, y [batch][d_inner] and x_proj's outputs
  return 4 * (size_t)mamba_decode::kCtlWords +
         4 * (size_t)(3 * round_up4(batch * d_inner) + round_up4(batch * (rank + 2 * dstate)));
}

int mamba_decode_selftest_barrier_timeout(int64_t limit_ns, void* scratch, size_t scratch_bytes,
                                          void* stream) {
  using mamba_scan::set_last_error;
  namespace md = mamba_decode;
  if (limit_ns <= 0 || limit_ns > 10000000000LL)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "limit_ns must be in (0, 10 s]");
  if (!scratch || scratch_bytes < 4 * (size_t)md::kCtlWords ||
      (reinterpret_cast<uintptr_t>(scratch) & 15u) != 0)
    return set_last_error(MAMBA_SCAN_ERR_WORKSPACE,
                          "decode barrier self-test: scratch of at least 128 aligned bytes");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(scratch, 0, 4 * md::kCtlWords, st);
  if (e == cudaSuccess) {
    md::barrier_selftest_kernel<<<1, 32, 0, st>>>(static_cast<unsigned int*>(scratch),
                                                  (uint64_t)limit_ns);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return set_last_error(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));
  return MAMBA_SCAN_OK;
}

int mamba_decode_step(const mamba_decode_layer* layers, int64_t n_layer, float* h,
                      const float* norm_f_weight, const float* lm_head, float* logits,
                      void* scratch, size_t scratch_bytes, int64_t batch, int64_t d_model,
                      int64_t d_inner, int64_t d_conv, int64_t rank, int64_t dstate,
                      int64_t vocab, float eps, void* stream) {
  using mamba_scan::set_last_error;
  namespace md = mamba_decode;
  if (batch < 1 || batch > md::kMaxBatch || d_model < 4 || d_inner < 4 || n_layer < 0 ||
      d_conv < 1 || d_conv > md::kMaxConv || rank < 1 || rank > md::kMaxRankPre ||
      dstate != md::kN || vocab < 1 || (d_model & 3) != 0 || (d_inner & 3) != 0 ||
      d_model > md::kMaxModel || d_inner > md::kMaxInner || vocab > (1 << 30))
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT,
                          "decode_step: batch 1..4, dstate 16, d_conv 1..4, dt_rank 1..64, "
                          "d_model <= 1024 and d_inner <= 2048, multiples of 4");
  if (!layers || !h || !norm_f_weight || !lm_head || !logits || !scratch)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "decode_step: NULL pointer");
  if (scratch_bytes < mamba_decode_scratch_size(batch, d_inner, rank, dstate) ||
      (reinterpret_cast<uintptr_t>(scratch) & 15u) != 0)
    return set_last_error(MAMBA_SCAN_ERR_WORKSPACE,
                          "decode_step: scratch smaller than mamba_decode_scratch_size() or not "
                          "16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(lm_head) & 15u) != 0)
    return set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "decode_step: lm_head not 16-byte aligned");
  {  // h, logits and scratch are written: pairwise disjoint, and apart from the LM head
    const size_t hb = (size_t)(batch * d_model) * 4, lb = (size_t)(batch * vocab) * 4;
    const size_t eb = (size_t)(vocab * d_model) * 4;
    auto over = [](const void* x, size_t xb, const void* y, size_t yb) {
      const auto x0 = reinterpret_cast<uintptr_t>(x), y0 = reinterpret_cast<uintptr_t>(y);
      return x0 < y0 + yb && y0 < x0 + xb;
    };
    if (over(h, hb, logits, lb) || over(h, hb, scratch, scratch_bytes) ||
        over(logits, lb, scratch, scratch_bytes) || over(lm_head, eb, h, hb) ||
        over(lm_head, eb, logits, lb) || over(lm_head, eb, scratch, scratch_bytes))
      return set_last_error(MAMBA_SCAN_ERR_ALIASING,
                            "decode_step: h, logits, scratch and lm_head must not overlap");
  }
  const size_t smem = sizeof(float) * (size_t)batch * (size_t)(d_model > d_inner ? d_model : d_inner);
  int dev = 0, sms = 0, coop = 0, per_sm = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(md::decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem);
  if (e == cudaSuccess)
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, md::decode_kernel, md::kThreads,
                                                      smem);
  if (e != cudaSuccess) return set_last_error(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));
  if (!coop || per_sm < 1)
    return set_last_error(MAMBA_SCAN_ERR_CUDA, "decode_step: cooperative launch unavailable");

  md::Args a{};
  a.layers = layers;
  a.n_layer = (int)n_layer;
  a.h = h;
  a.norm_f = norm_f_weight;
  a.lm_head = lm_head;
  a.logits = logits;
  a.ctl = static_cast<unsigned int*>(scratch);
  float* f = reinterpret_cast<float*>(scratch) + md::kCtlWords;
  const int64_t nd = round_up4(batch * d_inner);
  a.xbuf = f;
  a.zbuf = f + nd;
  a.ybuf = f + 2 * nd;
  a.xdbl = f + 3 * nd;
  a.batch = (int)batch;
  a.d_model = (int)d_model;
  a.d_inner = (int)d_inner;
  a.width = (int)d_conv;
  a.rank = (int)rank;
  a.vocab = (int)vocab;
  a.eps = eps;

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  e = cudaMemsetAsync(scratch, 0, 4 * md::kCtlWords, st);  // barrier counter, abort flag
  if (e != cudaSuccess) return set_last_error(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)sms);
  cfg.blockDim = dim3(md::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, md::decode_kernel, a);
  if (e != cudaSuccess) return set_last_error(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));
  return MAMBA_SCAN_OK;
}

}  // extern "C"
