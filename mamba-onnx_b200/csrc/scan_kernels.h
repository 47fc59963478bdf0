// Host-visible interface of the selective-scan kernels (internal to the library).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <utility>

namespace mamba_scan {

// Everything a scan kernel reads, besides the TMA descriptors.
struct ScanParams {
  const float* u;
  const float* delta;
  const float* A;
  const float* B;
  const float* C;
  const float* D;
  const float* z;
  const float* delta_bias;
  const float* h0;
  float* out;
  float* h_last;
  // chunk aggregates, [n_tail*32 rows][n_chunks-1][32 floats]: the chunk's end
  // state from zero (16) and its decay (16); the carry kernel then replaces
  // the end state of chunk c with the state entering chunk c+1.
  float* ws;
  int64_t batch;
  int64_t dim;
  int64_t seqlen;
  // Work plan over the B*ceil(D/32) row tiles (32 rows each): row tiles
  // [0, n_full) are scanned in one pass over the whole sequence; row tiles
  // [n_full, n_full + n_tail) are split into n_chunks chunks of chunk_len
  // steps (the last chunk takes the rest) that run in parallel: an aggregate
  // launch over chunks 0..n_chunks-2, the carry kernel, then the emit launch.
  int64_t chunk_len;    // multiple of 32
  int tiles_per_batch;  // ceil(dim / 32)
  int n_full;
  int n_tail;
  int n_chunks;
};

// TMA descriptors: u/delta/z/out as [B][D][L] boxes of 32 rows x 16 steps
// (64-byte swizzle); B/C as [B][L][16] boxes of 16 steps x 16 states.
struct TmaMaps {
  CUtensorMap u, delta, z, out, B, C;
};

enum LaunchMode { kLaunchEmit = 0, kLaunchAggregate = 1 };

// Enqueue one scan kernel (variant 0..3, mode, TMA or plain-load tile path)
// on `stream` with a 1-D grid of `blocks` CTAs: n_full + n_tail * n_chunks
// for emit, n_tail * (n_chunks - 1) for aggregate. `pdl`: programmatic
// dependent launch (the emit pass after the carry kernel).
// exp_mode: how the exact variants form exp (ExpMode of scan_device.cuh:
// 0 SFU, 1 CUDA expf, 2 the reference backend's exp); ignored otherwise.
cudaError_t launch_scan_kernel(int variant, int exp_mode, int mode, bool tma,
                               const ScanParams& p, const TmaMaps& maps, unsigned blocks,
                               cudaStream_t stream, bool pdl);

// Enqueue the carry kernel (between the aggregate and emit passes of a split
// plan), as a programmatic dependent launch.
cudaError_t launch_carry_kernel(const ScanParams& p, cudaStream_t stream);

// One CTA whose mbarrier wait cannot complete and gives up after limit_ns
// (see mamba_scan_selftest_wait_timeout).
cudaError_t launch_wait_selftest(uint64_t limit_ns, cudaStream_t stream);

// Resident CTAs per SM of one kernel instantiation (occupancy calculator).
cudaError_t max_blocks_per_sm(int variant, int exp_mode, int mode, bool tma, int* blocks);

// Record `msg` as the calling thread's mamba_scan_last_error(); returns status.
int set_last_error(int status, const std::string& msg);

// Device error word accessors (see mamba_scan_check_device_error).
cudaError_t read_and_clear_device_error(int* code);

// Enqueue `kernel` on `st` as a programmatic dependent launch: its CTAs may
// be scheduled once every CTA of the previous kernel in the stream has
// started (or called griddepcontrol.launch_dependents), and it must call
// griddepcontrol.wait before touching global memory that the previous
// kernels read or write. The model kernels (mamba_model_ops.h) all do, at
// their top (the GEMM after its shared-memory and TMEM set-up).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace mamba_scan

namespace mamba_decode {
// The persistent decoding kernel's error word (a barrier wait that gave up):
// its code, or -1 when it cannot be read; cleared when set.
int read_and_clear_error();
}  // namespace mamba_decode

namespace mamba_gemm {
// The tensor-core GEMM's own error word (a bounded wait that gave up): its
// code, or -1 when it cannot be read; cleared when set.
int read_and_clear_error();
}  // namespace mamba_gemm
