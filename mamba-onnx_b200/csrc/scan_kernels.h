// Host-visible interface of the selective-scan kernels (internal to the library).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

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
  float* ws;  // chunk aggregates: [B*D][n_chunks-1][32] (16 states, 16 decays)
  int64_t batch;
  int64_t dim;
  int64_t seqlen;
  int64_t chunk_len;    // multiple of 32, or seqlen for a single pass
  int tiles_per_batch;  // ceil(dim / 32)
  int n_chunks;
};

// TMA descriptors: u/delta/z/out as [B][D][L] boxes of 32 rows x 16 steps
// (64-byte swizzle); B/C as [B][L][16] boxes of 16 steps x 16 states.
struct TmaMaps {
  CUtensorMap u, delta, z, out, B, C;
};

enum LaunchMode { kLaunchEmit = 0, kLaunchAggregate = 1 };

// Enqueue one scan kernel (variant 0..3, mode, TMA or plain-load tile path)
// on `stream` with grid (row_tiles, chunks).
cudaError_t launch_scan_kernel(int variant, int mode, bool tma, const ScanParams& p,
                               const TmaMaps& maps, dim3 grid, cudaStream_t stream);

// Device error word accessors (see mamba_scan_check_device_error).
cudaError_t read_and_clear_device_error(int* code);

}  // namespace mamba_scan
