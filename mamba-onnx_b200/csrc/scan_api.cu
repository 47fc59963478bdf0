// C ABI of the selective-scan kernels (include/mamba_scan.h).
//
// Host side of the reference compute entry
// (acmiyaguchi/mamba-onnx src/native/cpp/selective_scan.cc:163-230): argument
// validation, the single-pass / chunked plan, TMA descriptor encoding and the
// launches. Nothing here allocates device memory or synchronises the stream.
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/mamba_scan.h"
#include "scan_kernels.h"

namespace {

using mamba_scan::ScanParams;
using mamba_scan::TmaMaps;

constexpr int kRows = 32;
constexpr int kTile = 16;
constexpr int64_t kMinChunk = 16;  // chunks are multiples of 16 steps (one tile), at least one
constexpr int64_t kMinSplit = 32;  // sequences up to this many steps are never split

thread_local std::string t_last_error;

int fail(int status, const std::string& msg) {
  t_last_error = msg;
  return status;
}

// SM count per device, cached (the plan depends on it).
int sm_count(int device) {
  static std::atomic<int> cache[64];
  if (device < 0 || device >= 64) return 148;
  int v = cache[device].load(std::memory_order_relaxed);
  if (v > 0) return v;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || v <= 0)
    v = 148;
  cache[device].store(v, std::memory_order_relaxed);
  return v;
}

struct Plan {
  int64_t n_full = 0;  // row tiles scanned in one pass
  int64_t n_tail = 0;  // row tiles split into chunks
  int n_chunks = 1;
  int64_t chunk_len = 0;
};

int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

// Plan for a kernel that fits `slots` one-warp CTAs per SM.
//
// A row tile runs fastest with at most two warps on each of the SM's four
// sub-partitions (it is then latency-bound; more warps only share the
// sub-partition's issue slots), and a CTA that ends frees its slot for the
// next one. So the plan thinks in waves of slots x SMs CTAs:
// * fewer row tiles than sub-partitions: every row tile is split into
//   sequence chunks so that row tiles x chunks gives about two warps per
//   sub-partition, within one wave;
// * otherwise full waves of row tiles run in one pass, and a last, partial
//   wave of R row tiles (if small enough) is split into c chunks, about one
//   per sub-partition: the tail then costs an aggregate pass and a chunk
//   pass of ~1/c of a row tile each instead of a whole row tile.
// Chunks are multiples of 16 steps (one tile), so every chunk but the last
// starts and ends on a tile boundary. (Rounding them to 32 instead left the
// Mamba-130m layer, 1x1536x1024, at 16 chunks of 64 steps, 36.1 us per
// FusedExact call, against 22 chunks of 48 steps, 30.0 us.)
Plan make_plan(int64_t batch, int64_t dim, int64_t seqlen, int sms, int slots) {
  Plan pl;
  const int64_t N = batch * ((dim + kRows - 1) / kRows);
  const int64_t subparts = 4LL * sms;
  const int64_t wave = std::max<int64_t>(1, (int64_t)slots * sms);
  pl.n_full = N;
  pl.chunk_len = seqlen;
  if (N <= 0 || seqlen <= kMinSplit) return pl;
  int64_t tail = 0, want = 0;
  if (N < subparts) {
    tail = N;
    want = std::min((2 * subparts + N - 1) / N, std::max<int64_t>(1, wave / N));
  } else {
    tail = N % wave;
    if (N < wave || tail == 0) return pl;
    // about one chunk per sub-partition; below 3 chunks the aggregate pass
    // and the per-chunk start-up cost more than they save
    want = subparts / tail;
    if (want < 3) return pl;
  }
  int64_t len = round_up((seqlen + want - 1) / want, kMinChunk);
  len = std::max<int64_t>(len, kMinChunk);
  const int64_t n = (seqlen + len - 1) / len;
  if (n < 2 || n > 4096) return pl;
  pl.n_full = N - tail;
  pl.n_tail = tail;
  pl.n_chunks = (int)n;
  pl.chunk_len = len;
  return pl;
}

// Resident emit CTAs per SM for a variant and exp mode (cached per device).
int emit_slots(int device, int variant, int exp_mode, bool tma) {
  static std::atomic<int> cache[64][4][3][2];
  if (device < 0 || device >= 64 || variant < 0 || variant > 3 || exp_mode < 0 || exp_mode > 2)
    return 8;
  auto& slot = cache[device][variant][exp_mode][tma ? 1 : 0];
  int v = slot.load(std::memory_order_relaxed);
  if (v > 0) return v;
  if (mamba_scan::max_blocks_per_sm(variant, exp_mode, mamba_scan::kLaunchEmit, tma, &v) !=
          cudaSuccess ||
      v <= 0)
    v = 8;
  slot.store(v, std::memory_order_relaxed);
  return v;
}

// Splits a variant argument into the variant (0..3) and the exp mode of its
// MAMBA_SCAN_EXP_* flag (0 none, 1 IEEE, 2 reference); false if malformed.
bool decode_variant(int code, int* variant, int* exp_mode) {
  const int v = code & 0xff, flags = code & ~0xff;
  if (v < 0 || v > 3) return false;
  int e = 0;
  if (flags == MAMBA_SCAN_EXP_IEEE) e = 1;
  else if (flags == MAMBA_SCAN_EXP_REFERENCE) e = 2;
  else if (flags != 0) return false;
  if (e != 0 && v != MAMBA_SCAN_EXACT && v != MAMBA_SCAN_FUSED_EXACT) return false;
  *variant = v;
  *exp_mode = e;
  return true;
}

size_t workspace_bytes_for(const Plan& pl) {
  if (pl.n_tail == 0 || pl.n_chunks <= 1) return 0;
  return (size_t)pl.n_tail * kRows * (size_t)(pl.n_chunks - 1) * 32 * sizeof(float);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool overlaps(const void* a, size_t abytes, const void* b, size_t bbytes) {
  if (!a || !b || !abytes || !bbytes) return false;
  const auto a0 = reinterpret_cast<uintptr_t>(a), b0 = reinterpret_cast<uintptr_t>(b);
  return a0 < b0 + bbytes && b0 < a0 + abytes;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// [B][D][L] fp32 tensor, boxes of 32 rows x 16 steps, 64-byte swizzle.
bool encode_rows(PFN_cuTensorMapEncodeTiled_v12000 enc, CUtensorMap* m, const float* ptr,
                 int64_t B, int64_t D, int64_t L) {
  const cuuint64_t dims[3] = {(cuuint64_t)L, (cuuint64_t)D, (cuuint64_t)B};
  const cuuint64_t strides[2] = {(cuuint64_t)L * 4, (cuuint64_t)(D * L) * 4};
  const cuuint32_t box[3] = {kTile, kRows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(ptr), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

// [B][L][16] fp32 tensor, boxes of 16 steps x 16 states.
bool encode_bc(PFN_cuTensorMapEncodeTiled_v12000 enc, CUtensorMap* m, const float* ptr, int64_t B,
               int64_t L) {
  const cuuint64_t dims[3] = {16, (cuuint64_t)L, (cuuint64_t)B};
  const cuuint64_t strides[2] = {16 * 4, (cuuint64_t)L * 16 * 4};
  const cuuint32_t box[3] = {16, kTile, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(ptr), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

bool is_fused(int v) { return v == MAMBA_SCAN_FUSED || v == MAMBA_SCAN_FUSED_EXACT; }

}  // namespace

namespace mamba_scan {
int set_last_error(int status, const std::string& msg) { return fail(status, msg); }
}  // namespace mamba_scan

extern "C" {

size_t mamba_scan_workspace_size(int variant_code, int64_t batch, int64_t dim, int64_t seqlen,
                                 int64_t dstate) {
  int variant = 0, exp_mode = 0;
  if (!decode_variant(variant_code, &variant, &exp_mode) || batch <= 0 || dim <= 0 ||
      seqlen <= 0 || dstate != 16)
    return 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
  return workspace_bytes_for(
      make_plan(batch, dim, seqlen, sm_count(dev), emit_slots(dev, variant, exp_mode, true)));
}

int mamba_scan_launch(int variant_code, const mamba_scan_args* a, void* workspace,
                      size_t workspace_bytes, void* stream) {
  t_last_error.clear();
  if (a == nullptr) return fail(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "args is NULL");
  int variant = 0, exp_mode = 0;
  if (!decode_variant(variant_code, &variant, &exp_mode))
    return fail(MAMBA_SCAN_ERR_INVALID_ARGUMENT,
                "variant must be 0..3, with at most one MAMBA_SCAN_EXP_* flag (exact variants "
                "only)");
  if (a->batch < 0 || a->dim < 0 || a->seqlen < 0 || a->dstate < 0)
    return fail(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "negative dimension");
  // selective_scan.cc:228-230 accepts only dstate == 16.
  if (a->dstate != 16)
    return fail(MAMBA_SCAN_ERR_UNSUPPORTED_DSTATE,
                "Only dstate=16 is supported in this kernel (got " + std::to_string(a->dstate) +
                    ")");
  if (a->dim > (int64_t)1 << 31 || a->batch > (int64_t)1 << 31 || a->seqlen > (int64_t)1 << 31 ||
      a->batch * ((a->dim + kRows - 1) / kRows) * 64 > (int64_t)1 << 31)
    return fail(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "dimension exceeds 2^31 (or batch x dim too large)");
  const int64_t B = a->batch, D = a->dim, L = a->seqlen;
  if (B == 0 || D == 0) return MAMBA_SCAN_OK;  // empty output
  if (!a->A || !a->D) return fail(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "A and D must be non-NULL");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t state_bytes = (size_t)B * D * 16 * sizeof(float);
  if (L == 0) {
    // No steps: the final state is the initial one.
    if (a->h_last) {
      const cudaError_t e =
          a->h0 ? cudaMemcpyAsync(a->h_last, a->h0, state_bytes, cudaMemcpyDeviceToDevice, st)
                : cudaMemsetAsync(a->h_last, 0, state_bytes, st);
      if (e != cudaSuccess) return fail(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));
    }
    return MAMBA_SCAN_OK;
  }
  if (!a->u || !a->delta || !a->B || !a->C || !a->out)
    return fail(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "u, delta, B, C and out must be non-NULL");
  if (is_fused(variant) && !a->z)
    return fail(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "the fused variants need z");

  // The output must not alias an input: rows are read and written by
  // different CTAs at different times.
  const size_t big = (size_t)B * D * L * sizeof(float);
  const size_t bc = (size_t)B * L * 16 * sizeof(float);
  const void* ins[] = {a->u, a->delta, is_fused(variant) ? a->z : nullptr, a->B, a->C, a->A,
                       a->D, a->h0};
  const size_t in_bytes[] = {big, big, big, bc, bc, (size_t)D * 64, (size_t)D * 4, state_bytes};
  for (int i = 0; i < 8; ++i) {
    if (overlaps(a->out, big, ins[i], in_bytes[i]))
      return fail(MAMBA_SCAN_ERR_ALIASING, "out overlaps an input");
    if (overlaps(a->h_last, state_bytes, ins[i], in_bytes[i]))
      return fail(MAMBA_SCAN_ERR_ALIASING, "h_last overlaps an input");
  }
  if (overlaps(a->out, big, a->h_last, state_bytes))
    return fail(MAMBA_SCAN_ERR_ALIASING, "h_last overlaps out");
  // The caller's whole workspace region must be disjoint from every tensor:
  // the aggregate pass writes it while the emit pass reads the inputs.
  if (workspace != nullptr && workspace_bytes > 0) {
    if (overlaps(workspace, workspace_bytes, a->out, big))
      return fail(MAMBA_SCAN_ERR_ALIASING, "workspace overlaps out");
    if (overlaps(workspace, workspace_bytes, a->h_last, state_bytes))
      return fail(MAMBA_SCAN_ERR_ALIASING, "workspace overlaps h_last");
    for (int i = 0; i < 8; ++i)
      if (overlaps(workspace, workspace_bytes, ins[i], in_bytes[i]))
        return fail(MAMBA_SCAN_ERR_ALIASING, "workspace overlaps an input");
  }

  ScanParams p{};
  p.u = a->u;
  p.delta = a->delta;
  p.A = a->A;
  p.B = a->B;
  p.C = a->C;
  p.D = a->D;
  p.z = is_fused(variant) ? a->z : nullptr;
  p.delta_bias = is_fused(variant) ? a->delta_bias : nullptr;
  p.h0 = a->h0;
  p.out = a->out;
  p.h_last = a->h_last;
  p.batch = B;
  p.dim = D;
  p.seqlen = L;
  p.tiles_per_batch = (int)((D + kRows - 1) / kRows);

  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));

  // TMA needs 16-byte aligned bases and 16-byte multiple strides (L % 4 == 0).
  TmaMaps maps;
  std::memset(&maps, 0, sizeof maps);
  bool tma = (L % 4 == 0) && aligned16(a->u) && aligned16(a->delta) && aligned16(a->out) &&
             aligned16(a->B) && aligned16(a->C) && (!p.z || aligned16(p.z));
  if (tma) {
    auto enc = encode_fn();
    tma = enc != nullptr && encode_rows(enc, &maps.u, a->u, B, D, L) &&
          encode_rows(enc, &maps.delta, a->delta, B, D, L) &&
          encode_rows(enc, &maps.z, p.z ? p.z : a->u, B, D, L) &&
          encode_rows(enc, &maps.out, a->out, B, D, L) && encode_bc(enc, &maps.B, a->B, B, L) &&
          encode_bc(enc, &maps.C, a->C, B, L);
  }

  // (planned with the TMA kernel's occupancy, as mamba_scan_workspace_size does)
  Plan pl = make_plan(B, D, L, sm_count(dev), emit_slots(dev, variant, exp_mode, true));
  const size_t need = workspace_bytes_for(pl);
  if (need > 0) {
    if (workspace == nullptr) {
      pl = Plan{};  // no workspace: every row tile runs as one pass
      pl.n_full = B * ((D + kRows - 1) / kRows);
      pl.chunk_len = L;
    } else if (workspace_bytes < need) {
      return fail(MAMBA_SCAN_ERR_WORKSPACE, "workspace holds " + std::to_string(workspace_bytes) +
                                                " bytes; this shape needs " +
                                                std::to_string(need));
    } else if (!aligned16(workspace)) {
      return fail(MAMBA_SCAN_ERR_WORKSPACE, "workspace must be 16-byte aligned");
    }
  }

  p.ws = static_cast<float*>(workspace);
  p.chunk_len = pl.chunk_len;
  p.n_full = (int)pl.n_full;
  p.n_tail = (int)pl.n_tail;
  p.n_chunks = pl.n_chunks;
  // Split plan: aggregate pass, carry kernel, emit pass. The last two are
  // programmatic dependent launches, so the emit pass's whole row tiles run
  // alongside the aggregate pass; its chunk CTAs wait for the carry kernel.
  const bool split = pl.n_tail > 0 && pl.n_chunks > 1;
  if (split) {
    e = mamba_scan::launch_scan_kernel(variant, exp_mode, mamba_scan::kLaunchAggregate, tma, p,
                                       maps, (unsigned)(pl.n_tail * (pl.n_chunks - 1)), st,
                                       false);
    if (e != cudaSuccess) return fail(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));
    e = mamba_scan::launch_carry_kernel(p, st);
    if (e != cudaSuccess) return fail(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));
  }
  e = mamba_scan::launch_scan_kernel(variant, exp_mode, mamba_scan::kLaunchEmit, tma, p, maps,
                                     (unsigned)(pl.n_full + pl.n_tail * pl.n_chunks), st, split);
  if (e != cudaSuccess) return fail(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));
  return MAMBA_SCAN_OK;
}

const char* mamba_scan_last_error(void) { return t_last_error.c_str(); }

const char* mamba_scan_status_string(int status) {
  switch (status) {
    case MAMBA_SCAN_OK: return "ok";
    case MAMBA_SCAN_ERR_INVALID_ARGUMENT: return "invalid argument";
    case MAMBA_SCAN_ERR_UNSUPPORTED_DSTATE: return "unsupported dstate";
    case MAMBA_SCAN_ERR_WORKSPACE: return "workspace too small or misaligned";
    case MAMBA_SCAN_ERR_ALIASING: return "output aliases an input";
    case MAMBA_SCAN_ERR_CUDA: return "CUDA error";
    case MAMBA_SCAN_ERR_DEVICE_TIMEOUT: return "device wait timed out";
    default: return "unknown status";
  }
}

int mamba_scan_check_device_error(void) {
  int code = 0;
  const cudaError_t e = mamba_scan::read_and_clear_device_error(&code);
  if (e != cudaSuccess) return fail(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));
  // the model-ops GEMM keeps its own word (same codes)
  const int g = mamba_gemm::read_and_clear_error();
  if (g < 0) return fail(MAMBA_SCAN_ERR_CUDA, "cannot read the GEMM error word");
  // and so does the persistent decoding kernel
  const int dc = mamba_decode::read_and_clear_error();
  if (dc < 0) return fail(MAMBA_SCAN_ERR_CUDA, "cannot read the decode error word");
  return code != 0 ? code : (g != 0 ? g : dc);
}

int mamba_scan_selftest_wait_timeout(int64_t limit_ns, void* stream) {
  t_last_error.clear();
  if (limit_ns <= 0 || limit_ns > 10000000000LL)
    return fail(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "limit_ns must be in (0, 10 s]");
  const cudaError_t e =
      mamba_scan::launch_wait_selftest((uint64_t)limit_ns, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));
  return MAMBA_SCAN_OK;
}

int mamba_scan_abi_version(void) { return MAMBA_SCAN_ABI_VERSION; }

}  // extern "C"
