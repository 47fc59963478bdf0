/*
 * mamba_scan.h — C ABI of the sm_100a selective-scan kernels.
 *
 * This is the launch boundary under the ONNX Runtime custom ops (and the one a
 * non-ORT caller binds through cgo / JNI / ctypes). It replaces the body of the
 * reference plugin's compute entry,
 *   acmiyaguchi/mamba-onnx src/native/cpp/selective_scan.cc:163-308
 *   (SelectiveScanKernelImpl<UseFused,UseExact>::Compute),
 * and the Zig equivalent, src/native/zig/selective_scan.zig:449-544
 * (computeKernel). Same tensors, same layouts, same four variants; the data
 * lives in device memory and the work is enqueued on a caller's CUDA stream.
 *
 * Plain C: pointers, sizes and ints only. Every pointer in mamba_scan_args is
 * a DEVICE pointer. All calls are asynchronous with respect to the host unless
 * stated; none allocates device memory.
 */
#ifndef MAMBA_SCAN_H_
#define MAMBA_SCAN_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MAMBA_SCAN_ABI_VERSION 2

#if defined(__GNUC__)
#define MAMBA_SCAN_API __attribute__((visibility("default")))
#else
#define MAMBA_SCAN_API
#endif

/* The four ops of the reference (selective_scan.cc:315-318, :332-360). */
typedef enum mamba_scan_variant {
  MAMBA_SCAN_LINEAR = 0,      /* "SelectiveScan":           abar = 1 + delta*A           */
  MAMBA_SCAN_EXACT = 1,       /* "SelectiveScanExact":      abar = exp(delta*A)          */
  MAMBA_SCAN_FUSED = 2,       /* "SelectiveScanFused":      softplus(delta), y*silu(z)   */
  MAMBA_SCAN_FUSED_EXACT = 3  /* "SelectiveScanFusedExact": both                         */
} mamba_scan_variant;

/*
 * Exact variants only: how exp is formed, OR'ed into the variant argument of
 * mamba_scan_launch, mamba_scan_launch_static_workspace and
 * mamba_scan_workspace_size. No flag: abar = exp(delta*A) and the chunk decay
 * on the SFU (ex2.approx, relative error ~2 ulp), softplus/SiLU with CUDA's
 * expf/log1pf.
 *   MAMBA_SCAN_EXP_IEEE       CUDA's expf for abar and the chunk decay too.
 *   MAMBA_SCAN_EXP_REFERENCE  the reference C++ backend's own exp (its
 *     published degree-5 Taylor polynomial times 2^n, selective_scan.cc:33-69;
 *     relative error up to ~8.6e-5) for abar, softplus and SiLU, so that the
 *     output follows that backend's numbers (normwise within ~1e-6 of them)
 *     rather than the exact function (~3e-4 from float64 at the benchmark
 *     distributions). It also keeps that exp's one defect: -inf for
 *     arguments below about -88.03.
 * At most one flag; a flag on a non-exact variant is MAMBA_SCAN_ERR_INVALID_ARGUMENT.
 */
#define MAMBA_SCAN_EXP_IEEE 0x100
#define MAMBA_SCAN_EXP_REFERENCE 0x200

typedef enum mamba_scan_status {
  MAMBA_SCAN_OK = 0,
  MAMBA_SCAN_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad variant, negative size   */
  MAMBA_SCAN_ERR_UNSUPPORTED_DSTATE = 2, /* dstate != 16 (selective_scan.cc:228-230) */
  MAMBA_SCAN_ERR_WORKSPACE = 3,        /* workspace given but smaller than required  */
  MAMBA_SCAN_ERR_ALIASING = 4,         /* out (or h_last) overlaps an input          */
  MAMBA_SCAN_ERR_CUDA = 5,             /* a CUDA runtime/driver call failed          */
  MAMBA_SCAN_ERR_DEVICE_TIMEOUT = 6    /* a kernel's bounded wait gave up            */
} mamba_scan_status;

/*
 * Tensors (fp32, contiguous, row-major; layouts of selective_scan.cc:245-246):
 *   u, delta, z, out : [batch, dim, seqlen]
 *   A                : [dim, dstate]
 *   B, C             : [batch, seqlen, dstate]
 *   D                : [dim]
 * Extensions beyond the reference signature (all optional, NULL = absent):
 *   delta_bias : [dim], added to delta before softplus (fused variants only;
 *                ignored otherwise). The reference has no such input.
 *   h0         : [batch, dim, dstate] initial state (reference: zeros, cc:241).
 *   h_last     : [batch, dim, dstate] receives the state after the last step.
 */
typedef struct mamba_scan_args {
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
  int64_t batch;
  int64_t dim;
  int64_t seqlen;
  int64_t dstate;
} mamba_scan_args;

/*
 * Bytes of device workspace that mamba_scan_launch can use for this shape on
 * the current device (0 when the shape runs as a single pass). A workspace
 * lets short-batch / long-sequence shapes split the sequence into chunks that
 * run in parallel; without one they run as a single pass over the sequence.
 */
MAMBA_SCAN_API size_t mamba_scan_workspace_size(int variant, int64_t batch, int64_t dim, int64_t seqlen,
                                 int64_t dstate);

/*
 * Enqueue one selective scan on `stream` (a cudaStream_t; NULL = the legacy
 * default stream). `workspace` may be NULL (workspace_bytes ignored); when it
 * is not NULL it must hold at least mamba_scan_workspace_size(...) bytes, be
 * 16-byte aligned, and its workspace_bytes must not overlap out, h_last or
 * any input (MAMBA_SCAN_ERR_ALIASING). Returns a mamba_scan_status; on failure nothing was
 * enqueued and mamba_scan_last_error() describes the cause.
 */
MAMBA_SCAN_API int mamba_scan_launch(int variant, const mamba_scan_args* args, void* workspace,
                      size_t workspace_bytes, void* stream);

/*
 * Same as mamba_scan_launch, for callers that cannot allocate device memory
 * (a runtime whose memory planner owns every buffer, a launch path that must
 * not call cudaMalloc, an FFI caller without a device allocator). It takes no
 * workspace: the scratch that long-sequence shapes need comes from an array
 * compiled into the library, MAMBA_SCAN_STATIC_WORKSPACE_BYTES bytes per GPU,
 * held from the moment the library's kernels are loaded on that GPU until the
 * process exits. It allocates nothing and calls no allocating routine.
 *
 * - Shapes that need more scratch than that (see mamba_scan_workspace_size)
 *   are rejected with MAMBA_SCAN_ERR_WORKSPACE; nothing is enqueued.
 * - Every call looks up the array's address in the CUDA context current on
 *   the calling thread (cudaGetSymbolAddress: a host-side query that
 *   allocates nothing), so a context that changes under the same device index
 *   never receives a stale address. The first call on a device also loads the
 *   library's kernels there: make one call before any stream capture.
 * - Every call on a device uses the same array. Calls whose work can overlap
 *   on the GPU (different streams without ordering between them, several
 *   host threads) race on it; order them on one stream. No call depends on
 *   what an earlier call left in the array.
 * The reference has no counterpart: its CPU kernel needs no scratch.
 */
#define MAMBA_SCAN_STATIC_WORKSPACE_BYTES (8u << 20)
MAMBA_SCAN_API int mamba_scan_launch_static_workspace(int variant, const mamba_scan_args* args,
                                                      void* stream);

/* Message for the calling thread's most recent failed call ("" if none). */
MAMBA_SCAN_API const char* mamba_scan_last_error(void);

/* Static name of a status code. */
MAMBA_SCAN_API const char* mamba_scan_status_string(int status);

/*
 * Synchronises the current device, then returns and clears the device-side
 * error words that the kernels (the scan kernels and the model-ops GEMM of
 * mamba_model_ops.h) set when a bounded wait times out (MAMBA_SCAN_OK or
 * MAMBA_SCAN_ERR_DEVICE_TIMEOUT). Diagnostic only.
 */
MAMBA_SCAN_API int mamba_scan_check_device_error(void);

/*
 * Self-test of the device-side failure detection (no counterpart in the
 * reference, which has no device code). Enqueues on `stream` one CTA whose
 * mbarrier wait can never complete (a transaction is announced that no copy
 * delivers) and which gives up after limit_ns nanoseconds (0 < limit_ns <=
 * 10 s), exactly as a scan kernel's tile wait gives up after 2 s. A following
 * mamba_scan_check_device_error() returns MAMBA_SCAN_ERR_DEVICE_TIMEOUT; the
 * context stays usable. Nothing faults and nothing is left in flight.
 * Returns MAMBA_SCAN_OK once enqueued.
 */
MAMBA_SCAN_API int mamba_scan_selftest_wait_timeout(int64_t limit_ns, void* stream);

/* MAMBA_SCAN_ABI_VERSION of the loaded library. */
MAMBA_SCAN_API int mamba_scan_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* MAMBA_SCAN_H_ */
