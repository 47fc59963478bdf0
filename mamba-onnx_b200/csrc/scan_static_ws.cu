// mamba_scan_launch_static_workspace: the selective scan without any device
// allocation, for callers that cannot allocate.
//
// Some hosts cannot hand this library scratch memory: an inference runtime
// whose memory planner owns every device buffer, an embedding that must not
// call cudaMalloc on its launch path (cudaMalloc synchronises the device and
// can fail under memory pressure), or an FFI caller with no device allocator
// at all. mamba_scan_launch needs a workspace only when it splits long
// sequences into chunks; this entry point supplies that workspace from a
// fixed array compiled into the library instead of asking the caller for one.
//
// The array is a file-scope __device__ variable: every GPU on which the
// library's kernels are loaded holds its own copy, MAMBA_SCAN_STATIC_WORKSPACE_BYTES
// bytes, until the process exits. Its device address is looked up with
// cudaGetSymbolAddress once per device, on the first call made with that
// device current.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/mamba_scan.h"
#include "scan_kernels.h"

namespace {

// Chunk aggregates of the calls made through this entry point, shared by all
// of them.
static __device__ __align__(256) unsigned char g_static_workspace[MAMBA_SCAN_STATIC_WORKSPACE_BYTES];

constexpr int kMaxDevices = 64;

// Device address of g_static_workspace on `device` (the current device).
// In host code the name g_static_workspace is only a handle for the runtime;
// the address a kernel can use comes from cudaGetSymbolAddress.
cudaError_t static_workspace_address(int device, void** out) {
  static std::mutex mu;
  static void* addr[kMaxDevices] = {};
  std::lock_guard<std::mutex> lock(mu);
  if (addr[device] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_static_workspace);
    if (e != cudaSuccess) return e;
    addr[device] = p;
  }
  *out = addr[device];
  return cudaSuccess;
}

}  // namespace

extern "C" int mamba_scan_launch_static_workspace(int variant, const mamba_scan_args* args,
                                                  void* stream) {
  if (args == nullptr)
    return mamba_scan::set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "args is NULL");
  const size_t need =
      mamba_scan_workspace_size(variant, args->batch, args->dim, args->seqlen, args->dstate);
  if (need > MAMBA_SCAN_STATIC_WORKSPACE_BYTES)
    return mamba_scan::set_last_error(
        MAMBA_SCAN_ERR_WORKSPACE,
        "this shape needs " + std::to_string(need) + " bytes of workspace; the built-in workspace " +
            "holds " + std::to_string((size_t)MAMBA_SCAN_STATIC_WORKSPACE_BYTES) +
            " (use mamba_scan_launch with a caller-provided workspace)");
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess)
    return mamba_scan::set_last_error(MAMBA_SCAN_ERR_CUDA, cudaGetErrorString(e));
  if (device < 0 || device >= kMaxDevices)
    return mamba_scan::set_last_error(MAMBA_SCAN_ERR_INVALID_ARGUMENT, "device index above 63");
  void* ws = nullptr;
  e = static_workspace_address(device, &ws);
  if (e != cudaSuccess)
    return mamba_scan::set_last_error(
        MAMBA_SCAN_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
  return mamba_scan_launch(variant, args, ws, MAMBA_SCAN_STATIC_WORKSPACE_BYTES, stream);
}
