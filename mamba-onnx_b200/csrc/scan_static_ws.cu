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
// cudaGetSymbolAddress on every call, with the caller's device current: the
// address belongs to the CUDA context the module is loaded in, which can
// change under the same device index (after cudaDeviceReset, or for a
// driver-API caller that makes another context current), so it is never
// reused from an earlier call. The lookup is a host-side query that allocates
// nothing; the first one on a device also loads the library's kernels there.
#include <cuda_runtime.h>

#include <string>

#include "../../include/mamba_scan.h"
#include "scan_kernels.h"

namespace {

// Chunk aggregates of the calls made through this entry point, shared by all
// of them.
static __device__ __align__(256) unsigned char g_static_workspace[MAMBA_SCAN_STATIC_WORKSPACE_BYTES];

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
  // In host code g_static_workspace only names the variable for the runtime;
  // the address a kernel can use comes from cudaGetSymbolAddress, for the
  // context current now.
  void* ws = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&ws, g_static_workspace);
  if (e != cudaSuccess)
    return mamba_scan::set_last_error(
        MAMBA_SCAN_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
  return mamba_scan_launch(variant, args, ws, MAMBA_SCAN_STATIC_WORKSPACE_BYTES, stream);
}
