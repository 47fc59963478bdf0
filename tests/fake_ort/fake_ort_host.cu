// Test harness: a minimal stand-in for ONNX Runtime's CUDA execution provider.
//
// Loads a custom-op library with dlopen, calls its RegisterCustomOps with the
// OrtApi table below (the stand-in layout of mamba-onnx_b200/csrc/ort), and
// runs one op per call the way ORT's CUDA EP would: inputs and the output are
// device buffers owned by the caller, KernelContext_GetGPUComputeStream hands
// out the caller's stream, and KernelContext_GetAllocator returns a device
// allocator. A test can make the next call of a named OrtApi entry fail, to
// check that the plugin returns that status instead of launching.
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "onnxruntime_c_api.h"

namespace {

struct HostStatus {
  OrtErrorCode code;
  std::string msg;
};

struct HostValue {
  void* data = nullptr;
  std::vector<int64_t> dims;
  ONNXTensorElementDataType type = ONNX_TENSOR_ELEMENT_DATA_TYPE_FLOAT;
};

struct HostContext {
  std::vector<HostValue*> inputs;  // nullptr = optional input left out
  HostValue out;
  std::vector<int64_t> out_expected;
  void* stream = nullptr;
};

struct Domain {
  std::vector<const OrtCustomOp*> ops;
};

struct Library {
  void* handle = nullptr;
  std::vector<const OrtCustomOp*> ops;
};

std::vector<Library> g_libs;
std::string g_fail_next;  // name of the OrtApi entry whose next call fails
int g_alloc_live = 0;     // outstanding allocator blocks
char g_meminfo_tag;       // address used as the device OrtMemoryInfo

OrtStatus* make_status(OrtErrorCode c, const char* m) {
  return reinterpret_cast<OrtStatus*>(new HostStatus{c, m ? m : ""});
}
bool injected(const char* name) {
  if (g_fail_next == name) {
    g_fail_next.clear();
    return true;
  }
  return false;
}
#define FAKE_INJECT(name)                                                        \
  if (injected(name)) return make_status(ORT_FAIL, "injected failure in " name);

OrtErrorCode status_code(const OrtStatus* s) { return reinterpret_cast<const HostStatus*>(s)->code; }
const char* status_msg(const OrtStatus* s) { return reinterpret_cast<const HostStatus*>(s)->msg.c_str(); }
void release_status(OrtStatus* s) { delete reinterpret_cast<HostStatus*>(s); }

OrtStatusPtr create_domain(const char* name, OrtCustomOpDomain** out) {
  FAKE_INJECT("CreateCustomOpDomain");
  if (std::strcmp(name, "mamba") != 0) return make_status(ORT_INVALID_ARGUMENT, "domain name");
  *out = reinterpret_cast<OrtCustomOpDomain*>(new Domain);
  return nullptr;
}
OrtStatusPtr domain_add(OrtCustomOpDomain* d, const OrtCustomOp* op) {
  FAKE_INJECT("CustomOpDomain_Add");
  reinterpret_cast<Domain*>(d)->ops.push_back(op);
  return nullptr;
}
OrtStatusPtr add_domain(OrtSessionOptions* opts, OrtCustomOpDomain* d) {
  FAKE_INJECT("AddCustomOpDomain");
  auto* lib = reinterpret_cast<Library*>(opts);
  lib->ops = reinterpret_cast<Domain*>(d)->ops;
  return nullptr;
}
void release_domain(OrtCustomOpDomain* d) { delete reinterpret_cast<Domain*>(d); }

OrtStatusPtr get_input_count(const OrtKernelContext* c, size_t* out) {
  FAKE_INJECT("KernelContext_GetInputCount");
  *out = reinterpret_cast<const HostContext*>(c)->inputs.size();
  return nullptr;
}
OrtStatusPtr get_output_count(const OrtKernelContext*, size_t* out) {
  *out = 1;
  return nullptr;
}
OrtStatusPtr get_input(const OrtKernelContext* c, size_t i, const OrtValue** out) {
  FAKE_INJECT("KernelContext_GetInput");
  auto* ctx = reinterpret_cast<const HostContext*>(c);
  if (i >= ctx->inputs.size()) return make_status(ORT_INVALID_ARGUMENT, "input index");
  *out = reinterpret_cast<const OrtValue*>(ctx->inputs[i]);
  return nullptr;
}
OrtStatusPtr get_output(OrtKernelContext* c, size_t i, const int64_t* dims, size_t n,
                        OrtValue** out) {
  FAKE_INJECT("KernelContext_GetOutput");
  auto* ctx = reinterpret_cast<HostContext*>(c);
  if (i != 0) return make_status(ORT_INVALID_ARGUMENT, "output index");
  if (std::vector<int64_t>(dims, dims + n) != ctx->out_expected)
    return make_status(ORT_INVALID_ARGUMENT, "output shape differs from the host's buffer");
  ctx->out.dims = ctx->out_expected;
  *out = reinterpret_cast<OrtValue*>(&ctx->out);
  return nullptr;
}
OrtStatusPtr get_stream(const OrtKernelContext* c, void** out) {
  FAKE_INJECT("KernelContext_GetGPUComputeStream");
  *out = reinterpret_cast<const HostContext*>(c)->stream;
  return nullptr;
}

void* ORT_API_CALL dev_alloc(OrtAllocator*, size_t n) {
  void* p = nullptr;
  if (cudaMalloc(&p, n) != cudaSuccess) return nullptr;
  ++g_alloc_live;
  return p;
}
void ORT_API_CALL dev_free(OrtAllocator*, void* p) {
  if (!p) return;
  cudaFree(p);  // synchronising: work already enqueued on the block finishes first
  --g_alloc_live;
}
const OrtMemoryInfo* ORT_API_CALL dev_info(const OrtAllocator*) {
  return reinterpret_cast<const OrtMemoryInfo*>(&g_meminfo_tag);
}
OrtAllocator g_allocator = {1, dev_alloc, dev_free, dev_info};

OrtStatusPtr get_allocator(const OrtKernelContext*, const OrtMemoryInfo* mi, OrtAllocator** out) {
  FAKE_INJECT("KernelContext_GetAllocator");
  if (mi != reinterpret_cast<const OrtMemoryInfo*>(&g_meminfo_tag))
    return make_status(ORT_INVALID_ARGUMENT, "unknown memory info");
  *out = &g_allocator;
  return nullptr;
}
void release_allocator(OrtAllocator*) {}
OrtStatusPtr get_data(OrtValue* v, void** out) {
  FAKE_INJECT("GetTensorMutableData");
  *out = reinterpret_cast<HostValue*>(v)->data;
  return nullptr;
}
OrtStatusPtr get_meminfo(const OrtValue*, const OrtMemoryInfo** out) {
  *out = reinterpret_cast<const OrtMemoryInfo*>(&g_meminfo_tag);
  return nullptr;
}
OrtStatusPtr get_type_shape(const OrtValue* v, OrtTensorTypeAndShapeInfo** out) {
  FAKE_INJECT("GetTensorTypeAndShape");
  *out = reinterpret_cast<OrtTensorTypeAndShapeInfo*>(const_cast<OrtValue*>(v));
  return nullptr;
}
OrtStatusPtr get_elem_type(const OrtTensorTypeAndShapeInfo* i, ONNXTensorElementDataType* out) {
  *out = reinterpret_cast<const HostValue*>(i)->type;
  return nullptr;
}
OrtStatusPtr get_dim_count(const OrtTensorTypeAndShapeInfo* i, size_t* out) {
  *out = reinterpret_cast<const HostValue*>(i)->dims.size();
  return nullptr;
}
OrtStatusPtr get_dims(const OrtTensorTypeAndShapeInfo* i, int64_t* d, size_t n) {
  auto* v = reinterpret_cast<const HostValue*>(i);
  for (size_t k = 0; k < n; ++k) d[k] = k < v->dims.size() ? v->dims[k] : 0;
  return nullptr;
}
void release_type_shape(OrtTensorTypeAndShapeInfo*) {}

OrtApi make_api() {
  OrtApi a;
  std::memset(&a, 0, sizeof a);
  a.CreateStatus = make_status;
  a.GetErrorCode = status_code;
  a.GetErrorMessage = status_msg;
  a.ReleaseStatus = release_status;
  a.CreateCustomOpDomain = create_domain;
  a.CustomOpDomain_Add = domain_add;
  a.AddCustomOpDomain = add_domain;
  a.ReleaseCustomOpDomain = release_domain;
  a.KernelContext_GetInputCount = get_input_count;
  a.KernelContext_GetOutputCount = get_output_count;
  a.KernelContext_GetInput = get_input;
  a.KernelContext_GetOutput = get_output;
  a.KernelContext_GetGPUComputeStream = get_stream;
  a.KernelContext_GetAllocator = get_allocator;
  a.ReleaseAllocator = release_allocator;
  a.GetTensorMutableData = get_data;
  a.GetTensorMemoryInfo = get_meminfo;
  a.GetTensorTypeAndShape = get_type_shape;
  a.GetTensorElementType = get_elem_type;
  a.GetDimensionsCount = get_dim_count;
  a.GetDimensions = get_dims;
  a.ReleaseTensorTypeAndShapeInfo = release_type_shape;
  return a;
}
// Filled by member name: the layout is ONNX Runtime's (unused slots stay NULL).
const OrtApi kApi = make_api();
const OrtApi* get_api(uint32_t) { return &kApi; }
const char* version_string() { return "fake-cuda-ep"; }
const OrtApiBase kBase = {get_api, version_string};

void set_err(char* err, size_t n, const std::string& m) {
  if (err && n) std::snprintf(err, n, "%s", m.c_str());
}

const OrtCustomOp* find_op(int lib, const char* name) {
  if (lib < 0 || lib >= (int)g_libs.size()) return nullptr;
  for (auto* op : g_libs[lib].ops)
    if (std::strcmp(op->GetName(op), name) == 0) return op;
  return nullptr;
}

}  // namespace

extern "C" {

// dlopen `path`, run its RegisterCustomOps; returns a library handle >= 0, or
// -1 with the reason in err (including the status RegisterCustomOps returned).
int fake_ort_load(const char* path, char* err, size_t err_len) {
  void* h = dlopen(path, RTLD_NOW | RTLD_LOCAL);
  if (!h) {
    set_err(err, err_len, dlerror());
    return -1;
  }
  using RegFn = OrtStatus* (*)(OrtSessionOptions*, const OrtApiBase*);
  auto reg = reinterpret_cast<RegFn>(dlsym(h, "RegisterCustomOps"));
  if (!reg) {
    set_err(err, err_len, "RegisterCustomOps not exported");
    return -1;
  }
  g_libs.push_back(Library{h, {}});
  Library& lib = g_libs.back();
  if (OrtStatus* s = reg(reinterpret_cast<OrtSessionOptions*>(&lib), &kBase)) {
    set_err(err, err_len, status_msg(s));
    release_status(s);
    g_libs.pop_back();
    return -1;
  }
  return (int)g_libs.size() - 1;
}

int fake_ort_op_count(int lib) {
  return (lib >= 0 && lib < (int)g_libs.size()) ? (int)g_libs[lib].ops.size() : -1;
}

// Describe op i: name, EP, input count, output count, version range, whether
// the V2 entries are present, and input characteristics (one char per input:
// 'R' required, 'O' optional).
int fake_ort_op_info(int lib, int i, char* name, size_t name_len, char* ep, size_t ep_len,
                     int* n_in, int* n_out, int* v_start, int* v_end, int* has_v2, char* chars,
                     size_t chars_len) {
  if (lib < 0 || lib >= (int)g_libs.size() || i < 0 || i >= (int)g_libs[lib].ops.size())
    return -1;
  const OrtCustomOp* op = g_libs[lib].ops[i];
  set_err(name, name_len, op->GetName(op));
  set_err(ep, ep_len, op->GetExecutionProviderType(op));
  *n_in = (int)op->GetInputTypeCount(op);
  *n_out = (int)op->GetOutputTypeCount(op);
  *v_start = op->GetStartVersion(op);
  *v_end = op->GetEndVersion(op);
  *has_v2 = (op->CreateKernelV2 && op->KernelComputeV2) ? 1 : 0;
  std::string c;
  for (int k = 0; k < *n_in; ++k)
    c += op->GetInputCharacteristic(op, k) == INPUT_OUTPUT_REQUIRED ? 'R' : 'O';
  set_err(chars, chars_len, c);
  return 0;
}

// Make the next call of the named OrtApi entry return an ORT_FAIL status.
void fake_ort_fail_next(const char* api_name) { g_fail_next = api_name ? api_name : ""; }

int fake_ort_live_allocations(void) { return g_alloc_live; }

// A kernel created once and run any number of times, as ORT keeps one kernel
// object per graph node for the life of a session.
struct HostKernel {
  const OrtCustomOp* op = nullptr;
  void* kernel = nullptr;
  bool v2 = false;
};
std::vector<HostKernel*> g_kernels;

// Create a kernel of op `name`; returns a handle >= 0, or -1 (reason in err).
int fake_ort_kernel_create(int lib, const char* name, int use_v2, char* err, size_t err_len) {
  const OrtCustomOp* op = find_op(lib, name);
  if (!op) {
    set_err(err, err_len, std::string("no op named ") + name);
    return -1;
  }
  auto* hk = new HostKernel;
  hk->op = op;
  hk->v2 = use_v2 && op->CreateKernelV2 && op->KernelComputeV2;
  if (hk->v2) {
    if (OrtStatus* s = op->CreateKernelV2(op, &kApi, nullptr, &hk->kernel)) {
      set_err(err, err_len, status_msg(s));
      release_status(s);
      delete hk;
      return -1;
    }
  } else {
    hk->kernel = op->CreateKernel(op, &kApi, nullptr);
  }
  g_kernels.push_back(hk);
  return (int)g_kernels.size() - 1;
}

// Run kernel `handle` once (see fake_ort_run for the arguments).
int fake_ort_kernel_run(int handle, int n_inputs, void* const* ptrs, const int64_t* dims,
                        const int* ranks, const int* types, void* out, const int64_t* out_dims,
                        int out_rank, void* stream, char* err, size_t err_len) {
  if (handle < 0 || handle >= (int)g_kernels.size() || g_kernels[handle] == nullptr) {
    set_err(err, err_len, "bad kernel handle");
    return ORT_INVALID_ARGUMENT;
  }
  HostKernel* hk = g_kernels[handle];
  std::vector<HostValue> vals(n_inputs);
  HostContext ctx;
  const int64_t* dp = dims;
  for (int i = 0; i < n_inputs; ++i) {
    vals[i].data = ptrs[i];
    vals[i].dims.assign(dp, dp + ranks[i]);
    vals[i].type = static_cast<ONNXTensorElementDataType>(types[i]);
    dp += ranks[i];
    ctx.inputs.push_back(ptrs[i] ? &vals[i] : nullptr);
  }
  ctx.out.data = out;
  ctx.out_expected.assign(out_dims, out_dims + out_rank);
  ctx.stream = stream;
  auto* kctx = reinterpret_cast<OrtKernelContext*>(&ctx);
  int rc = 0;
  if (hk->v2) {
    if (OrtStatus* s = hk->op->KernelComputeV2(hk->kernel, kctx)) {
      set_err(err, err_len, status_msg(s));
      rc = status_code(s);
      release_status(s);
    }
  } else {
    hk->op->KernelCompute(hk->kernel, kctx);
  }
  return rc;
}

void fake_ort_kernel_destroy(int handle) {
  if (handle < 0 || handle >= (int)g_kernels.size() || g_kernels[handle] == nullptr) return;
  g_kernels[handle]->op->KernelDestroy(g_kernels[handle]->kernel);
  delete g_kernels[handle];
  g_kernels[handle] = nullptr;
}

// Run op `name` of library `lib` once with a kernel of its own (created and
// destroyed around the call). ptrs[i] == NULL marks an omitted optional
// input. dims holds the inputs' dims back to back (ranks[i] each); types[i]
// is the ONNX element type. Returns 0 or the OrtErrorCode of the status the
// op returned (message in err). use_v2 = 0 runs the void KernelCompute entry.
int fake_ort_run(int lib, const char* name, int n_inputs, void* const* ptrs,
                 const int64_t* dims, const int* ranks, const int* types, void* out,
                 const int64_t* out_dims, int out_rank, void* stream, int use_v2, char* err,
                 size_t err_len) {
  const int h = fake_ort_kernel_create(lib, name, use_v2, err, err_len);
  if (h < 0) {
    return find_op(lib, name) ? ORT_FAIL : ORT_NOT_IMPLEMENTED;
  }
  const int rc = fake_ort_kernel_run(h, n_inputs, ptrs, dims, ranks, types, out, out_dims,
                                     out_rank, stream, err, err_len);
  fake_ort_kernel_destroy(h);
  return rc;
}

}  // extern "C"
