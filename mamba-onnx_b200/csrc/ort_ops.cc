// ONNX Runtime custom ops over the CUDA selective-scan kernels.
//
// The op table and registration mirror the reference plugin
// (acmiyaguchi/mamba-onnx src/native/cpp/selective_scan.cc:324-422): domain
// "mamba", the same four op names and input counts, float32 tensors, opset
// versions 1..INT_MAX. What differs, by design:
//
// * execution provider "CUDAExecutionProvider" (reference: "CPUExecutionProvider",
//   cc:363): inputs/outputs are device tensors, the kernels run on the EP's
//   compute stream (KernelContext_GetGPUComputeStream), nothing synchronises;
// * the status-returning entries (CreateKernelV2 / KernelComputeV2) report
//   errors as OrtStatus; no exception crosses the C ABI (reference: cc:16-24);
// * shapes, ranks, element types and dstate are validated before any launch;
// * SelectiveScanFused / SelectiveScanFusedExact accept an OPTIONAL 8th input,
//   delta_bias [D], added to delta before softplus; 7-input graphs are unchanged;
// * scratch for the chunked long-sequence path is a per-kernel buffer for
//   each (device, stream) the kernel is run on, taken from the context's
//   allocator for the output's memory the first time it is needed, grown when
//   a larger shape needs more, and returned to that allocator in
//   KernelDestroy. A buffer is only ever used by work on its own stream, so
//   concurrent runs on different streams (ORT's multi-stream execution,
//   several sessions threads) never share scratch, and runs on one stream
//   are ordered by the stream itself; an outgrown buffer is kept until
//   KernelDestroy because work already enqueued may still read it.
//
// Compiles against the real onnxruntime_c_api.h or the one in csrc/ort, which
// has ONNX Runtime's slot order (checked below).
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "onnxruntime_c_api.h"

#include "../../include/mamba_ops_cuda.h"
#include "../../include/mamba_scan.h"

// OrtApi slot indices: the last entry of each API version's block (the
// counts ONNX Runtime asserts for its own table) and every entry called here.
#define MAMBA_ORT_SLOT(member, index)                                             \
  static_assert(offsetof(OrtApi, member) / sizeof(void*) == (index),               \
                "OrtApi::" #member " must be slot " #index " of ONNX Runtime's table")
MAMBA_ORT_SLOT(ReleaseCustomOpDomain, 101);
MAMBA_ORT_SLOT(ReleaseModelMetadata, 118);
MAMBA_ORT_SLOT(AddFreeDimensionOverrideByName, 124);
MAMBA_ORT_SLOT(ReleaseAvailableProviders, 126);
MAMBA_ORT_SLOT(SetGlobalSpinControl, 149);
MAMBA_ORT_SLOT(ReleaseArenaCfg, 157);
MAMBA_ORT_SLOT(GetCurrentGpuDeviceId, 161);
MAMBA_ORT_SLOT(CreateSessionFromArrayWithPrepackedWeightsContainer, 169);
MAMBA_ORT_SLOT(GetSparseTensorIndices, 191);
MAMBA_ORT_SLOT(SynchronizeBoundOutputs, 203);
MAMBA_ORT_SLOT(SessionOptionsAppendExecutionProvider_MIGraphX, 209);
MAMBA_ORT_SLOT(ReleaseKernelInfo, 218);
MAMBA_ORT_SLOT(ReleaseCANNProviderOptions, 224);
MAMBA_ORT_SLOT(GetSessionConfigEntry, 238);
MAMBA_ORT_SLOT(GetBuildInfoString, 254);
MAMBA_ORT_SLOT(KernelContext_GetResource, 265);
MAMBA_ORT_SLOT(SessionOptionsAppendExecutionProvider_OpenVINO_V2, 275);
MAMBA_ORT_SLOT(CreateStatus, 0);
MAMBA_ORT_SLOT(GetErrorCode, 1);
MAMBA_ORT_SLOT(GetErrorMessage, 2);
MAMBA_ORT_SLOT(CreateCustomOpDomain, 26);
MAMBA_ORT_SLOT(CustomOpDomain_Add, 27);
MAMBA_ORT_SLOT(AddCustomOpDomain, 28);
MAMBA_ORT_SLOT(GetTensorMutableData, 51);
MAMBA_ORT_SLOT(GetTensorElementType, 60);
MAMBA_ORT_SLOT(GetDimensionsCount, 61);
MAMBA_ORT_SLOT(GetDimensions, 62);
MAMBA_ORT_SLOT(GetTensorTypeAndShape, 65);
MAMBA_ORT_SLOT(KernelContext_GetInputCount, 88);
MAMBA_ORT_SLOT(KernelContext_GetOutputCount, 89);
MAMBA_ORT_SLOT(KernelContext_GetInput, 90);
MAMBA_ORT_SLOT(KernelContext_GetOutput, 91);
MAMBA_ORT_SLOT(ReleaseStatus, 93);
MAMBA_ORT_SLOT(ReleaseTensorTypeAndShapeInfo, 99);
MAMBA_ORT_SLOT(ReleaseAllocator, 132);
MAMBA_ORT_SLOT(KernelContext_GetGPUComputeStream, 193);
MAMBA_ORT_SLOT(GetTensorMemoryInfo, 194);
MAMBA_ORT_SLOT(KernelContext_GetAllocator, 253);
#undef MAMBA_ORT_SLOT
// OrtCustomOp member order (the table ORT reads, up to version 17).
static_assert(offsetof(OrtCustomOp, CreateKernel) == sizeof(void*), "OrtCustomOp layout");
static_assert(offsetof(OrtCustomOp, KernelCompute) == 8 * sizeof(void*), "OrtCustomOp layout");
static_assert(offsetof(OrtCustomOp, GetInputMemoryType) == 12 * sizeof(void*), "OrtCustomOp layout");
static_assert(offsetof(OrtCustomOp, CreateKernelV2) == 17 * sizeof(void*), "OrtCustomOp layout");
static_assert(offsetof(OrtCustomOp, GetEndVersion) == 21 * sizeof(void*), "OrtCustomOp layout");

namespace {

struct OpDesc {
  const char* name;
  int variant;        // mamba_scan_variant
  size_t n_required;  // reference input count (cc:333, :342, :351, :360)
  size_t n_total;     // including optional inputs
};

constexpr OpDesc kOps[4] = {
    {"SelectiveScan", MAMBA_SCAN_LINEAR, 6, 6},
    {"SelectiveScanExact", MAMBA_SCAN_EXACT, 6, 6},
    {"SelectiveScanFused", MAMBA_SCAN_FUSED, 7, 8},
    {"SelectiveScanFusedExact", MAMBA_SCAN_FUSED_EXACT, 7, 8},
};

// OrtCustomOp first, so an OrtCustomOp* handed back by ORT is a ScanOp*.
struct ScanOp {
  OrtCustomOp base;
  const OpDesc* desc;
};

// Runs an ORT call; on failure returns its status from the enclosing function.
#define MAMBA_ORT_TRY(expr)                 \
  do {                                      \
    OrtStatus* mamba_status_ = (expr);      \
    if (mamba_status_) return mamba_status_; \
  } while (0)

// Scratch of one kernel on one (device, stream).
struct Scratch {
  int device;
  void* stream;
  void* ptr;
  size_t bytes;
};

struct ScanKernel {
  const OrtApi* api;
  const OpDesc* desc;
  std::mutex mu;                 // held from scratch lookup to the end of the launch
  OrtAllocator* alloc = nullptr;  // released in KernelDestroy
  std::vector<Scratch> scratch;
  std::vector<void*> retired;    // outgrown buffers: enqueued work may still read them
};

// The kernel's scratch for (device, stream), at least `bytes` long; taken from
// (or grown through) the context's allocator for the output's memory. Called
// with k.mu held.
OrtStatus* scratch_for(const OrtApi& api, ScanKernel& k, OrtKernelContext* ctx, OrtValue* out_v,
                       int device, void* stream, size_t bytes, void** ptr) {
  Scratch* s = nullptr;
  for (auto& e : k.scratch)
    if (e.device == device && e.stream == stream) s = &e;
  if (s != nullptr && s->bytes >= bytes) {
    *ptr = s->ptr;
    return nullptr;
  }
  if (k.alloc == nullptr) {
    const OrtMemoryInfo* mem = nullptr;
    MAMBA_ORT_TRY(api.GetTensorMemoryInfo(out_v, &mem));
    MAMBA_ORT_TRY(api.KernelContext_GetAllocator(ctx, mem, &k.alloc));
  }
  void* p = k.alloc->Alloc(k.alloc, bytes);
  if (p == nullptr) return api.CreateStatus(ORT_RUNTIME_EXCEPTION, "scan workspace allocation failed");
  if (s != nullptr) {
    k.retired.push_back(s->ptr);
    s->ptr = p;
    s->bytes = bytes;
  } else {
    k.scratch.push_back(Scratch{device, stream, p, bytes});
  }
  *ptr = p;
  return nullptr;
}

const OpDesc* desc_of(const OrtCustomOp* op) { return reinterpret_cast<const ScanOp*>(op)->desc; }

struct TensorView {
  const OrtValue* value = nullptr;
  ONNXTensorElementDataType type = ONNX_TENSOR_ELEMENT_DATA_TYPE_UNDEFINED;
  int64_t dims[4] = {0, 0, 0, 0};
  size_t rank = 0;
  void* data = nullptr;
};

OrtStatus* inspect(const OrtApi& api, const OrtValue* v, TensorView* t) {
  t->value = v;
  OrtTensorTypeAndShapeInfo* info = nullptr;
  MAMBA_ORT_TRY(api.GetTensorTypeAndShape(v, &info));
  OrtStatus* s = api.GetTensorElementType(info, &t->type);
  if (!s) s = api.GetDimensionsCount(info, &t->rank);
  if (!s && t->rank > 4) s = api.CreateStatus(ORT_INVALID_ARGUMENT, "tensor rank above 4");
  if (!s) s = api.GetDimensions(info, t->dims, t->rank);
  api.ReleaseTensorTypeAndShapeInfo(info);
  if (s) return s;
  return api.GetTensorMutableData(const_cast<OrtValue*>(v), &t->data);
}

OrtStatus* invalid(const OrtApi& api, const std::string& op, const std::string& msg) {
  return api.CreateStatus(ORT_INVALID_ARGUMENT, (op + ": " + msg).c_str());
}

std::string shape_str(const TensorView& t) {
  std::string s = "[";
  for (size_t i = 0; i < t.rank; ++i) s += (i ? "," : "") + std::to_string(t.dims[i]);
  return s + "]";
}

OrtStatus* compute(ScanKernel& k, OrtKernelContext* ctx) {
  const OrtApi& api = *k.api;
  const OpDesc& op = *k.desc;
  size_t n_in = 0;
  MAMBA_ORT_TRY(api.KernelContext_GetInputCount(ctx, &n_in));
  if (n_in < op.n_required || n_in > op.n_total)
    return invalid(api, op.name, "expected " + std::to_string(op.n_required) + " inputs, got " +
                                     std::to_string(n_in));
  // Inputs: u, delta, A, B, C, D, [z], [delta_bias] (cc:167-186).
  TensorView in[8];
  for (size_t i = 0; i < n_in; ++i) {
    const OrtValue* v = nullptr;
    MAMBA_ORT_TRY(api.KernelContext_GetInput(ctx, i, &v));
    if (v == nullptr) {
      if (i >= op.n_required) continue;  // optional input left out
      return invalid(api, op.name, "input " + std::to_string(i) + " is missing");
    }
    MAMBA_ORT_TRY(inspect(api, v, &in[i]));
    if (in[i].type != ONNX_TENSOR_ELEMENT_DATA_TYPE_FLOAT)
      return invalid(api, op.name, "input " + std::to_string(i) + " must be float32");
  }
  const TensorView &u = in[0], &dl = in[1], &A = in[2], &Bm = in[3], &Cm = in[4], &Dv = in[5];
  if (u.rank != 3) return invalid(api, op.name, "u must be [batch, dim, seqlen], got " + shape_str(u));
  const int64_t batch = u.dims[0], dim = u.dims[1], seqlen = u.dims[2];
  if (A.rank != 2 || A.dims[0] != dim)
    return invalid(api, op.name, "A must be [dim, dstate], got " + shape_str(A));
  const int64_t dstate = A.dims[1];
  auto same3 = [](const TensorView& t, int64_t a, int64_t b, int64_t c) {
    return t.rank == 3 && t.dims[0] == a && t.dims[1] == b && t.dims[2] == c;
  };
  if (!same3(dl, batch, dim, seqlen))
    return invalid(api, op.name, "delta must match u, got " + shape_str(dl));
  if (!same3(Bm, batch, seqlen, dstate) || !same3(Cm, batch, seqlen, dstate))
    return invalid(api, op.name, "B and C must be [batch, seqlen, dstate]");
  if (Dv.rank != 1 || Dv.dims[0] != dim) return invalid(api, op.name, "D must be [dim]");
  const bool fused = op.variant == MAMBA_SCAN_FUSED || op.variant == MAMBA_SCAN_FUSED_EXACT;
  if (fused && !same3(in[6], batch, dim, seqlen))
    return invalid(api, op.name, "z must match u, got " + shape_str(in[6]));
  const bool has_bias = fused && n_in > 7 && in[7].value != nullptr;
  if (has_bias && (in[7].rank != 1 || in[7].dims[0] != dim))
    return invalid(api, op.name, "delta_bias must be [dim]");
  if (dstate != 16)  // cc:228-230
    return api.CreateStatus(ORT_INVALID_ARGUMENT,
                            (std::string(op.name) + ": Only dstate=16 is supported in this kernel")
                                .c_str());

  // Output [batch, dim, seqlen], allocated by ORT on the device (cc:222-226).
  const int64_t out_shape[3] = {batch, dim, seqlen};
  OrtValue* out_v = nullptr;
  MAMBA_ORT_TRY(api.KernelContext_GetOutput(ctx, 0, out_shape, 3, &out_v));
  void* out = nullptr;
  MAMBA_ORT_TRY(api.GetTensorMutableData(out_v, &out));
  void* stream = nullptr;
  MAMBA_ORT_TRY(api.KernelContext_GetGPUComputeStream(ctx, &stream));

  mamba_scan_args a;
  std::memset(&a, 0, sizeof a);
  a.u = static_cast<const float*>(u.data);
  a.delta = static_cast<const float*>(dl.data);
  a.A = static_cast<const float*>(A.data);
  a.B = static_cast<const float*>(Bm.data);
  a.C = static_cast<const float*>(Cm.data);
  a.D = static_cast<const float*>(Dv.data);
  a.z = fused ? static_cast<const float*>(in[6].data) : nullptr;
  a.delta_bias = has_bias ? static_cast<const float*>(in[7].data) : nullptr;
  a.out = static_cast<float*>(out);
  a.batch = batch;
  a.dim = dim;
  a.seqlen = seqlen;
  a.dstate = dstate;

  // Scratch for the chunked path: this kernel's buffer for (device, stream).
  const size_t ws_bytes = mamba_scan_workspace_size(op.variant, batch, dim, seqlen, dstate);
  int rc = MAMBA_SCAN_OK;
  if (ws_bytes > 0) {
    int device = 0;
    const cudaError_t ce = cudaGetDevice(&device);
    if (ce != cudaSuccess)
      return api.CreateStatus(ORT_RUNTIME_EXCEPTION,
                              (std::string(op.name) + ": " + cudaGetErrorString(ce)).c_str());
    std::lock_guard<std::mutex> lock(k.mu);
    void* ws = nullptr;
    MAMBA_ORT_TRY(scratch_for(api, k, ctx, out_v, device, stream, ws_bytes, &ws));
    rc = mamba_scan_launch(op.variant, &a, ws, ws_bytes, stream);
  } else {
    rc = mamba_scan_launch(op.variant, &a, nullptr, 0, stream);
  }
  if (rc != MAMBA_SCAN_OK) {
    const OrtErrorCode code = (rc == MAMBA_SCAN_ERR_CUDA || rc == MAMBA_SCAN_ERR_DEVICE_TIMEOUT)
                                  ? ORT_RUNTIME_EXCEPTION
                                  : ORT_INVALID_ARGUMENT;
    return api.CreateStatus(code, (std::string(op.name) + ": " + mamba_scan_status_string(rc) +
                                   ": " + mamba_scan_last_error())
                                      .c_str());
  }
  return nullptr;
}

// ---- OrtCustomOp callbacks ----

OrtStatusPtr ORT_API_CALL create_kernel_v2(const OrtCustomOp* op, const OrtApi* api,
                                           const OrtKernelInfo*, void** kernel) {
  auto* k = new ScanKernel;
  k->api = api;
  k->desc = desc_of(op);
  *kernel = k;
  return nullptr;
}

void* ORT_API_CALL create_kernel(const OrtCustomOp* op, const OrtApi* api,
                                 const OrtKernelInfo* info) {
  void* k = nullptr;
  create_kernel_v2(op, api, info, &k);
  return k;
}

OrtStatusPtr ORT_API_CALL kernel_compute_v2(void* kernel, OrtKernelContext* ctx) {
  return compute(*static_cast<ScanKernel*>(kernel), ctx);
}

// Entry for hosts without the V2 table slots: the status cannot be returned,
// so it is reported on stderr (never thrown across the C ABI).
void ORT_API_CALL kernel_compute(void* kernel, OrtKernelContext* ctx) {
  auto* k = static_cast<ScanKernel*>(kernel);
  if (OrtStatus* s = compute(*k, ctx)) {
    std::fprintf(stderr, "[mamba_ops_cuda] %s\n", k->api->GetErrorMessage(s));
    k->api->ReleaseStatus(s);
  }
}

// Returns the kernel's scratch to the allocator it came from, after the work
// on each device that may still read it has finished.
void ORT_API_CALL kernel_destroy(void* kernel) {
  auto* k = static_cast<ScanKernel*>(kernel);
  if (k->alloc != nullptr) {
    int current = 0;
    const bool have_current = cudaGetDevice(&current) == cudaSuccess;
    std::vector<int> synced;
    for (const auto& e : k->scratch) {
      bool seen = false;
      for (int d : synced) seen = seen || d == e.device;
      if (seen) continue;
      synced.push_back(e.device);
      if (cudaSetDevice(e.device) == cudaSuccess) cudaDeviceSynchronize();
    }
    if (have_current) cudaSetDevice(current);
    for (const auto& e : k->scratch) k->alloc->Free(k->alloc, e.ptr);
    for (void* p : k->retired) k->alloc->Free(k->alloc, p);
    k->api->ReleaseAllocator(k->alloc);
  }
  delete k;
}

const char* ORT_API_CALL op_name(const OrtCustomOp* op) { return desc_of(op)->name; }
const char* ORT_API_CALL op_ep(const OrtCustomOp*) { return "CUDAExecutionProvider"; }
size_t ORT_API_CALL op_input_count(const OrtCustomOp* op) { return desc_of(op)->n_total; }
ONNXTensorElementDataType ORT_API_CALL op_input_type(const OrtCustomOp*, size_t) {
  return ONNX_TENSOR_ELEMENT_DATA_TYPE_FLOAT;
}
size_t ORT_API_CALL op_output_count(const OrtCustomOp*) { return 1; }
ONNXTensorElementDataType ORT_API_CALL op_output_type(const OrtCustomOp*, size_t) {
  return ONNX_TENSOR_ELEMENT_DATA_TYPE_FLOAT;
}
OrtCustomOpInputOutputCharacteristic ORT_API_CALL op_input_char(const OrtCustomOp* op, size_t i) {
  return i < desc_of(op)->n_required ? INPUT_OUTPUT_REQUIRED : INPUT_OUTPUT_OPTIONAL;
}
OrtCustomOpInputOutputCharacteristic ORT_API_CALL op_output_char(const OrtCustomOp*, size_t) {
  return INPUT_OUTPUT_REQUIRED;
}
OrtMemType ORT_API_CALL op_input_mem(const OrtCustomOp*, size_t) { return OrtMemTypeDefault; }
int ORT_API_CALL op_start_version(const OrtCustomOp*) { return 1; }
int ORT_API_CALL op_end_version(const OrtCustomOp*) { return 2147483647; }

ScanOp g_ops[4];
std::once_flag g_ops_once;
uint32_t g_ops_version = ORT_API_VERSION;  // the API version the runtime offered

void init_ops() {
  for (int i = 0; i < 4; ++i) {
    ScanOp& s = g_ops[i];
    std::memset(&s, 0, sizeof s);
    OrtCustomOp& o = s.base;
    o.version = g_ops_version;
    o.CreateKernel = create_kernel;
    o.GetName = op_name;
    o.GetExecutionProviderType = op_ep;
    o.GetInputType = op_input_type;
    o.GetInputTypeCount = op_input_count;
    o.GetOutputType = op_output_type;
    o.GetOutputTypeCount = op_output_count;
    o.KernelCompute = kernel_compute;
    o.KernelDestroy = kernel_destroy;
    o.GetInputCharacteristic = op_input_char;
    o.GetOutputCharacteristic = op_output_char;
    o.GetInputMemoryType = op_input_mem;
    o.CreateKernelV2 = create_kernel_v2;
    o.KernelComputeV2 = kernel_compute_v2;
    o.GetStartVersion = op_start_version;
    o.GetEndVersion = op_end_version;
    s.desc = &kOps[i];
  }
}

}  // namespace

// Registers the four ops with the newest OrtApi version (17, 16 or 15) the
// runtime offers; the op tables declare that version, so an older runtime
// reads only the members it knows (before 16: the void KernelCompute entry,
// which reports failures on stderr). Without any usable API (no api_base, or
// a runtime older than 15) nothing can carry a status back: the reason goes
// to stderr and the call returns NULL with no op registered.
extern "C" OrtStatus* ORT_API_CALL RegisterCustomOps(OrtSessionOptions* options,
                                                     const OrtApiBase* api_base) {
  if (api_base == nullptr) {
    std::fprintf(stderr, "[mamba_ops_cuda] RegisterCustomOps: no OrtApiBase; ops not registered\n");
    return nullptr;
  }
  const OrtApi* api = nullptr;
  uint32_t version = ORT_API_VERSION;
  for (; version >= 15 && api == nullptr; --version) api = api_base->GetApi(version);
  ++version;
  if (api == nullptr) {
    std::fprintf(stderr,
                 "[mamba_ops_cuda] RegisterCustomOps: ONNX Runtime %s offers no OrtApi version "
                 "15..%d; ops not registered\n",
                 api_base->GetVersionString ? api_base->GetVersionString() : "?", ORT_API_VERSION);
    return nullptr;
  }
  std::call_once(g_ops_once, [version] {
    g_ops_version = version;
    init_ops();
  });
  OrtCustomOpDomain* domain = nullptr;
  MAMBA_ORT_TRY(api->CreateCustomOpDomain("mamba", &domain));
  for (auto& op : g_ops) {
    if (OrtStatus* s = api->CustomOpDomain_Add(domain, &op.base)) {
      api->ReleaseCustomOpDomain(domain);
      return s;
    }
  }
  // The domain must outlive the sessions built from these options; ORT does
  // not take ownership, so it is intentionally kept for the process lifetime.
  return api->AddCustomOpDomain(options, domain);
}
