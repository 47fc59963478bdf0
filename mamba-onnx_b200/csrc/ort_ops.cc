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
// * scratch for the chunked long-sequence path comes from the context's
//   allocator for the output's memory (freed right after the launch; ORT's
//   stream-ordered arena keeps it valid for work already enqueued).
//
// Compiles against the real onnxruntime_c_api.h or the stand-in in csrc/ort.
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "onnxruntime_c_api.h"

#include "../../include/mamba_ops_cuda.h"
#include "../../include/mamba_scan.h"

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

struct ScanKernel {
  const OrtApi* api;
  const OpDesc* desc;
};

const OpDesc* desc_of(const OrtCustomOp* op) { return reinterpret_cast<const ScanOp*>(op)->desc; }

// Runs an ORT call; on failure returns its status from the enclosing function.
#define MAMBA_ORT_TRY(expr)                 \
  do {                                      \
    OrtStatus* mamba_status_ = (expr);      \
    if (mamba_status_) return mamba_status_; \
  } while (0)

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

OrtStatus* compute(const OrtApi& api, const OpDesc& op, OrtKernelContext* ctx) {
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

  // Workspace for the chunked path, from the allocator of the output's memory.
  const size_t ws_bytes = mamba_scan_workspace_size(op.variant, batch, dim, seqlen, dstate);
  OrtAllocator* alloc = nullptr;
  void* ws = nullptr;
  if (ws_bytes > 0) {
    const OrtMemoryInfo* mem = nullptr;
    MAMBA_ORT_TRY(api.GetTensorMemoryInfo(out_v, &mem));
    MAMBA_ORT_TRY(api.KernelContext_GetAllocator(ctx, mem, &alloc));
    ws = alloc->Alloc(alloc, ws_bytes);
    if (ws == nullptr) {
      api.ReleaseAllocator(alloc);
      return api.CreateStatus(ORT_RUNTIME_EXCEPTION, "workspace allocation failed");
    }
  }
  const int rc = mamba_scan_launch(op.variant, &a, ws, ws_bytes, stream);
  if (alloc) {
    alloc->Free(alloc, ws);
    api.ReleaseAllocator(alloc);
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
  *kernel = new ScanKernel{api, desc_of(op)};
  return nullptr;
}

void* ORT_API_CALL create_kernel(const OrtCustomOp* op, const OrtApi* api,
                                 const OrtKernelInfo* info) {
  void* k = nullptr;
  create_kernel_v2(op, api, info, &k);
  return k;
}

OrtStatusPtr ORT_API_CALL kernel_compute_v2(void* kernel, OrtKernelContext* ctx) {
  auto* k = static_cast<ScanKernel*>(kernel);
  return compute(*k->api, *k->desc, ctx);
}

// Entry for hosts without the V2 table slots: the status cannot be returned,
// so it is reported on stderr (never thrown across the C ABI).
void ORT_API_CALL kernel_compute(void* kernel, OrtKernelContext* ctx) {
  auto* k = static_cast<ScanKernel*>(kernel);
  if (OrtStatus* s = compute(*k->api, *k->desc, ctx)) {
    std::fprintf(stderr, "[mamba_ops_cuda] %s\n", k->api->GetErrorMessage(s));
    k->api->ReleaseStatus(s);
  }
}

void ORT_API_CALL kernel_destroy(void* kernel) { delete static_cast<ScanKernel*>(kernel); }

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

void init_ops() {
  for (int i = 0; i < 4; ++i) {
    ScanOp& s = g_ops[i];
    std::memset(&s, 0, sizeof s);
    OrtCustomOp& o = s.base;
    o.version = ORT_API_VERSION;
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

extern "C" OrtStatus* ORT_API_CALL RegisterCustomOps(OrtSessionOptions* options,
                                                     const OrtApiBase* api_base) {
  if (api_base == nullptr) return nullptr;  // nothing to report the error through
  const OrtApi* api = api_base->GetApi(ORT_API_VERSION);
  if (api == nullptr) return nullptr;
  std::call_once(g_ops_once, init_ops);
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
