// ORACLE HARNESS — test infrastructure, never shipped.
//
// A minimal CPU host that plays the part of ONNX Runtime for the REFERENCE's
// own C++ plugin (acmiyaguchi/mamba-onnx src/native/cpp/selective_scan.cc,
// compiled unmodified next to this file by oracle/Makefile into
// oracle/_ref/libref_scan.so). It implements the handful of OrtApi entries
// the plugin calls (selective_scan.cc:168-226 and :401-422) over caller-owned
// host buffers, registers the plugin's four ops through its exported
// RegisterCustomOps, and runs one op per call through the plugin's own
// CreateKernel / KernelCompute / KernelDestroy entries — the same path ORT's
// CPU execution provider takes (selective_scan.cc:324-360).
//
// Exposed to Python through ctypes:
//   ref_scan_run(...)  — run one op; returns 0, or <0 with a message in err.
//   ref_scan_op_count() / ref_scan_op_name(i) — the ops the plugin registered.
#include <omp.h>

#include <cstdio>
#include <cstring>
#include <exception>
#include <string>
#include <vector>

#include "onnxruntime_c_api.h"

extern "C" OrtStatus* RegisterCustomOps(OrtSessionOptions* options, const OrtApiBase* api);

namespace {

struct HostStatus {
  OrtErrorCode code;
  std::string msg;
};

struct HostValue {
  void* data = nullptr;
  std::vector<int64_t> dims;
};

struct HostContext {
  std::vector<const HostValue*> inputs;
  HostValue out;
  float* out_buf = nullptr;
  std::vector<int64_t> expected_out;
  std::string error;
};

std::vector<const OrtCustomOp*> g_ops;

OrtStatus* make_status(OrtErrorCode c, const char* m) {
  return reinterpret_cast<OrtStatus*>(new HostStatus{c, m ? m : ""});
}
OrtErrorCode status_code(const OrtStatus* s) {
  return reinterpret_cast<const HostStatus*>(s)->code;
}
const char* status_msg(const OrtStatus* s) {
  return reinterpret_cast<const HostStatus*>(s)->msg.c_str();
}
void release_status(OrtStatus* s) { delete reinterpret_cast<HostStatus*>(s); }

OrtStatusPtr create_domain(const char*, OrtCustomOpDomain** out) {
  *out = reinterpret_cast<OrtCustomOpDomain*>(&g_ops);
  return nullptr;
}
OrtStatusPtr domain_add(OrtCustomOpDomain*, const OrtCustomOp* op) {
  g_ops.push_back(op);
  return nullptr;
}
OrtStatusPtr add_domain(OrtSessionOptions*, OrtCustomOpDomain*) { return nullptr; }
void release_domain(OrtCustomOpDomain*) {}

OrtStatusPtr get_input_count(const OrtKernelContext* c, size_t* out) {
  *out = reinterpret_cast<const HostContext*>(c)->inputs.size();
  return nullptr;
}
OrtStatusPtr get_output_count(const OrtKernelContext*, size_t* out) {
  *out = 1;
  return nullptr;
}
OrtStatusPtr get_input(const OrtKernelContext* c, size_t i, const OrtValue** out) {
  auto* ctx = reinterpret_cast<const HostContext*>(c);
  if (i >= ctx->inputs.size()) return make_status(ORT_INVALID_ARGUMENT, "input index");
  *out = reinterpret_cast<const OrtValue*>(ctx->inputs[i]);
  return nullptr;
}
OrtStatusPtr get_output(OrtKernelContext* c, size_t i, const int64_t* dims, size_t n,
                        OrtValue** out) {
  auto* ctx = reinterpret_cast<HostContext*>(c);
  if (i != 0) return make_status(ORT_INVALID_ARGUMENT, "output index");
  std::vector<int64_t> d(dims, dims + n);
  if (d != ctx->expected_out) return make_status(ORT_INVALID_ARGUMENT, "output shape");
  ctx->out.dims = d;
  ctx->out.data = ctx->out_buf;
  *out = reinterpret_cast<OrtValue*>(&ctx->out);
  return nullptr;
}
OrtStatusPtr get_stream(const OrtKernelContext*, void** out) {
  *out = nullptr;
  return nullptr;
}
OrtStatusPtr get_allocator(const OrtKernelContext*, const OrtMemoryInfo*, OrtAllocator**) {
  return make_status(ORT_NOT_IMPLEMENTED, "no allocator in the CPU oracle host");
}
void release_allocator(OrtAllocator*) {}
OrtStatusPtr get_data(OrtValue* v, void** out) {
  *out = reinterpret_cast<HostValue*>(v)->data;
  return nullptr;
}
OrtStatusPtr get_meminfo(const OrtValue*, const OrtMemoryInfo** out) {
  *out = nullptr;
  return nullptr;
}
OrtStatusPtr get_type_shape(const OrtValue* v, OrtTensorTypeAndShapeInfo** out) {
  *out = reinterpret_cast<OrtTensorTypeAndShapeInfo*>(const_cast<OrtValue*>(v));
  return nullptr;
}
OrtStatusPtr get_elem_type(const OrtTensorTypeAndShapeInfo*, ONNXTensorElementDataType* out) {
  *out = ONNX_TENSOR_ELEMENT_DATA_TYPE_FLOAT;
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
const char* version_string() { return "oracle-host"; }
const OrtApiBase kBase = {get_api, version_string};

bool ensure_registered() {
  if (!g_ops.empty()) return true;
  RegisterCustomOps(nullptr, &kBase);
  return !g_ops.empty();
}

}  // namespace

extern "C" int ref_scan_op_count() { return ensure_registered() ? (int)g_ops.size() : 0; }

extern "C" const char* ref_scan_op_name(int i) {
  if (!ensure_registered() || i < 0 || i >= (int)g_ops.size()) return nullptr;
  return g_ops[i]->GetName(g_ops[i]);
}

extern "C" int ref_scan_run(const char* op_name, const float* u, const float* delta,
                            const float* A, const float* B, const float* C, const float* D,
                            const float* z, float* out, int64_t batch, int64_t dim,
                            int64_t seqlen, int64_t dstate, int n_threads, char* err,
                            size_t err_len) {
  auto fail = [&](int code, const std::string& m) {
    if (err && err_len) std::snprintf(err, err_len, "%s", m.c_str());
    return code;
  };
  if (!ensure_registered()) return fail(-1, "RegisterCustomOps registered nothing");
  const OrtCustomOp* op = nullptr;
  for (auto* o : g_ops)
    if (std::strcmp(o->GetName(o), op_name) == 0) op = o;
  if (!op) return fail(-1, std::string("no op named ") + op_name);
  if (n_threads > 0) omp_set_num_threads(n_threads);

  HostValue vu{(void*)u, {batch, dim, seqlen}}, vd{(void*)delta, {batch, dim, seqlen}};
  HostValue vA{(void*)A, {dim, dstate}}, vB{(void*)B, {batch, seqlen, dstate}};
  HostValue vC{(void*)C, {batch, seqlen, dstate}}, vD{(void*)D, {dim}};
  HostValue vz{(void*)z, {batch, dim, seqlen}};
  HostContext ctx;
  ctx.inputs = {&vu, &vd, &vA, &vB, &vC, &vD};
  if (op->GetInputTypeCount(op) == 7) ctx.inputs.push_back(&vz);
  ctx.out_buf = out;
  ctx.expected_out = {batch, dim, seqlen};

  void* kernel = op->CreateKernel(op, &kApi, nullptr);
  int rc = 0;
  try {
    op->KernelCompute(kernel, reinterpret_cast<OrtKernelContext*>(&ctx));
  } catch (const std::exception& e) {
    rc = fail(-2, e.what());
  }
  op->KernelDestroy(kernel);
  return rc;
}
