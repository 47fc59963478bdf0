// Self-written stand-in for onnxruntime_c_api.h.
//
// ONNX Runtime's C API header is not available in this build environment (the
// reference vendors it as an empty git submodule, vendor/onnxruntime). This file
// declares ONLY the names the custom-op layer uses, with the argument lists of
// the public ORT C API, so that the same ort_ops.cc compiles unchanged against
// either this file or the real header.
//
// The struct LAYOUTS below are NOT ONNX Runtime's: OrtApi here is a short table
// in our own order. A library built against this file works only with a host
// that was built against this file too (the test harnesses in this repository).
// A library for a real ONNX Runtime must be built against the real header
// (build flag ORT_INCLUDE_DIR), which defines the real OrtApi and OrtCustomOp.
#pragma once
#include <stddef.h>
#include <stdint.h>

#define MAMBA_ORT_STANDIN_HEADER 1

#ifdef __cplusplus
extern "C" {
#endif

#define ORT_API_CALL
#define ORT_API_VERSION 17

typedef struct OrtStatus OrtStatus;
typedef OrtStatus* OrtStatusPtr;
typedef struct OrtKernelContext OrtKernelContext;
typedef struct OrtKernelInfo OrtKernelInfo;
typedef struct OrtValue OrtValue;
typedef struct OrtTensorTypeAndShapeInfo OrtTensorTypeAndShapeInfo;
typedef struct OrtSessionOptions OrtSessionOptions;
typedef struct OrtCustomOpDomain OrtCustomOpDomain;
typedef struct OrtMemoryInfo OrtMemoryInfo;
typedef struct OrtShapeInferContext OrtShapeInferContext;

typedef enum OrtErrorCode {
  ORT_OK = 0,
  ORT_FAIL = 1,
  ORT_INVALID_ARGUMENT = 2,
  ORT_NO_SUCHFILE = 3,
  ORT_NO_MODEL = 4,
  ORT_ENGINE_ERROR = 5,
  ORT_RUNTIME_EXCEPTION = 6,
  ORT_INVALID_PROTOBUF = 7,
  ORT_MODEL_LOADED = 8,
  ORT_NOT_IMPLEMENTED = 9,
  ORT_INVALID_GRAPH = 10,
  ORT_EP_FAIL = 11,
} OrtErrorCode;

typedef enum ONNXTensorElementDataType {
  ONNX_TENSOR_ELEMENT_DATA_TYPE_UNDEFINED = 0,
  ONNX_TENSOR_ELEMENT_DATA_TYPE_FLOAT = 1,
  ONNX_TENSOR_ELEMENT_DATA_TYPE_UINT8 = 2,
  ONNX_TENSOR_ELEMENT_DATA_TYPE_INT8 = 3,
  ONNX_TENSOR_ELEMENT_DATA_TYPE_UINT16 = 4,
  ONNX_TENSOR_ELEMENT_DATA_TYPE_INT16 = 5,
  ONNX_TENSOR_ELEMENT_DATA_TYPE_INT32 = 6,
  ONNX_TENSOR_ELEMENT_DATA_TYPE_INT64 = 7,
  ONNX_TENSOR_ELEMENT_DATA_TYPE_STRING = 8,
  ONNX_TENSOR_ELEMENT_DATA_TYPE_BOOL = 9,
  ONNX_TENSOR_ELEMENT_DATA_TYPE_FLOAT16 = 10,
  ONNX_TENSOR_ELEMENT_DATA_TYPE_DOUBLE = 11,
} ONNXTensorElementDataType;

typedef enum OrtCustomOpInputOutputCharacteristic {
  INPUT_OUTPUT_REQUIRED = 0,
  INPUT_OUTPUT_OPTIONAL,
  INPUT_OUTPUT_VARIADIC,
} OrtCustomOpInputOutputCharacteristic;

typedef enum OrtMemType {
  OrtMemTypeCPUInput = -2,
  OrtMemTypeCPUOutput = -1,
  OrtMemTypeCPU = OrtMemTypeCPUOutput,
  OrtMemTypeDefault = 0,
} OrtMemType;

typedef struct OrtAllocator {
  uint32_t version;
  void*(ORT_API_CALL* Alloc)(struct OrtAllocator* this_, size_t size);
  void(ORT_API_CALL* Free)(struct OrtAllocator* this_, void* p);
  const OrtMemoryInfo*(ORT_API_CALL* Info)(const struct OrtAllocator* this_);
} OrtAllocator;

struct OrtCustomOp;

typedef struct OrtApi {
  OrtStatus*(ORT_API_CALL* CreateStatus)(OrtErrorCode code, const char* msg);
  OrtErrorCode(ORT_API_CALL* GetErrorCode)(const OrtStatus* status);
  const char*(ORT_API_CALL* GetErrorMessage)(const OrtStatus* status);
  void(ORT_API_CALL* ReleaseStatus)(OrtStatus* input);

  OrtStatusPtr(ORT_API_CALL* CreateCustomOpDomain)(const char* domain, OrtCustomOpDomain** out);
  OrtStatusPtr(ORT_API_CALL* CustomOpDomain_Add)(OrtCustomOpDomain* custom_op_domain,
                                                  const struct OrtCustomOp* op);
  OrtStatusPtr(ORT_API_CALL* AddCustomOpDomain)(OrtSessionOptions* options,
                                                 OrtCustomOpDomain* custom_op_domain);
  void(ORT_API_CALL* ReleaseCustomOpDomain)(OrtCustomOpDomain* input);

  OrtStatusPtr(ORT_API_CALL* KernelContext_GetInputCount)(const OrtKernelContext* context,
                                                           size_t* out);
  OrtStatusPtr(ORT_API_CALL* KernelContext_GetOutputCount)(const OrtKernelContext* context,
                                                            size_t* out);
  OrtStatusPtr(ORT_API_CALL* KernelContext_GetInput)(const OrtKernelContext* context,
                                                      size_t index, const OrtValue** out);
  OrtStatusPtr(ORT_API_CALL* KernelContext_GetOutput)(OrtKernelContext* context, size_t index,
                                                       const int64_t* dim_values,
                                                       size_t dim_count, OrtValue** out);
  OrtStatusPtr(ORT_API_CALL* KernelContext_GetGPUComputeStream)(const OrtKernelContext* context,
                                                                 void** out);
  OrtStatusPtr(ORT_API_CALL* KernelContext_GetAllocator)(const OrtKernelContext* context,
                                                          const OrtMemoryInfo* mem_info,
                                                          OrtAllocator** out);
  void(ORT_API_CALL* ReleaseAllocator)(OrtAllocator* input);

  OrtStatusPtr(ORT_API_CALL* GetTensorMutableData)(OrtValue* value, void** out);
  OrtStatusPtr(ORT_API_CALL* GetTensorMemoryInfo)(const OrtValue* value,
                                                   const OrtMemoryInfo** mem_info);
  OrtStatusPtr(ORT_API_CALL* GetTensorTypeAndShape)(const OrtValue* value,
                                                     OrtTensorTypeAndShapeInfo** out);
  OrtStatusPtr(ORT_API_CALL* GetTensorElementType)(const OrtTensorTypeAndShapeInfo* info,
                                                    ONNXTensorElementDataType* out);
  OrtStatusPtr(ORT_API_CALL* GetDimensionsCount)(const OrtTensorTypeAndShapeInfo* info,
                                                  size_t* out);
  OrtStatusPtr(ORT_API_CALL* GetDimensions)(const OrtTensorTypeAndShapeInfo* info,
                                             int64_t* dim_values, size_t dim_values_length);
  void(ORT_API_CALL* ReleaseTensorTypeAndShapeInfo)(OrtTensorTypeAndShapeInfo* input);
} OrtApi;

typedef struct OrtApiBase {
  const OrtApi*(ORT_API_CALL* GetApi)(uint32_t version);
  const char*(ORT_API_CALL* GetVersionString)(void);
} OrtApiBase;

// Field names and signatures follow the public OrtCustomOp (the V2 entries,
// which return a status instead of throwing, exist in ORT 1.16 and later).
typedef struct OrtCustomOp {
  uint32_t version;
  void*(ORT_API_CALL* CreateKernel)(const struct OrtCustomOp* op, const OrtApi* api,
                                    const OrtKernelInfo* info);
  const char*(ORT_API_CALL* GetName)(const struct OrtCustomOp* op);
  const char*(ORT_API_CALL* GetExecutionProviderType)(const struct OrtCustomOp* op);
  ONNXTensorElementDataType(ORT_API_CALL* GetInputType)(const struct OrtCustomOp* op,
                                                         size_t index);
  size_t(ORT_API_CALL* GetInputTypeCount)(const struct OrtCustomOp* op);
  ONNXTensorElementDataType(ORT_API_CALL* GetOutputType)(const struct OrtCustomOp* op,
                                                          size_t index);
  size_t(ORT_API_CALL* GetOutputTypeCount)(const struct OrtCustomOp* op);
  void(ORT_API_CALL* KernelCompute)(void* op_kernel, OrtKernelContext* context);
  void(ORT_API_CALL* KernelDestroy)(void* op_kernel);
  OrtCustomOpInputOutputCharacteristic(ORT_API_CALL* GetInputCharacteristic)(
      const struct OrtCustomOp* op, size_t index);
  OrtCustomOpInputOutputCharacteristic(ORT_API_CALL* GetOutputCharacteristic)(
      const struct OrtCustomOp* op, size_t index);
  OrtMemType(ORT_API_CALL* GetInputMemoryType)(const struct OrtCustomOp* op, size_t index);
  int(ORT_API_CALL* GetVariadicInputMinArity)(const struct OrtCustomOp* op);
  int(ORT_API_CALL* GetVariadicInputHomogeneity)(const struct OrtCustomOp* op);
  int(ORT_API_CALL* GetVariadicOutputMinArity)(const struct OrtCustomOp* op);
  int(ORT_API_CALL* GetVariadicOutputHomogeneity)(const struct OrtCustomOp* op);
  OrtStatusPtr(ORT_API_CALL* CreateKernelV2)(const struct OrtCustomOp* op, const OrtApi* api,
                                             const OrtKernelInfo* info, void** kernel);
  OrtStatusPtr(ORT_API_CALL* KernelComputeV2)(void* op_kernel, OrtKernelContext* context);
  OrtStatusPtr(ORT_API_CALL* InferOutputShapeFn)(const struct OrtCustomOp* op,
                                                 OrtShapeInferContext* ctx);
  int(ORT_API_CALL* GetStartVersion)(const struct OrtCustomOp* op);
  int(ORT_API_CALL* GetEndVersion)(const struct OrtCustomOp* op);
} OrtCustomOp;

#ifdef __cplusplus
}
#endif
