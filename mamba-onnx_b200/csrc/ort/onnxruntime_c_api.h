// onnxruntime_c_api.h for this library: the part of ONNX Runtime's public C
// API that the custom-op layer touches, laid out exactly as ONNX Runtime lays
// it out.
//
// ONNX Runtime's own header is not available in this build environment (the
// reference vendors it as an empty git submodule, vendor/onnxruntime), so this
// file is written from the public API's documented contents:
//
// * OrtApi is a table of function pointers whose slot order is part of ORT's
//   binary interface: entries are only ever appended, one block per API
//   version. Every slot up to the end of ORT_API_VERSION 17 is declared here in
//   that order, under its public name. The entries this library calls carry
//   their real signatures; the others are typed as an opaque OrtApiSlot, which
//   has the size of any function pointer. The end slot of each version's block
//   is checked at compile time in ort_ops.cc (and by tests/test_ort_layout.py)
//   against the fixed counts ORT itself asserts (101 for version 1 ... 275 for
//   version 17).
// * OrtApiBase, OrtAllocator and OrtCustomOp (up to GetEndVersion, the last
//   member of the version-17 table) have ORT's member order; the enums have
//   ORT's values.
//
// A library built against this file therefore binds to an ONNX Runtime whose
// API version is 15 or later (RegisterCustomOps asks for the newest of 17, 16,
// 15 the runtime offers). Building against the real header instead
// (make ORT_INCLUDE_DIR=...) gives the same layout.
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

// Slot type of the OrtApi entries this library does not call.
typedef void (*OrtApiSlot)(void);

typedef struct OrtApi {
  /*   0 */ OrtStatus*(ORT_API_CALL* CreateStatus)(OrtErrorCode code, const char* msg);
  /*   1 */ OrtErrorCode(ORT_API_CALL* GetErrorCode)(const OrtStatus* status);
  /*   2 */ const char*(ORT_API_CALL* GetErrorMessage)(const OrtStatus* status);
  /*   3 */ OrtApiSlot CreateEnv;
  /*   4 */ OrtApiSlot CreateEnvWithCustomLogger;
  /*   5 */ OrtApiSlot EnableTelemetryEvents;
  /*   6 */ OrtApiSlot DisableTelemetryEvents;
  /*   7 */ OrtApiSlot CreateSession;
  /*   8 */ OrtApiSlot CreateSessionFromArray;
  /*   9 */ OrtApiSlot Run;
  /*  10 */ OrtApiSlot CreateSessionOptions;
  /*  11 */ OrtApiSlot SetOptimizedModelFilePath;
  /*  12 */ OrtApiSlot CloneSessionOptions;
  /*  13 */ OrtApiSlot SetSessionExecutionMode;
  /*  14 */ OrtApiSlot EnableProfiling;
  /*  15 */ OrtApiSlot DisableProfiling;
  /*  16 */ OrtApiSlot EnableMemPattern;
  /*  17 */ OrtApiSlot DisableMemPattern;
  /*  18 */ OrtApiSlot EnableCpuMemArena;
  /*  19 */ OrtApiSlot DisableCpuMemArena;
  /*  20 */ OrtApiSlot SetSessionLogId;
  /*  21 */ OrtApiSlot SetSessionLogVerbosityLevel;
  /*  22 */ OrtApiSlot SetSessionLogSeverityLevel;
  /*  23 */ OrtApiSlot SetSessionGraphOptimizationLevel;
  /*  24 */ OrtApiSlot SetIntraOpNumThreads;
  /*  25 */ OrtApiSlot SetInterOpNumThreads;
  /*  26 */ OrtStatusPtr(ORT_API_CALL* CreateCustomOpDomain)(const char* domain, OrtCustomOpDomain** out);
  /*  27 */ OrtStatusPtr(ORT_API_CALL* CustomOpDomain_Add)(OrtCustomOpDomain* custom_op_domain,
                                                              const struct OrtCustomOp* op);
  /*  28 */ OrtStatusPtr(ORT_API_CALL* AddCustomOpDomain)(OrtSessionOptions* options,
                                                             OrtCustomOpDomain* custom_op_domain);
  /*  29 */ OrtApiSlot RegisterCustomOpsLibrary;
  /*  30 */ OrtApiSlot SessionGetInputCount;
  /*  31 */ OrtApiSlot SessionGetOutputCount;
  /*  32 */ OrtApiSlot SessionGetOverridableInitializerCount;
  /*  33 */ OrtApiSlot SessionGetInputTypeInfo;
  /*  34 */ OrtApiSlot SessionGetOutputTypeInfo;
  /*  35 */ OrtApiSlot SessionGetOverridableInitializerTypeInfo;
  /*  36 */ OrtApiSlot SessionGetInputName;
  /*  37 */ OrtApiSlot SessionGetOutputName;
  /*  38 */ OrtApiSlot SessionGetOverridableInitializerName;
  /*  39 */ OrtApiSlot CreateRunOptions;
  /*  40 */ OrtApiSlot RunOptionsSetRunLogVerbosityLevel;
  /*  41 */ OrtApiSlot RunOptionsSetRunLogSeverityLevel;
  /*  42 */ OrtApiSlot RunOptionsSetRunTag;
  /*  43 */ OrtApiSlot RunOptionsGetRunLogVerbosityLevel;
  /*  44 */ OrtApiSlot RunOptionsGetRunLogSeverityLevel;
  /*  45 */ OrtApiSlot RunOptionsGetRunTag;
  /*  46 */ OrtApiSlot RunOptionsSetTerminate;
  /*  47 */ OrtApiSlot RunOptionsUnsetTerminate;
  /*  48 */ OrtApiSlot CreateTensorAsOrtValue;
  /*  49 */ OrtApiSlot CreateTensorWithDataAsOrtValue;
  /*  50 */ OrtApiSlot IsTensor;
  /*  51 */ OrtStatusPtr(ORT_API_CALL* GetTensorMutableData)(OrtValue* value, void** out);
  /*  52 */ OrtApiSlot FillStringTensor;
  /*  53 */ OrtApiSlot GetStringTensorDataLength;
  /*  54 */ OrtApiSlot GetStringTensorContent;
  /*  55 */ OrtApiSlot CastTypeInfoToTensorInfo;
  /*  56 */ OrtApiSlot GetOnnxTypeFromTypeInfo;
  /*  57 */ OrtApiSlot CreateTensorTypeAndShapeInfo;
  /*  58 */ OrtApiSlot SetTensorElementType;
  /*  59 */ OrtApiSlot SetDimensions;
  /*  60 */ OrtStatusPtr(ORT_API_CALL* GetTensorElementType)(const OrtTensorTypeAndShapeInfo* info,
                                                                ONNXTensorElementDataType* out);
  /*  61 */ OrtStatusPtr(ORT_API_CALL* GetDimensionsCount)(const OrtTensorTypeAndShapeInfo* info,
                                                              size_t* out);
  /*  62 */ OrtStatusPtr(ORT_API_CALL* GetDimensions)(const OrtTensorTypeAndShapeInfo* info,
                                                         int64_t* dim_values, size_t dim_values_length);
  /*  63 */ OrtApiSlot GetSymbolicDimensions;
  /*  64 */ OrtApiSlot GetTensorShapeElementCount;
  /*  65 */ OrtStatusPtr(ORT_API_CALL* GetTensorTypeAndShape)(const OrtValue* value,
                                                                 OrtTensorTypeAndShapeInfo** out);
  /*  66 */ OrtApiSlot GetTypeInfo;
  /*  67 */ OrtApiSlot GetValueType;
  /*  68 */ OrtApiSlot CreateMemoryInfo;
  /*  69 */ OrtApiSlot CreateCpuMemoryInfo;
  /*  70 */ OrtApiSlot CompareMemoryInfo;
  /*  71 */ OrtApiSlot MemoryInfoGetName;
  /*  72 */ OrtApiSlot MemoryInfoGetId;
  /*  73 */ OrtApiSlot MemoryInfoGetMemType;
  /*  74 */ OrtApiSlot MemoryInfoGetType;
  /*  75 */ OrtApiSlot AllocatorAlloc;
  /*  76 */ OrtApiSlot AllocatorFree;
  /*  77 */ OrtApiSlot AllocatorGetInfo;
  /*  78 */ OrtApiSlot GetAllocatorWithDefaultOptions;
  /*  79 */ OrtApiSlot AddFreeDimensionOverride;
  /*  80 */ OrtApiSlot GetValue;
  /*  81 */ OrtApiSlot GetValueCount;
  /*  82 */ OrtApiSlot CreateValue;
  /*  83 */ OrtApiSlot CreateOpaqueValue;
  /*  84 */ OrtApiSlot GetOpaqueValue;
  /*  85 */ OrtApiSlot KernelInfoGetAttribute_float;
  /*  86 */ OrtApiSlot KernelInfoGetAttribute_int64;
  /*  87 */ OrtApiSlot KernelInfoGetAttribute_string;
  /*  88 */ OrtStatusPtr(ORT_API_CALL* KernelContext_GetInputCount)(const OrtKernelContext* context,
                                                                       size_t* out);
  /*  89 */ OrtStatusPtr(ORT_API_CALL* KernelContext_GetOutputCount)(const OrtKernelContext* context,
                                                                        size_t* out);
  /*  90 */ OrtStatusPtr(ORT_API_CALL* KernelContext_GetInput)(const OrtKernelContext* context,
                                                                  size_t index, const OrtValue** out);
  /*  91 */ OrtStatusPtr(ORT_API_CALL* KernelContext_GetOutput)(OrtKernelContext* context, size_t index,
                                                                   const int64_t* dim_values,
                                                                   size_t dim_count, OrtValue** out);
  /*  92 */ OrtApiSlot ReleaseEnv;
  /*  93 */ void(ORT_API_CALL* ReleaseStatus)(OrtStatus* input);
  /*  94 */ OrtApiSlot ReleaseMemoryInfo;
  /*  95 */ OrtApiSlot ReleaseSession;
  /*  96 */ OrtApiSlot ReleaseValue;
  /*  97 */ OrtApiSlot ReleaseRunOptions;
  /*  98 */ OrtApiSlot ReleaseTypeInfo;
  /*  99 */ void(ORT_API_CALL* ReleaseTensorTypeAndShapeInfo)(OrtTensorTypeAndShapeInfo* input);
  /* 100 */ OrtApiSlot ReleaseSessionOptions;
  /* 101 */ void(ORT_API_CALL* ReleaseCustomOpDomain)(OrtCustomOpDomain* input);
  /* ---- end of the version 1 entries ---- */
  /* 102 */ OrtApiSlot GetDenotationFromTypeInfo;
  /* 103 */ OrtApiSlot CastTypeInfoToMapTypeInfo;
  /* 104 */ OrtApiSlot CastTypeInfoToSequenceTypeInfo;
  /* 105 */ OrtApiSlot GetMapKeyType;
  /* 106 */ OrtApiSlot GetMapValueType;
  /* 107 */ OrtApiSlot GetSequenceElementType;
  /* 108 */ OrtApiSlot ReleaseMapTypeInfo;
  /* 109 */ OrtApiSlot ReleaseSequenceTypeInfo;
  /* 110 */ OrtApiSlot SessionEndProfiling;
  /* 111 */ OrtApiSlot SessionGetModelMetadata;
  /* 112 */ OrtApiSlot ModelMetadataGetProducerName;
  /* 113 */ OrtApiSlot ModelMetadataGetGraphName;
  /* 114 */ OrtApiSlot ModelMetadataGetDomain;
  /* 115 */ OrtApiSlot ModelMetadataGetDescription;
  /* 116 */ OrtApiSlot ModelMetadataLookupCustomMetadataMap;
  /* 117 */ OrtApiSlot ModelMetadataGetVersion;
  /* 118 */ OrtApiSlot ReleaseModelMetadata;
  /* ---- end of the version 2 entries ---- */
  /* 119 */ OrtApiSlot CreateEnvWithGlobalThreadPools;
  /* 120 */ OrtApiSlot DisablePerSessionThreads;
  /* 121 */ OrtApiSlot CreateThreadingOptions;
  /* 122 */ OrtApiSlot ReleaseThreadingOptions;
  /* 123 */ OrtApiSlot ModelMetadataGetCustomMetadataMapKeys;
  /* 124 */ OrtApiSlot AddFreeDimensionOverrideByName;
  /* ---- end of the version 3 entries ---- */
  /* 125 */ OrtApiSlot GetAvailableProviders;
  /* 126 */ OrtApiSlot ReleaseAvailableProviders;
  /* ---- end of the version 4 entries ---- */
  /* 127 */ OrtApiSlot GetStringTensorElementLength;
  /* 128 */ OrtApiSlot GetStringTensorElement;
  /* 129 */ OrtApiSlot FillStringTensorElement;
  /* 130 */ OrtApiSlot AddSessionConfigEntry;
  /* 131 */ OrtApiSlot CreateAllocator;
  /* 132 */ void(ORT_API_CALL* ReleaseAllocator)(OrtAllocator* input);
  /* 133 */ OrtApiSlot RunWithBinding;
  /* 134 */ OrtApiSlot CreateIoBinding;
  /* 135 */ OrtApiSlot ReleaseIoBinding;
  /* 136 */ OrtApiSlot BindInput;
  /* 137 */ OrtApiSlot BindOutput;
  /* 138 */ OrtApiSlot BindOutputToDevice;
  /* 139 */ OrtApiSlot GetBoundOutputNames;
  /* 140 */ OrtApiSlot GetBoundOutputValues;
  /* 141 */ OrtApiSlot ClearBoundInputs;
  /* 142 */ OrtApiSlot ClearBoundOutputs;
  /* 143 */ OrtApiSlot TensorAt;
  /* 144 */ OrtApiSlot CreateAndRegisterAllocator;
  /* 145 */ OrtApiSlot SetLanguageProjection;
  /* 146 */ OrtApiSlot SessionGetProfilingStartTimeNs;
  /* 147 */ OrtApiSlot SetGlobalIntraOpNumThreads;
  /* 148 */ OrtApiSlot SetGlobalInterOpNumThreads;
  /* 149 */ OrtApiSlot SetGlobalSpinControl;
  /* ---- end of the version 5 entries ---- */
  /* 150 */ OrtApiSlot AddInitializer;
  /* 151 */ OrtApiSlot CreateEnvWithCustomLoggerAndGlobalThreadPools;
  /* 152 */ OrtApiSlot SessionOptionsAppendExecutionProvider_CUDA;
  /* 153 */ OrtApiSlot SessionOptionsAppendExecutionProvider_ROCM;
  /* 154 */ OrtApiSlot SessionOptionsAppendExecutionProvider_OpenVINO;
  /* 155 */ OrtApiSlot SetGlobalDenormalAsZero;
  /* 156 */ OrtApiSlot CreateArenaCfg;
  /* 157 */ OrtApiSlot ReleaseArenaCfg;
  /* ---- end of the version 6 entries ---- */
  /* 158 */ OrtApiSlot ModelMetadataGetGraphDescription;
  /* 159 */ OrtApiSlot SessionOptionsAppendExecutionProvider_TensorRT;
  /* 160 */ OrtApiSlot SetCurrentGpuDeviceId;
  /* 161 */ OrtApiSlot GetCurrentGpuDeviceId;
  /* ---- end of the version 7 entries ---- */
  /* 162 */ OrtApiSlot KernelInfoGetAttributeArray_float;
  /* 163 */ OrtApiSlot KernelInfoGetAttributeArray_int64;
  /* 164 */ OrtApiSlot CreateArenaCfgV2;
  /* 165 */ OrtApiSlot AddRunConfigEntry;
  /* 166 */ OrtApiSlot CreatePrepackedWeightsContainer;
  /* 167 */ OrtApiSlot ReleasePrepackedWeightsContainer;
  /* 168 */ OrtApiSlot CreateSessionWithPrepackedWeightsContainer;
  /* 169 */ OrtApiSlot CreateSessionFromArrayWithPrepackedWeightsContainer;
  /* ---- end of the version 8 entries ---- */
  /* 170 */ OrtApiSlot SessionOptionsAppendExecutionProvider_TensorRT_V2;
  /* 171 */ OrtApiSlot CreateTensorRTProviderOptions;
  /* 172 */ OrtApiSlot UpdateTensorRTProviderOptions;
  /* 173 */ OrtApiSlot GetTensorRTProviderOptionsAsString;
  /* 174 */ OrtApiSlot ReleaseTensorRTProviderOptions;
  /* 175 */ OrtApiSlot EnableOrtCustomOps;
  /* 176 */ OrtApiSlot RegisterAllocator;
  /* 177 */ OrtApiSlot UnregisterAllocator;
  /* 178 */ OrtApiSlot IsSparseTensor;
  /* 179 */ OrtApiSlot CreateSparseTensorAsOrtValue;
  /* 180 */ OrtApiSlot FillSparseTensorCoo;
  /* 181 */ OrtApiSlot FillSparseTensorCsr;
  /* 182 */ OrtApiSlot FillSparseTensorBlockSparse;
  /* 183 */ OrtApiSlot CreateSparseTensorWithValuesAsOrtValue;
  /* 184 */ OrtApiSlot UseCooIndices;
  /* 185 */ OrtApiSlot UseCsrIndices;
  /* 186 */ OrtApiSlot UseBlockSparseIndices;
  /* 187 */ OrtApiSlot GetSparseTensorFormat;
  /* 188 */ OrtApiSlot GetSparseTensorValuesTypeAndShape;
  /* 189 */ OrtApiSlot GetSparseTensorValues;
  /* 190 */ OrtApiSlot GetSparseTensorIndicesTypeShape;
  /* 191 */ OrtApiSlot GetSparseTensorIndices;
  /* ---- end of the version 9 entries ---- */
  /* 192 */ OrtApiSlot HasValue;
  /* 193 */ OrtStatusPtr(ORT_API_CALL* KernelContext_GetGPUComputeStream)(const OrtKernelContext* context,
                                                                             void** out);
  /* 194 */ OrtStatusPtr(ORT_API_CALL* GetTensorMemoryInfo)(const OrtValue* value,
                                                               const OrtMemoryInfo** mem_info);
  /* 195 */ OrtApiSlot GetExecutionProviderApi;
  /* 196 */ OrtApiSlot SessionOptionsSetCustomCreateThreadFn;
  /* 197 */ OrtApiSlot SessionOptionsSetCustomThreadCreationOptions;
  /* 198 */ OrtApiSlot SessionOptionsSetCustomJoinThreadFn;
  /* 199 */ OrtApiSlot SetGlobalCustomCreateThreadFn;
  /* 200 */ OrtApiSlot SetGlobalCustomThreadCreationOptions;
  /* 201 */ OrtApiSlot SetGlobalCustomJoinThreadFn;
  /* 202 */ OrtApiSlot SynchronizeBoundInputs;
  /* 203 */ OrtApiSlot SynchronizeBoundOutputs;
  /* ---- end of the version 10 entries ---- */
  /* 204 */ OrtApiSlot SessionOptionsAppendExecutionProvider_CUDA_V2;
  /* 205 */ OrtApiSlot CreateCUDAProviderOptions;
  /* 206 */ OrtApiSlot UpdateCUDAProviderOptions;
  /* 207 */ OrtApiSlot GetCUDAProviderOptionsAsString;
  /* 208 */ OrtApiSlot ReleaseCUDAProviderOptions;
  /* 209 */ OrtApiSlot SessionOptionsAppendExecutionProvider_MIGraphX;
  /* ---- end of the version 11 entries ---- */
  /* 210 */ OrtApiSlot AddExternalInitializers;
  /* 211 */ OrtApiSlot CreateOpAttr;
  /* 212 */ OrtApiSlot ReleaseOpAttr;
  /* 213 */ OrtApiSlot CreateOp;
  /* 214 */ OrtApiSlot InvokeOp;
  /* 215 */ OrtApiSlot ReleaseOp;
  /* 216 */ OrtApiSlot SessionOptionsAppendExecutionProvider;
  /* 217 */ OrtApiSlot CopyKernelInfo;
  /* 218 */ OrtApiSlot ReleaseKernelInfo;
  /* ---- end of the version 12 entries ---- */
  /* 219 */ OrtApiSlot GetTrainingApi;
  /* 220 */ OrtApiSlot SessionOptionsAppendExecutionProvider_CANN;
  /* 221 */ OrtApiSlot CreateCANNProviderOptions;
  /* 222 */ OrtApiSlot UpdateCANNProviderOptions;
  /* 223 */ OrtApiSlot GetCANNProviderOptionsAsString;
  /* 224 */ OrtApiSlot ReleaseCANNProviderOptions;
  /* ---- end of the version 13 entries ---- */
  /* 225 */ OrtApiSlot MemoryInfoGetDeviceType;
  /* 226 */ OrtApiSlot UpdateEnvWithCustomLogLevel;
  /* 227 */ OrtApiSlot SetGlobalIntraOpThreadAffinity;
  /* 228 */ OrtApiSlot RegisterCustomOpsLibrary_V2;
  /* 229 */ OrtApiSlot RegisterCustomOpsUsingFunction;
  /* 230 */ OrtApiSlot KernelInfo_GetInputCount;
  /* 231 */ OrtApiSlot KernelInfo_GetOutputCount;
  /* 232 */ OrtApiSlot KernelInfo_GetInputName;
  /* 233 */ OrtApiSlot KernelInfo_GetOutputName;
  /* 234 */ OrtApiSlot KernelInfo_GetInputTypeInfo;
  /* 235 */ OrtApiSlot KernelInfo_GetOutputTypeInfo;
  /* 236 */ OrtApiSlot KernelInfoGetAttribute_tensor;
  /* 237 */ OrtApiSlot HasSessionConfigEntry;
  /* 238 */ OrtApiSlot GetSessionConfigEntry;
  /* ---- end of the version 14 entries ---- */
  /* 239 */ OrtApiSlot SessionOptionsAppendExecutionProvider_Dnnl;
  /* 240 */ OrtApiSlot CreateDnnlProviderOptions;
  /* 241 */ OrtApiSlot UpdateDnnlProviderOptions;
  /* 242 */ OrtApiSlot GetDnnlProviderOptionsAsString;
  /* 243 */ OrtApiSlot ReleaseDnnlProviderOptions;
  /* 244 */ OrtApiSlot KernelInfo_GetNodeName;
  /* 245 */ OrtApiSlot KernelInfo_GetLogger;
  /* 246 */ OrtApiSlot KernelContext_GetLogger;
  /* 247 */ OrtApiSlot Logger_LogMessage;
  /* 248 */ OrtApiSlot Logger_GetLoggingSeverityLevel;
  /* 249 */ OrtApiSlot KernelInfoGetConstantInput_tensor;
  /* 250 */ OrtApiSlot CastTypeInfoToOptionalTypeInfo;
  /* 251 */ OrtApiSlot GetOptionalContainedTypeInfo;
  /* 252 */ OrtApiSlot GetResizedStringTensorElementBuffer;
  /* 253 */ OrtStatusPtr(ORT_API_CALL* KernelContext_GetAllocator)(const OrtKernelContext* context,
                                                                      const OrtMemoryInfo* mem_info,
                                                                      OrtAllocator** out);
  /* 254 */ OrtApiSlot GetBuildInfoString;
  /* ---- end of the version 15 entries ---- */
  /* 255 */ OrtApiSlot CreateROCMProviderOptions;
  /* 256 */ OrtApiSlot UpdateROCMProviderOptions;
  /* 257 */ OrtApiSlot GetROCMProviderOptionsAsString;
  /* 258 */ OrtApiSlot ReleaseROCMProviderOptions;
  /* 259 */ OrtApiSlot CreateAndRegisterAllocatorV2;
  /* 260 */ OrtApiSlot RunAsync;
  /* 261 */ OrtApiSlot UpdateTensorRTProviderOptionsWithValue;
  /* 262 */ OrtApiSlot GetTensorRTProviderOptionsByName;
  /* 263 */ OrtApiSlot UpdateCUDAProviderOptionsWithValue;
  /* 264 */ OrtApiSlot GetCUDAProviderOptionsByName;
  /* 265 */ OrtApiSlot KernelContext_GetResource;
  /* ---- end of the version 16 entries ---- */
  /* 266 */ OrtApiSlot SetUserLoggingFunction;
  /* 267 */ OrtApiSlot ShapeInferContext_GetInputCount;
  /* 268 */ OrtApiSlot ShapeInferContext_GetInputTypeShape;
  /* 269 */ OrtApiSlot ShapeInferContext_GetAttribute;
  /* 270 */ OrtApiSlot ShapeInferContext_SetOutputTypeShape;
  /* 271 */ OrtApiSlot SetSymbolicDimensions;
  /* 272 */ OrtApiSlot ReadOpAttr;
  /* 273 */ OrtApiSlot SetDeterministicCompute;
  /* 274 */ OrtApiSlot KernelContext_ParallelFor;
  /* 275 */ OrtApiSlot SessionOptionsAppendExecutionProvider_OpenVINO_V2;
  /* ---- end of the version 17 entries ---- */
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
