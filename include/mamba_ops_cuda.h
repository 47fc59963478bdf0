/*
 * mamba_ops_cuda.h — ONNX Runtime plugin entry of libmamba_ops_cuda.so.
 *
 * Replaces the reference plugin's library entry,
 *   acmiyaguchi/mamba-onnx src/native/cpp/selective_scan.cc:401-422
 *   (RegisterCustomOps; Zig: src/native/zig/selective_scan.zig:631-652),
 * which ONNX Runtime calls after SessionOptions.register_custom_ops_library(path)
 * (src/mamba_onnx/__init__.py:106). Registers domain "mamba" with the ops
 * SelectiveScan, SelectiveScanExact (6 inputs), SelectiveScanFused and
 * SelectiveScanFusedExact (7 inputs, plus an optional 8th input delta_bias [D]),
 * for the CUDAExecutionProvider: inputs and the output are device tensors and
 * the work runs on the provider's compute stream.
 *
 * Unlike the reference (which returns NULL on every failure, cc:414-419, and
 * throws C++ exceptions through the C ABI, cc:16-24), failures come back as
 * OrtStatus objects.
 */
#ifndef MAMBA_OPS_CUDA_H_
#define MAMBA_OPS_CUDA_H_

#ifdef __cplusplus
extern "C" {
#endif

struct OrtStatus;
struct OrtSessionOptions;
struct OrtApiBase;

#if defined(__GNUC__)
__attribute__((visibility("default")))
#endif
struct OrtStatus* RegisterCustomOps(struct OrtSessionOptions* options,
                                    const struct OrtApiBase* api);

#ifdef __cplusplus
}
#endif

#endif /* MAMBA_OPS_CUDA_H_ */
