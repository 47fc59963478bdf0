/*
 * mamba_model_ops.h — kernels of the Mamba block around the selective scan.
 *
 * Not part of the reference's plugin interface: the reference ships only the
 * scan op, and the block that feeds it (its dataflow: benchmarks/profiler.py:
 * 18-150, RMSNorm -> in_proj -> causal depthwise conv1d + SiLU -> x_proj ->
 * dt_proj -> scan -> out_proj) is left to the caller. These entry points serve
 * this package's Mamba model (mamba_onnx/model.py), which uses them on CUDA
 * tensors in place of chains of small torch kernels.
 *
 * Same conventions as mamba_scan.h: DEVICE pointers, fp32, contiguous unless
 * a stride is given, enqueued on `stream` (a cudaStream_t; NULL = the legacy
 * default stream), nothing allocated, a mamba_scan_status returned and
 * mamba_scan_last_error() describing a failure (nothing enqueued then).
 */
#ifndef MAMBA_MODEL_OPS_H_
#define MAMBA_MODEL_OPS_H_

#include <stdint.h>

#include "mamba_scan.h"

#ifdef __cplusplus
extern "C" {
#endif

/*
 * RMSNorm over the last dimension: for each of `rows` rows of `cols` floats,
 * y = x * rsqrt(mean(x^2) + eps) * weight (weight has `cols` entries); y must
 * not overlap x.
 */
MAMBA_SCAN_API int mamba_rmsnorm(const float* x, const float* weight, float* y, int64_t rows,
                                 int64_t cols, float eps, void* stream);

/*
 * Causal depthwise convolution over the sequence, then SiLU:
 *   y[b, d, t] = silu(bias[d] + sum_{k < width} weight[d, k] * x[b, d, t - (width-1) + k])
 * with x taken as 0 before t = 0 (torch's conv1d(groups=dim, padding=width-1)
 * sliced to the first seqlen outputs). x is [batch][dim][seqlen] with rows of
 * seqlen floats and `x_batch_stride` floats between batch entries (so x can be
 * the first half of the in_proj output [batch][2*dim][seqlen]); weight is
 * [dim][width], bias [dim] or NULL, y [batch][dim][seqlen] contiguous and not
 * overlapping x. width: 1..8.
 */
MAMBA_SCAN_API int mamba_causal_conv1d_silu(const float* x, int64_t x_batch_stride,
                                            const float* weight, const float* bias, float* y,
                                            int64_t batch, int64_t dim, int64_t seqlen,
                                            int64_t width, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MAMBA_MODEL_OPS_H_ */
