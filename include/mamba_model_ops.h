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
 * mamba_rmsnorm whose result goes straight into the operand form of
 * mamba_gemm_tf32x3: hi and lo ([rows][ld], ld >= cols, both multiples of 4;
 * x, weight, hi, lo 16-byte aligned and x, hi, lo not overlapping) receive
 * exactly what mamba_split_tf32 would write for mamba_rmsnorm's y, without y
 * being stored.
 */
MAMBA_SCAN_API int mamba_rmsnorm_split_tf32(const float* x, const float* weight, int64_t rows,
                                            int64_t cols, float eps, float* hi, float* lo,
                                            int64_t ld, void* stream);

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

/*
 * One decoding step of the causal depthwise convolution + SiLU:
 *   state[b, d, :] <- (state[b, d, 1:], x[b, d])   (oldest first)
 *   y[b, d] = silu(bias[d] + sum_k weight[d, k] * state[b, d, k])
 * state [batch][dim][width] is updated in place; x holds the new inputs,
 * dim floats per batch entry `x_batch_stride` floats apart (the x half of a
 * one-token in_proj output [batch][2*dim][1]); weight [dim][width], bias
 * [dim] or NULL, y [batch][dim]. No two of state, x, y may overlap. width: 1..8.
 */
MAMBA_SCAN_API int mamba_causal_conv1d_step(float* state, const float* x, int64_t x_batch_stride,
                                            const float* weight, const float* bias, float* y,
                                            int64_t batch, int64_t dim, int64_t width,
                                            void* stream);

/*
 * RMSNorm followed by a matrix-vector product, for a few tokens (a block's
 * norm and in_proj when decoding):
 *   out[b, j] = sum_c weight[j, c] * x[b, c] * rsqrt(mean(x[b]^2) + eps) * norm_weight[c]
 * x [batch][cols], norm_weight [cols], weight [rows_out][cols] (16-byte
 * aligned), out [batch][rows_out], not overlapping the inputs; cols a
 * multiple of 4, at most 4096.
 */
MAMBA_SCAN_API int mamba_rmsnorm_gemv(const float* x, const float* norm_weight, float eps,
                                      const float* weight, float* out, int64_t batch,
                                      int64_t cols, int64_t rows_out, void* stream);

/*
 * Matrix-vector product with an optional residual, for a few tokens (a
 * block's out_proj when decoding):
 *   out[b, j] = residual[b, j] + sum_c weight[j, c] * x[b, c]
 * x [batch][cols], weight [rows_out][cols] (16-byte aligned), residual and
 * out [batch][rows_out] (residual NULL for none, or out itself); out must
 * not overlap x or weight; cols a multiple of 4, at most 4096.
 */
MAMBA_SCAN_API int mamba_gemv(const float* x, const float* weight, const float* residual,
                              float* out, int64_t batch, int64_t cols, int64_t rows_out,
                              void* stream);

/*
 * One decoding step of a Mamba block's SSM, dt_proj included: for each
 * channel (b, d), with u = u[b, d] (the convolution output) and z = z[b, d]
 * (z_batch_stride floats between batch entries),
 *   delta = softplus(dt_weight[d] . dt[b] + dt_bias[d])
 *   state[b, d, n] = exp(delta A[d, n]) state[b, d, n] + delta u B[b, n]
 *   y[b, d] = (sum_n C[b, n] state[b, d, n] + D[d] u) * silu(z)
 * i.e. SelectiveScanFusedExact over one step with h0 = h_last = state
 * (updated in place) and delta = dt_proj(dt) computed here. dt [batch][rank]
 * (rank <= 256), B and C [batch][dstate], dt_weight [dim][rank], dt_bias
 * [dim] or NULL, A [dim][dstate], D [dim], state [batch][dim][dstate], y
 * [batch][dim]. dstate must be 16; y and state must not overlap the inputs.
 */
MAMBA_SCAN_API int mamba_ssm_decode_step(const float* u, const float* z, int64_t z_batch_stride,
                                         const float* dt, const float* B, const float* C,
                                         const float* dt_weight, const float* dt_bias,
                                         const float* A, const float* D, float* state, float* y,
                                         int64_t batch, int64_t dim, int64_t rank, int64_t dstate,
                                         void* stream);

/*
 * Mamba's x_proj for every token, split into the scan's inputs:
 *   [dt | B | C][b, t, :] = weight . x[b, :, t]
 * x is [batch][dim][seqlen] contiguous (the convolution output, channel
 * rows), weight is x_proj's [rank + 2*dstate][dim]; the first `rank` outputs
 * go to dt [batch][seqlen][rank], the next `dstate` to B and the last
 * `dstate` to C ([batch][seqlen][dstate] each, the scan op's B/C layout).
 * fp32 throughout, deterministic; rank + 2*dstate <= 128. No output may
 * overlap an input or another output. Up to 16 tokens (batch * seqlen, as
 * when decoding) take 4 warps per output; more, a cluster of 8 CTAs per 32
 * tokens splitting dim.
 */
MAMBA_SCAN_API int mamba_x_proj(const float* x, const float* weight, float* dt, float* B, float* C,
                                int64_t batch, int64_t dim, int64_t seqlen, int64_t rank,
                                int64_t dstate, void* stream);

/*
 * mamba_x_proj with Mamba's dt_proj fused behind it (its bias left to the
 * scan op's delta_bias input, which adds it before softplus):
 *   delta[b, d, t] = sum_{k < rank} dt_weight[d, k] * dt[b, t, k]
 * where dt is the first `rank` outputs of x_proj, which are not written out;
 * B and C as mamba_x_proj writes them. x [batch][dim][seqlen], weight
 * [rank + 2*dstate][dim], dt_weight [dim][rank], delta [batch][dim][seqlen]
 * (the scan op's layout), B and C [batch][seqlen][dstate]. rank <= 96 and
 * rank + 2*dstate <= 128; fp32, deterministic (dt summed as mamba_x_proj
 * does, then delta in k order). No output may overlap an input or another
 * output.
 */
MAMBA_SCAN_API int mamba_x_proj_delta(const float* x, const float* weight, const float* dt_weight,
                                      float* delta, float* B, float* C, int64_t batch,
                                      int64_t dim, int64_t seqlen, int64_t rank, int64_t dstate,
                                      void* stream);

/*
 * Mamba's dt_proj for every token, without its bias (the scan op adds it
 * through its delta_bias input before softplus):
 *   delta[b, d, t] = sum_{k < rank} weight[d, k] * dt[b, t, k]
 * dt is x_proj's [batch][seqlen][rank] output, weight dt_proj's [dim][rank],
 * delta [batch][dim][seqlen] (the scan op's layout), not overlapping either
 * input. fp32, summed in k order (deterministic).
 */
MAMBA_SCAN_API int mamba_dt_proj(const float* dt, const float* weight, float* delta,
                                 int64_t batch, int64_t dim, int64_t seqlen, int64_t rank,
                                 void* stream);

/*
 * One Mamba block's weights and decoding state for mamba_decode_step (device
 * pointers; fp32, contiguous): norm_weight [d_model], in_proj_weight
 * [2*d_inner][d_model], conv_weight [d_inner][d_conv], conv_bias [d_inner] or
 * NULL, x_proj_weight [rank + 2*dstate][d_inner], dt_proj_weight
 * [d_inner][rank], dt_proj_bias [d_inner] or NULL, A [d_inner][dstate]
 * (= -exp(A_log)), D [d_inner], out_proj_weight [d_model][d_inner]
 * (in_proj_weight and out_proj_weight 16-byte aligned);
 * conv_state [batch][d_inner][d_conv] (last inputs, oldest first) and
 * ssm_state [batch][d_inner][dstate], both updated in place.
 */
typedef struct mamba_decode_layer {
  const float* norm_weight;
  const float* in_proj_weight;
  const float* conv_weight;
  const float* conv_bias;
  const float* x_proj_weight;
  const float* dt_proj_weight;
  const float* dt_proj_bias;
  const float* A;
  const float* D;
  const float* out_proj_weight;
  float* conv_state;
  float* ssm_state;
} mamba_decode_layer;

/* Bytes of scratch mamba_decode_step needs (0 for a bad shape). */
MAMBA_SCAN_API size_t mamba_decode_scratch_size(int64_t batch, int64_t d_inner, int64_t rank,
                                                int64_t dstate);

/*
 * One decoding step of a whole Mamba model in one persistent kernel:
 * for each of the n_layer blocks (layers: a DEVICE array of n_layer
 * mamba_decode_layer), h += out_proj(SSM step(x_proj(conv step(in_proj(
 * RMSNorm(h)))))) exactly as mamba_rmsnorm_gemv, mamba_causal_conv1d_step,
 * mamba_x_proj, mamba_ssm_decode_step and mamba_gemv compute it (the same
 * values, bit for bit), then logits = lm_head . RMSNorm(h; norm_f_weight).
 * h [batch][d_model] is the residual stream after the embedding (updated in
 * place), lm_head [vocab][d_model] (16-byte aligned), logits [batch][vocab].
 * scratch: mamba_decode_scratch_size() bytes, 16-byte aligned, not
 * overlapping any other argument; its first 128 bytes (the barrier counter) are zeroed on `stream`
 * before the launch. batch 1..4, dstate 16, d_conv 1..8, rank 1..256,
 * d_model and d_inner multiples of 4, batch * max(d_model, d_inner) <= 40960.
 * A cooperative launch of one CTA per SM; its grid-wide barriers give up
 * after 2 s and report MAMBA_SCAN_ERR_DEVICE_TIMEOUT through
 * mamba_scan_check_device_error(). Calls on the same scratch must not
 * overlap on the GPU.
 */
MAMBA_SCAN_API int mamba_decode_step(const mamba_decode_layer* layers, int64_t n_layer, float* h,
                                     const float* norm_f_weight, const float* lm_head,
                                     float* logits, void* scratch, size_t scratch_bytes,
                                     int64_t batch, int64_t d_model, int64_t d_inner,
                                     int64_t d_conv, int64_t rank, int64_t dstate, int64_t vocab,
                                     float eps, void* stream);

/*
 * Self-test of mamba_decode_step's failure detection, without any fault:
 * enqueues one CTA that arrives at a grid barrier which no other CTA joins,
 * so its wait gives up after limit_ns (0 < limit_ns <= 10 s) exactly as a
 * decoding step's barrier gives up after 2 s; a following
 * mamba_scan_check_device_error() returns MAMBA_SCAN_ERR_DEVICE_TIMEOUT and
 * the context stays usable. scratch: at least 128 bytes, 16-byte aligned
 * (its first 128 bytes are zeroed first).
 */
MAMBA_SCAN_API int mamba_decode_selftest_barrier_timeout(int64_t limit_ns, void* scratch,
                                                         size_t scratch_bytes, void* stream);

/*
 * Split fp32 values into two tf32 parts for mamba_gemm_tf32x3:
 *   hi = tf32(x), lo = tf32(x - hi)   (round to nearest; x - hi is exact),
 * written as [rows][cols] with row stride `ld` (>= cols) into hi and lo.
 * transpose = 0: x is [rows][cols] with row stride ldx (>= cols);
 * transpose = 1: x is [cols][rows] with row stride ldx (>= rows), i.e. the
 * output is the split transpose of x. Finite inputs only.
 */
MAMBA_SCAN_API int mamba_split_tf32(const float* x, int64_t rows, int64_t cols, int64_t ldx,
                                    int transpose, float* hi, float* lo, int64_t ld,
                                    void* stream);

/*
 * fp32-accurate GEMM on the tensor cores (3xTF32):
 *   C[m][n] (+)= sum_k A[m][k] * B[n][k]   for m < M, n < N, k < K
 * computed as A_hi B_hi + A_hi B_lo + A_lo B_hi with an fp32 accumulator,
 * from the split operands of mamba_split_tf32: A parts [M][K] with row stride
 * lda, B parts [N][K] with row stride ldb (lda, ldb >= K, multiples of 4; all
 * four parts 16-byte aligned). C element (m, n) lives at c[m*ldc_m + n*ldc_n]
 * (any strides; C must not overlap the operands). c_in = NULL writes the
 * product; otherwise C = C_in + product, C_in laid out with C's strides (it
 * may be C itself, or must not overlap C). K >= 1.
 */
MAMBA_SCAN_API int mamba_gemm_tf32x3(const float* a_hi, const float* a_lo, int64_t lda,
                                     const float* b_hi, const float* b_lo, int64_t ldb,
                                     const float* c_in, float* c, int64_t ldc_m, int64_t ldc_n,
                                     int64_t M, int64_t N, int64_t K, void* stream);

/*
 * Workspace bytes that let mamba_gemm_tf32x3_ws split the K dimension of an
 * M x N x K product across CTAs: nonzero when the output has too few tiles
 * to keep the GPU's SMs busy (e.g. a 768 x 1024 output with K = 1536), 0
 * when the product runs unsplit. Depends on the current device's SM count.
 */
MAMBA_SCAN_API size_t mamba_gemm_tf32x3_workspace_size(int64_t M, int64_t N, int64_t K);

/*
 * mamba_gemm_tf32x3 with a caller-provided device workspace (16-byte
 * aligned, not overlapping the operands, C or C_in; its contents need no
 * initialisation). When mamba_gemm_tf32x3_workspace_size(M, N, K) is
 * nonzero, the product is computed as that many bytes of partial products
 * (K split into ranges), which a second kernel adds in a fixed order, then
 * C_in: the result does not depend on scheduling, and differs from the
 * unsplit product only by the order of the fp32 additions. workspace_bytes
 * below that size -> MAMBA_SCAN_ERR_WORKSPACE; workspace NULL runs unsplit
 * (mamba_gemm_tf32x3). Calls sharing a workspace must be ordered (one
 * stream, or synchronised).
 */
MAMBA_SCAN_API int mamba_gemm_tf32x3_ws(const float* a_hi, const float* a_lo, int64_t lda,
                                        const float* b_hi, const float* b_lo, int64_t ldb,
                                        const float* c_in, float* c, int64_t ldc_m,
                                        int64_t ldc_n, int64_t M, int64_t N, int64_t K,
                                        void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MAMBA_MODEL_OPS_H_ */
