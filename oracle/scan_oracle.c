/*
 * ORACLE — CPU restatement of the reference selective scan.
 *
 * This file is TEST INFRASTRUCTURE. It is the checker that the CUDA path is
 * compared against; it is never linked into, called by, or shipped with the
 * product library. Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg may load it.
 *
 * Two restatements of the reference algorithm
 * (acmiyaguchi/mamba-onnx, src/native/cpp/selective_scan.cc, "cc" below):
 *
 *   oracle_scan_f64   — float64 ground truth of the op's mathematics, as the
 *                       reference's own test oracle states it
 *                       (tests/test_ops.py:17-63, reference_selective_scan):
 *                         delta' = Fused ? softplus(delta) : delta
 *                         Abar   = Exact ? exp(delta'*A) : 1 + delta'*A
 *                         h      = Abar*h + delta'*B*u          (h starts at 0)
 *                         y      = sum_n C*h + D*u
 *                         y      = Fused ? y*silu(z) : y
 *                       Any dstate is accepted. Optional extensions (not in
 *                       the reference): a per-channel delta_bias added before
 *                       softplus, an initial state h0 and a final-state
 *                       output, used to check the chunked-carry kernels.
 *
 *   oracle_scan_f32ref — float32 restatement of the reference C++ numerics
 *                       (cc:157-309): the Taylor-5 fast_exp with its 2^n
 *                       exponent-bit construction (cc:33-69), fast_softplus
 *                       (cc:137-143), fast_silu (cc:145-148), the linear
 *                       update order h += delta*(A*h + B*u) (cc:277-282), the
 *                       exact update h = Abar*h + (delta*B)*u (cc:265-274),
 *                       and the sequential 16-lane horizontal sum
 *                       (cc:288-296). dstate must be 16, like the reference
 *                       (cc:228-230). Used to pin this restatement against
 *                       the compiled reference (oracle/_ref).
 *
 * Layouts (cc:245-246, tests/test_ops.py:22-28): u, delta, z, out [B,D,L]
 * (L fastest); B, C [B,L,N]; A [D,N]; D [D].
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

enum { ORACLE_LINEAR = 0, ORACLE_EXACT = 1, ORACLE_FUSED = 2, ORACLE_FUSED_EXACT = 3 };

static int is_fused(int v) { return v == ORACLE_FUSED || v == ORACLE_FUSED_EXACT; }
static int is_exact(int v) { return v == ORACLE_EXACT || v == ORACLE_FUSED_EXACT; }

/* torch.nn.functional.softplus(x) with beta=1, threshold=20
 * (tests/test_ops.py:42): x if x > 20 else log1p(exp(x)). */
static double softplus_f64(double x) { return x > 20.0 ? x : log1p(exp(x)); }

/* torch.nn.functional.silu (tests/test_ops.py:59): x * sigmoid(x). */
static double silu_f64(double x) { return x / (1.0 + exp(-x)); }

/*
 * Float64 ground truth over a list of rows.
 *   rows       — row indices r = b*dim + d to compute (NULL = all B*D rows)
 *   n_rows     — number of entries in rows (ignored when rows is NULL)
 *   out        — [n_rows][seqlen] (or [B*D][seqlen] when rows is NULL)
 *   delta_bias — optional [D], added to delta before softplus (Fused only)
 *   h0         — optional [B*D][N] initial state (NULL = zeros, cc:241-242)
 *   h_last     — optional [n_rows][N] final state
 * Returns 0, or -1 on a bad variant.
 */
int oracle_scan_f64(int variant, const float* u, const float* delta, const float* A,
                    const float* B, const float* C, const float* D, const float* z,
                    const float* delta_bias, const double* h0, double* out, double* h_last,
                    int64_t batch, int64_t dim, int64_t seqlen, int64_t dstate,
                    const int64_t* rows, int64_t n_rows) {
  if (variant < 0 || variant > 3) return -1;
  const int fused = is_fused(variant), exact = is_exact(variant);
  const int64_t total = rows ? n_rows : batch * dim;
  double h[1024];
  if (dstate > 1024) return -1;
  for (int64_t i = 0; i < total; ++i) {
    const int64_t r = rows ? rows[i] : i;
    const int64_t b = r / dim, d = r % dim;
    for (int64_t n = 0; n < dstate; ++n) h[n] = h0 ? h0[r * dstate + n] : 0.0;
    for (int64_t l = 0; l < seqlen; ++l) {
      const int64_t ui = (b * dim + d) * seqlen + l;     /* cc:245 */
      const int64_t bci = (b * seqlen + l) * dstate;    /* cc:246 */
      const double ut = u[ui];
      double dt = delta[ui];
      if (fused) dt = softplus_f64(dt + (delta_bias ? (double)delta_bias[d] : 0.0));
      double y = 0.0;
      for (int64_t n = 0; n < dstate; ++n) {
        const double a = A[d * dstate + n];
        const double abar = exact ? exp(dt * a) : 1.0 + dt * a;
        h[n] = abar * h[n] + dt * (double)B[bci + n] * ut;
        y += (double)C[bci + n] * h[n];
      }
      y += (double)D[d] * ut;
      if (fused) y *= silu_f64((double)z[ui]);
      out[i * seqlen + l] = y;
    }
    if (h_last)
      for (int64_t n = 0; n < dstate; ++n) h_last[i * dstate + n] = h[n];
  }
  return 0;
}

/* ---- float32 restatement of the reference's AVX2 numerics (cc:33-148) ---- */

/* cc:33-69: clamp to +-88.3762626647949, n = floor(x*log2e), f = x - n*ln2,
 * Taylor degree-5 polynomial in Horner form with FMAs, times 2^n built as
 * the bit pattern (n+127)<<23. For n = -128 that pattern is 0xFF800000,
 * i.e. -inf: the reference's fast_exp(x) is -inf for x below about -88.03,
 * and this restatement keeps that behaviour. */
static float ref_fast_exp_impl(float x, int contract) {
  const float hi = 88.3762626647949f, lo = -88.3762626647949f;
  x = x < hi ? x : hi;  /* _mm256_min_ps(x, max_val) */
  x = lo > x ? lo : x;  /* _mm256_max_ps(min_val, .) */
  const float t = x * 1.44269504089f;
  const float tf = floorf(t);
  const float f = contract ? fmaf(-tf, 0.6931471805599453f, x) : x - tf * 0.6931471805599453f;
  float p = fmaf(0.008333333333f, f, 0.041666666666f);
  p = fmaf(p, f, 0.166666666666f);
  p = fmaf(p, f, 0.5f);
  p = fmaf(p, f, 1.0f);
  p = fmaf(p, f, 1.0f);
  const int32_t n = (int32_t)tf;
  const uint32_t bits = ((uint32_t)(n + 127)) << 23;
  float pow2n;
  memcpy(&pow2n, &bits, sizeof pow2n);
  return p * pow2n;
}

/* The 8-lane copy inside the scan loop (cc:267-268) computes f with a
 * separate multiply and subtract. The scalar copies that fast_exp (cc:130-135)
 * inlines into fast_softplus and fast_silu come out of g++ -O3 -mfma (whose
 * default -ffp-contract=fast applies) with f = x - n*ln2 contracted into one
 * FMA. Matching both is what makes this restatement bit-exact against the
 * compiled reference. */
static float ref_fast_exp(float x) { return ref_fast_exp_impl(x, 0); }
static float ref_fast_exp_scalar(float x) { return ref_fast_exp_impl(x, 1); }

/* cc:137-143 */
static float ref_fast_softplus(float x) {
  if (x > 20.0f) return x;
  if (x < -20.0f) return ref_fast_exp_scalar(x);
  return log1pf(ref_fast_exp_scalar(x));
}

/* cc:145-148 */
static float ref_fast_silu(float x) { return x / (1.0f + ref_fast_exp_scalar(-x)); }

/* Flush a denormal to zero, as FTZ/DAZ do for the reference's SSE/AVX
 * arithmetic (cc:164-165). */
static float ftz(float x) { return (fabsf(x) < 1.17549435e-38f) ? 0.0f * x : x; }

int oracle_scan_f32ref(int variant, const float* u, const float* delta, const float* A,
                       const float* B, const float* C, const float* D, const float* z,
                       float* out, int64_t batch, int64_t dim, int64_t seqlen,
                       int64_t dstate) {
  if (variant < 0 || variant > 3) return -1;
  if (dstate != 16) return -2; /* cc:228-230 */
  const int fused = is_fused(variant), exact = is_exact(variant);
  for (int64_t b = 0; b < batch; ++b) {
    for (int64_t d = 0; d < dim; ++d) {
      const float* Ap = A + d * 16;
      const float Dv = D[d];
      float h[16] = {0};
      for (int64_t l = 0; l < seqlen; ++l) {
        const int64_t ui = b * dim * seqlen + d * seqlen + l;
        const int64_t bci = b * seqlen * 16 + l * 16;
        const float ut = u[ui];
        float dt = delta[ui];
        if (fused) dt = ref_fast_softplus(dt);
        for (int n = 0; n < 16; ++n) {
          const float Bt = B[bci + n];
          if (exact) {
            const float abar = ref_fast_exp(ftz(dt * Ap[n]));
            const float bbar = dt * Bt;
            h[n] = ftz(fmaf(abar, h[n], ftz(bbar * ut)));
          } else {
            float tmp = ftz(Bt * ut);
            tmp = ftz(fmaf(Ap[n], h[n], tmp));
            h[n] = ftz(fmaf(dt, tmp, h[n]));
          }
        }
        float y = 0.0f;
        for (int n = 0; n < 16; ++n) y = ftz(y + ftz(C[bci + n] * h[n]));
        y = ftz(fmaf(Dv, ut, y)); /* g++ -O3 -mfma contracts y += D*u (cc:297) */
        if (fused) y = ftz(y * ref_fast_silu(z[ui]));
        out[ui] = y;
      }
    }
  }
  return 0;
}

/* ---- the reference's fast_exp, exposed for accuracy measurements ---- */
void oracle_ref_fast_exp(const float* x, float* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = ref_fast_exp(x[i]);
}
