/*
 * CPU oracle of the BitNet ternary-weight x int8-activation linear — TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's baseline legs load this library, as the
 * checker of the B200 kernels; the product never links it.
 *
 * Plain-C restatement of the reference's integer path (src/models/bitnet.hpp):
 *   oracle_quantize_weight_ternary  <- quantize_weight_ternary   (bitnet.hpp:70-109)
 *       alpha = mean|w| accumulated in double in index order; q = clamp(round(w / alpha), -1, 1)
 *       computed as round(w * (1/alpha)) in double; alpha == 0 -> all zero, scale 0.
 *   oracle_quantize_activation_int8 <- quantize_activation_int8  (bitnet.hpp:123-165)
 *       amax = max|x| (double); scale = amax / 127; q = clamp(round(x * (1/scale)), -127, 127);
 *       scale == 0 -> all zero.  round() is half-away-from-zero, as std::round.
 *   oracle_bitlinear                <- BitNet::bitlinear         (bitnet.hpp:447-471)
 *       y[o] = float(double(sum_i wq[o,i] * xq[i]) * double(alpha_o) * double(scale_x)),
 *       with alpha per output row and one activation scale per call (per token).
 * Batched helpers run the same arithmetic over M tokens with pre-quantized weights.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>

float oracle_quantize_weight_ternary(const float* w, size_t n, int8_t* q) {
  double sum_abs = 0.0;
  for (size_t i = 0; i < n; ++i) sum_abs += fabs((double)w[i]);
  if (n == 0) return 0.0f;
  const double alpha = sum_abs / (double)n;
  if (alpha == 0.0) {
    for (size_t i = 0; i < n; ++i) q[i] = 0;
    return 0.0f;
  }
  const double inv = 1.0 / alpha;
  for (size_t i = 0; i < n; ++i) {
    double r = round((double)w[i] * inv);
    if (r > 1.0) r = 1.0;
    if (r < -1.0) r = -1.0;
    q[i] = (int8_t)r;
  }
  return (float)alpha;
}

float oracle_quantize_activation_int8(const float* x, size_t n, int8_t* q) {
  if (n == 0) return 0.0f;
  double amax = 0.0;
  for (size_t i = 0; i < n; ++i) {
    const double a = fabs((double)x[i]);
    if (a > amax) amax = a;
  }
  const double scale = amax / 127.0;
  if (scale == 0.0) {
    for (size_t i = 0; i < n; ++i) q[i] = 0;
    return 0.0f;
  }
  const double inv = 1.0 / scale;
  for (size_t i = 0; i < n; ++i) {
    double r = round((double)x[i] * inv);
    if (r > 127.0) r = 127.0;
    if (r < -127.0) r = -127.0;
    q[i] = (int8_t)r;
  }
  return (float)scale;
}

/* y[out_dim] = bitlinear(w[out_dim, in_dim], x[in_dim]); scratch q buffers of in_dim bytes. */
void oracle_bitlinear(const float* w, const float* x, int out_dim, int in_dim, float* y,
                      int8_t* wq_scratch, int8_t* xq_scratch) {
  const float xs = oracle_quantize_activation_int8(x, (size_t)in_dim, xq_scratch);
  for (int o = 0; o < out_dim; ++o) {
    const float a = oracle_quantize_weight_ternary(w + (size_t)o * in_dim, (size_t)in_dim, wq_scratch);
    long long acc = 0;
    for (int i = 0; i < in_dim; ++i) acc += (long long)wq_scratch[i] * (long long)xq_scratch[i];
    y[o] = (float)((double)acc * (double)a * (double)xs);
  }
}

/* Quantize every row of w [N, K]: q [N, K], alpha [N]. */
void oracle_quantize_weight_rows(const float* w, int N, int K, int8_t* q, float* alpha) {
  for (int n = 0; n < N; ++n)
    alpha[n] = oracle_quantize_weight_ternary(w + (size_t)n * K, (size_t)K, q + (size_t)n * K);
}

/* Quantize every token of x [M, K]: q [M, K], scale [M]. */
void oracle_quantize_act_rows(const float* x, int M, int K, int8_t* q, float* scale) {
  for (int m = 0; m < M; ++m)
    scale[m] = oracle_quantize_activation_int8(x + (size_t)m * K, (size_t)K, q + (size_t)m * K);
}

/* y[M, N] from quantized operands: int64 accumulation + the double epilogue of bitlinear;
 * acc_out (optional, [M, N]) receives the raw integer sums. */
void oracle_ternary_gemm(const int8_t* wq, const float* alpha, const int8_t* xq,
                         const float* xscale, int M, int N, int K, float* y, int32_t* acc_out) {
  for (int m = 0; m < M; ++m) {
    const int8_t* xr = xq + (size_t)m * K;
    for (int n = 0; n < N; ++n) {
      const int8_t* wr = wq + (size_t)n * K;
      long long acc = 0;
      for (int k = 0; k < K; ++k) acc += (long long)wr[k] * (long long)xr[k];
      if (acc_out) acc_out[(size_t)m * N + n] = (int32_t)acc;
      y[(size_t)m * N + n] = (float)((double)acc * (double)alpha[n] * (double)xscale[m]);
    }
  }
}
