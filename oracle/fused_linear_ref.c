/*
 * ORACLE — test infrastructure only.  Never linked into, or called by, the
 * engine; only tests/, __graft_entry__.smoke() and bench.py's CPU baseline
 * use it, and only as the checker or the CPU reference arm.
 *
 * CPU restatement of the reference's fused-linear oracle:
 *     ref = a @ b + bias                    deepx_op_gpukernelcompiler/kernel.py:64
 *     ref = ACTIVATION_PT[activation](ref)  kernel.py:65-66, fusion.py:87-92
 * extended with the residual add of the MLP chain (Y = ... + R) and with the
 * erf GELU the reference kernels compute (kernel_triton.py:61,
 * kernel_tilelang.py:17).
 *
 * Arithmetic is IEEE double throughout (products and sums in k order, then
 * bias, activation, residual), with libm's tanh/erf/exp.  Inputs arrive as
 * double arrays holding the values of the cast (fp32/fp16/bf16) inputs, so
 * the only error against exact math is double rounding — far below any
 * tolerance the tests use.
 *
 * act: 0 none, 1 relu, 2 gelu (tanh), 3 gelu (erf), 4 silu/swish.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>

static double act_apply(double x, int act) {
  switch (act) {
    case 1:
      return x > 0.0 ? x : 0.0;
    case 2: {
      /* F.gelu(approximate='tanh') */
      const double c = 0.79788456080286535588; /* sqrt(2/pi) */
      return 0.5 * x * (1.0 + tanh(c * (x + 0.044715 * x * x * x)));
    }
    case 3:
      return 0.5 * x * (1.0 + erf(x * 0.70710678118654752440));
    case 4:
      return x / (1.0 + exp(-x));
    default:
      return x;
  }
}

/* Y[m, n] = act(sum_k X[m, k] W[k, n] + bias[n]) + R[m, n]; all row-major,
 * dense.  bias and R may be NULL.  Returns 0, or -1 on a bad argument. */
int oracle_fused_linear_f64(const double* X, const double* W, const double* bias,
                            const double* R, double* Y, int64_t M, int64_t N, int64_t K,
                            int act) {
  if (M < 0 || N < 0 || K < 0 || act < 0 || act > 4) return -1;
  if (M == 0 || N == 0) return 0;
  if (Y == NULL || (K > 0 && (X == NULL || W == NULL))) return -1;
#pragma omp parallel for schedule(static)
  for (int64_t m = 0; m < M; ++m) {
    double* yrow = Y + m * N;
    for (int64_t n = 0; n < N; ++n) yrow[n] = 0.0;
    /* k-outer loop over contiguous rows of W keeps the accumulation order
     * k = 0..K-1 for every output element. */
    for (int64_t k = 0; k < K; ++k) {
      const double a = X[m * K + k];
      const double* wrow = W + k * N;
      for (int64_t n = 0; n < N; ++n) yrow[n] += a * wrow[n];
    }
    for (int64_t n = 0; n < N; ++n) {
      double v = yrow[n] + (bias ? bias[n] : 0.0);
      v = act_apply(v, act);
      if (R) v += R[m * N + n];
      yrow[n] = v;
    }
  }
  return 0;
}

/* Elementwise activation in double (for checking activation formulas). */
int oracle_activation_f64(const double* x, double* y, int64_t n, int act) {
  if (n < 0 || act < 0 || act > 4) return -1;
  for (int64_t i = 0; i < n; ++i) y[i] = act_apply(x[i], act);
  return 0;
}
