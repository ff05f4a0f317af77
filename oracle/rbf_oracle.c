/*
 * rbf_oracle.c -- TEST INFRASTRUCTURE ONLY.  CPU restatement of the reference's RBF algorithm,
 * used as the parity checker by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline.
 * It is never linked into, called by, or reachable from the product library.
 *
 * What it restates (reference paths, relative to the reference project root):
 *   forward   cases/rbf/reference.py:14-20      K = exp(-gamma * sum_d (X[:,None,:]-Y[None,:,:])^2)
 *             (direct-difference form, not the norm expansion the GPU kernels use)
 *   backward  autograd of the above, which is exactly the loop of
 *             cases/rbf/delivery/rbf_test.cu:36-52 / cases/rbf/kernels/rbf_backward.cu:16-57:
 *               coef[i,j] = -2*gamma*G[i,j]*K[i,j]
 *               dX[i,d]   = sum_j coef[i,j]*(X[i,d]-Y[j,d])
 *               dY[j,d]   = sum_i coef[i,j]*(Y[j,d]-X[i,d])
 *
 * Arithmetic: every sum is accumulated in fp64 and exp is evaluated in fp64, so the oracle is
 * more accurate than the fp32 reference; the reference's own fp32 outputs (golden fixtures in
 * tests/golden) are within ~1e-6 of it, which the CPU tests check.  K used in the backward is
 * the oracle's own fp64 K (as rbf_test.cu:87-89 uses the CPU's own K), not the GPU's.
 *
 * Threading is done by the Python caller (ctypes drops the GIL) over row blocks.
 * Every function works on a subset of rows / columns so that parity at full BASELINE sizes can
 * be checked on sampled rows without an O(N*M*D) CPU pass.
 */
#include <math.h>
#include <stdint.h>
#include <stddef.h>

static double sqdist(const float* x, const float* y, int64_t D) {
  double s = 0.0;
  for (int64_t d = 0; d < D; ++d) {
    const double t = (double)x[d] - (double)y[d];
    s += t * t;
  }
  return s;
}

/* K rows: out[r*M + j] = K[rows[r], j] for all j.  reference.py:14-20. */
void oracle_forward_rows(const float* X, const float* Y, int64_t N, int64_t M, int64_t D,
                         double gamma, const int64_t* rows, int64_t n_rows, double* out) {
  (void)N;
  for (int64_t r = 0; r < n_rows; ++r) {
    const float* x = X + rows[r] * D;
    for (int64_t j = 0; j < M; ++j) out[r * M + j] = exp(-gamma * sqdist(x, Y + j * D, D));
  }
}

/* dX rows: out[r*D + d] = dX[rows[r], d].  Needs G rows only (G is N x M row-major).
 * rbf_backward.cu:16-36 / rbf_test.cu:36-52 with fp64 K recomputed. */
void oracle_dx_rows(const float* X, const float* Y, const float* G, int64_t N, int64_t M,
                    int64_t D, double gamma, const int64_t* rows, int64_t n_rows, double* out) {
  (void)N;
  for (int64_t r = 0; r < n_rows; ++r) {
    const int64_t i = rows[r];
    const float* x = X + i * D;
    double* o = out + r * D;
    for (int64_t d = 0; d < D; ++d) o[d] = 0.0;
    for (int64_t j = 0; j < M; ++j) {
      const float* y = Y + j * D;
      const double k = exp(-gamma * sqdist(x, y, D));
      const double coef = -2.0 * gamma * (double)G[i * M + j] * k;
      for (int64_t d = 0; d < D; ++d) o[d] += coef * ((double)x[d] - (double)y[d]);
    }
  }
}

/* dY columns: out[c*D + d] = dY[cols[c], d].  Needs column cols[c] of G over all N rows.
 * rbf_backward.cu:39-57 / rbf_test.cu:36-52 with fp64 K recomputed. */
void oracle_dy_cols(const float* X, const float* Y, const float* G, int64_t N, int64_t M,
                    int64_t D, double gamma, const int64_t* cols, int64_t n_cols, double* out) {
  for (int64_t c = 0; c < n_cols; ++c) {
    const int64_t j = cols[c];
    const float* y = Y + j * D;
    double* o = out + c * D;
    for (int64_t d = 0; d < D; ++d) o[d] = 0.0;
    for (int64_t i = 0; i < N; ++i) {
      const float* x = X + i * D;
      const double k = exp(-gamma * sqdist(x, y, D));
      const double coef = -2.0 * gamma * (double)G[i * M + j] * k;
      for (int64_t d = 0; d < D; ++d) o[d] += coef * ((double)y[d] - (double)x[d]);
    }
  }
}

int oracle_abi_version(void) { return 1; }
