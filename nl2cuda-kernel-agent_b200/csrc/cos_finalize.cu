// cos_finalize.cu -- the last pass of the cosine-similarity backward.
//
//   S[i,j] = ah_i . bh_j,   ah = a / (|a| + eps)          (reference cases/cosine_sim/reference.py:14-21)
//
// The tensor-core backward (DOT instantiation) leaves gA = dS Bh in dA and gB = dS^T Ah in dB:
// the gradients with respect to the normalised rows.  Through ah = a / (|a| + eps),
//   d ah_k / d a_m = delta_km / (|a| + eps) - a_k a_m / (|a| (|a| + eps)^2),
// so with a = (|a| + eps) ah:
//   dA = gA / (|a| + eps) - (ah . gA) ah / |a|,
// the gradient torch autograd takes of the reference's expression (for a zero row torch's norm
// backward gives 0, so the second term is dropped and dA = gA / eps).  The reference's own
// kernel (cases/cosine_sim/kernels/cosine_sim.cu:63-102) uses (gA - (ah . gA) ah) / (|a| + eps),
// which differs from this by a relative eps / |a|.
//
// ah is read back as hi + lo (exact) and |a| from the workspace of the normalising split pass.
// One lane group (8, 16 or 32 lanes) per row, as in the split pass; HBM-bound and small:
// (N + M) * D * 4 bytes in and out plus the split rows.
#include "rbf_common.cuh"
#include "rbf_kernels.cuh"
#include "rbf_ptx.cuh"

namespace rbf {
namespace {

__global__ void __launch_bounds__(256) cos_finalize_kernel(
    float* __restrict__ dA, float* __restrict__ dB, int64_t N, int64_t M, int64_t D, int64_t Dp,
    int G, float eps, const float* __restrict__ an, const float* __restrict__ bn,
    const float* __restrict__ ahi, const float* __restrict__ alo, const float* __restrict__ bhi,
    const float* __restrict__ blo) {
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int sub = lane / G, l = lane % G;
  const int64_t warp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t row = warp * (32 / G) + sub;
  const bool valid = row < N + M;
  const bool is_a = row < N;
  const int64_t r = is_a ? row : row - N;
  float* g = (is_a ? dA : dB) + r * D;
  const float* hi = (is_a ? ahi : bhi) + r * Dp;
  const float* lo = (is_a ? alo : blo) + r * Dp;
  float p = 0.f;
  for (int64_t d = l; valid && d < D; d += G) p = fmaf(hi[d] + lo[d], g[d], p);
  for (int o = G >> 1; o > 0; o >>= 1) p += __shfl_xor_sync(0xffffffffu, p, o);
  if (!valid) return;
  const float n = (is_a ? an : bn)[r];
  const float den = n + eps;
  const float t = n > 0.f ? p / n : 0.f;
  for (int64_t d = l; d < D; d += G) g[d] = g[d] / den - t * (hi[d] + lo[d]);
}

}  // namespace

cudaError_t launch_cos_finalize(float* dA, float* dB, int64_t N, int64_t M, int64_t D, float eps,
                                const void* ws, cudaStream_t stream) {
  const int64_t rows = N + M;
  if (rows == 0 || D == 0) return cudaSuccess;
  const PrepLayout L = prep_layout(N, M, D);
  void* w = const_cast<void*>(ws);
  const int64_t q = (D + 3) / 4;
  const int G = q <= 8 ? 8 : (q <= 16 ? 16 : 32);
  const int rows_per_block = 8 * (32 / G);
  const cudaError_t e = launch_kernel(
      cos_finalize_kernel, dim3((unsigned)ceil_div(rows, rows_per_block)), dim3(256), 0, stream, dA,
      dB, N, M, D, L.Dp, G, eps, ws_at<const float>(w, L.xn), ws_at<const float>(w, L.yn),
      ws_at<const float>(w, L.xhi), ws_at<const float>(w, L.xlo), ws_at<const float>(w, L.yhi),
      ws_at<const float>(w, L.ylo));
  if (e != cudaSuccess) return e;
  note_launches(1);
  return cudaGetLastError();
}

}  // namespace rbf
