// rbf_simt.cu -- fp32 CUDA-core kernels for the RBF forward and backward.
//
// Forward: 128x128 output tile per 256-thread block, 8x8 outputs per thread, the -2 x.y term
// accumulated in fp32 over D in chunks of 16, then the fused epilogue
//   K = exp(-gamma * max(||x||^2 + ||y||^2 - 2 x.y, 0))
// with the norms from the split pass.
// Backward: one kernel template run twice (dX over rows of X reducing over j, dY over rows of Y
// reducing over i), each block owning 32 output rows x 64 features:
//   out[r,:] = -2 gamma * ( sum_k W[r,k] * self[r,:] - sum_k W[r,k] * other[k,:] ),  W = G o K.
#include "rbf_common.cuh"
#include "rbf_kernels.cuh"

namespace rbf {
namespace {

constexpr int kFT = 128;  // forward tile (rows and columns)
constexpr int kFK = 16;   // forward D chunk

__global__ void __launch_bounds__(256) forward_simt_kernel(
    const float* __restrict__ X, const float* __restrict__ Y, const float* __restrict__ xn,
    const float* __restrict__ yn, float* __restrict__ K, int64_t N, int64_t M, int64_t D,
    float neg_gamma) {
  __shared__ float As[kFK][kFT + 4];
  __shared__ float Bs[kFK][kFT + 4];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t i0 = (int64_t)blockIdx.y * kFT, j0 = (int64_t)blockIdx.x * kFT;
  float acc[8][8];
#pragma unroll
  for (int r = 0; r < 8; ++r)
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[r][c] = 0.f;

  for (int64_t k0 = 0; k0 < D; k0 += kFK) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int idx = tid + 256 * e, row = idx >> 4, kk = idx & 15;
      const int64_t k = k0 + kk;
      const int64_t gi = i0 + row, gj = j0 + row;
      As[kk][row] = (gi < N && k < D) ? __ldg(X + gi * D + k) : 0.f;
      Bs[kk][row] = (gj < M && k < D) ? __ldg(Y + gj * D + k) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kFK; ++kk) {
      float a[8], b[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) a[r] = As[kk][ty + 16 * r];
#pragma unroll
      for (int c = 0; c < 8; ++c) b[c] = Bs[kk][tx + 16 * c];
#pragma unroll
      for (int r = 0; r < 8; ++r)
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[r][c] = fmaf(a[r], b[c], acc[r][c]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const int64_t i = i0 + ty + 16 * r;
    if (i >= N) continue;
    const float xi = xn[i];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const int64_t j = j0 + tx + 16 * c;
      if (j >= M) continue;
      const float d = fmaxf(fmaf(-2.f, acc[r][c], xi + yn[j]), 0.f);
      K[i * M + j] = expf(neg_gamma * d);
    }
  }
}

// TRANS = false: rows r are rows of X, reduction k over columns j of G/K, other = Y.
// TRANS = true : rows r are rows of Y, reduction k over rows i of G/K, other = X.
template <bool TRANS>
__global__ void __launch_bounds__(256) backward_simt_kernel(
    const float* __restrict__ self, const float* __restrict__ other, const float* __restrict__ G,
    const float* __restrict__ Km, float* __restrict__ out, int64_t R, int64_t Kred, int64_t N,
    int64_t M, int64_t D, float c) {
  __shared__ float Ws[32][33];
  __shared__ float Os[32][64];
  const int tid = threadIdx.x, row = tid >> 3, dl = tid & 7;
  const int64_t r0 = (int64_t)blockIdx.x * 32, d0 = (int64_t)blockIdx.y * 64;
  (void)N;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float rs = 0.f;
  for (int64_t k0 = 0; k0 < Kred; k0 += 32) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int idx = tid + 256 * e;
      int rr, kk;
      if (!TRANS) { rr = idx >> 5; kk = idx & 31; } else { kk = idx >> 5; rr = idx & 31; }
      const int64_t gr = r0 + rr, gk = k0 + kk;
      float w = 0.f;
      if (gr < R && gk < Kred) {
        const int64_t off = TRANS ? gk * M + gr : gr * M + gk;
        w = __ldg(G + off) * __ldg(Km + off);
      }
      Ws[kk][rr] = w;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int idx = tid + 256 * e, kk = idx >> 6, dd = idx & 63;
      const int64_t gk = k0 + kk, gd = d0 + dd;
      Os[kk][dd] = (gk < Kred && gd < D) ? __ldg(other + gk * D + gd) : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < 32; ++kk) {
      const float w = Ws[kk][row];
      rs += w;
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] = fmaf(w, Os[kk][dl + 8 * q], acc[q]);
    }
    __syncthreads();
  }
  const int64_t gr = r0 + row;
  if (gr >= R) return;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const int64_t gd = d0 + dl + 8 * q;
    if (gd < D) out[gr * D + gd] = c * fmaf(rs, __ldg(self + gr * D + gd), -acc[q]);
  }
}

}  // namespace

cudaError_t launch_forward_simt(const float* X, const float* Y, float* K, int64_t N, int64_t M,
                                int64_t D, float gamma, const void* ws, cudaStream_t stream) {
  if (N == 0 || M == 0) return cudaSuccess;
  const PrepLayout L = prep_layout(N, M, D);
  dim3 grid((unsigned)ceil_div(M, kFT), (unsigned)ceil_div(N, kFT));
  forward_simt_kernel<<<grid, 256, 0, stream>>>(
      X, Y, ws_at<const float>(const_cast<void*>(ws), L.xn),
      ws_at<const float>(const_cast<void*>(ws), L.yn), K, N, M, D, -gamma);
  note_launches(1);
  return cudaGetLastError();
}

cudaError_t launch_backward_simt(const float* X, const float* Y, const float* G, const float* K,
                                 float* dX, float* dY, int64_t N, int64_t M, int64_t D,
                                 float gamma, cudaStream_t stream) {
  if (D == 0) return cudaSuccess;  // dX and dY are empty
  const float c = -2.f * gamma;
  const unsigned dblocks = (unsigned)ceil_div(D, 64);
  if (N > 0) {
    backward_simt_kernel<false><<<dim3((unsigned)ceil_div(N, 32), dblocks), 256, 0, stream>>>(
        X, Y, G, K, dX, N, M, N, M, D, c);
    note_launches(1);
  }
  if (M > 0) {
    backward_simt_kernel<true><<<dim3((unsigned)ceil_div(M, 32), dblocks), 256, 0, stream>>>(
        Y, X, G, K, dY, M, N, N, M, D, c);
    note_launches(1);
  }
  return cudaGetLastError();
}

}  // namespace rbf
