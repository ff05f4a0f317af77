// rbf_simt.cu -- fp32 CUDA-core backward for the shapes the tensor-core backward does not take
// (M % 4 != 0: the rows of G and K are not 16-byte pitched, so TMA cannot load them).
// One kernel template run twice (dX over rows of X reducing over j, dY over rows of Y
// reducing over i), each block owning 32 output rows x 64 features:
//   out[r,:] = -2 gamma * ( sum_k W[r,k] * self[r,:] - sum_k W[r,k] * other[k,:] ),  W = G o K.
// The DOT instantiation (cosine similarity) computes out[r,:] = sum_k G[r,k] * other[k,:] only,
// with other = the normalised rows, read back as hi + lo (pitch Dp) from the split workspace;
// K and self are not read.
#include "rbf_common.cuh"
#include "rbf_kernels.cuh"

namespace rbf {
namespace {

template <bool TRANS, bool DOT>
__global__ void __launch_bounds__(256) backward_simt_kernel(
    const float* __restrict__ self, const float* __restrict__ other, const float* __restrict__ G,
    const float* __restrict__ Km, float* __restrict__ out, int64_t R, int64_t Kred, int64_t N,
    int64_t M, int64_t D, float c, const float* __restrict__ other_lo, int64_t opitch) {
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
        w = DOT ? __ldg(G + off) : __ldg(G + off) * __ldg(Km + off);
      }
      Ws[kk][rr] = w;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int idx = tid + 256 * e, kk = idx >> 6, dd = idx & 63;
      const int64_t gk = k0 + kk, gd = d0 + dd;
      float o = 0.f;
      if (gk < Kred && gd < D) {
        o = __ldg(other + gk * opitch + gd);
        if (DOT) o += __ldg(other_lo + gk * opitch + gd);
      }
      Os[kk][dd] = o;
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
    if (gd < D) out[gr * D + gd] = DOT ? acc[q] : c * fmaf(rs, __ldg(self + gr * D + gd), -acc[q]);
  }
}

}  // namespace

cudaError_t launch_backward_simt(const float* X, const float* Y, const float* G, const float* K,
                                 float* dX, float* dY, int64_t N, int64_t M, int64_t D,
                                 float gamma, cudaStream_t stream, Epi epi, const void* ws) {
  if (D == 0) return cudaSuccess;  // dX and dY are empty
  const float c = -2.f * gamma;
  const unsigned dblocks = (unsigned)ceil_div(D, 64);
  const bool dot = epi == Epi::kDot;
  // The "other" operand of each pass: raw rows (pitch D), or for DOT the split rows (pitch Dp).
  const float *ox = X, *oy = Y, *ox_lo = nullptr, *oy_lo = nullptr;
  int64_t pitch = D;
  if (dot) {
    const PrepLayout L = prep_layout(N, M, D);
    void* w = const_cast<void*>(ws);
    ox = ws_at<float>(w, L.xhi);
    ox_lo = ws_at<float>(w, L.xlo);
    oy = ws_at<float>(w, L.yhi);
    oy_lo = ws_at<float>(w, L.ylo);
    pitch = L.Dp;
  }
  if (N > 0) {
    auto kernel = dot ? backward_simt_kernel<false, true> : backward_simt_kernel<false, false>;
    kernel<<<dim3((unsigned)ceil_div(N, 32), dblocks), 256, 0, stream>>>(
        X, oy, G, K, dX, N, M, N, M, D, c, oy_lo, pitch);
    note_launches(1);
  }
  if (M > 0) {
    auto kernel = dot ? backward_simt_kernel<true, true> : backward_simt_kernel<true, false>;
    kernel<<<dim3((unsigned)ceil_div(M, 32), dblocks), 256, 0, stream>>>(
        Y, ox, G, K, dY, M, N, N, M, D, c, ox_lo, pitch);
    note_launches(1);
  }
  return cudaGetLastError();
}

}  // namespace rbf
