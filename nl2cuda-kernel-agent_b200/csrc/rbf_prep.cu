// rbf_prep.cu -- the split pass shared by forward and backward.
//
// For every row r of X and of Y it writes
//   norm[r]        = sum_d x[r,d]^2                        (fp32, fixed warp-tree order)
//   hi[r, 0..Dp)   = TF32-exact high part of x[r,:], zero padded from D to Dp
//   lo[r, 0..Dp)   = x[r,:] - hi[r,:]                       (exact in fp32)
// hi/lo are the operands of the 3xTF32 tensor-core products (hi*hi + hi*lo + lo*hi), which
// keep fp32-level accuracy on TF32 hardware.  One warp per row; HBM-bound, (N+M)*D*4 bytes in
// and (N+M)*(2*Dp+1)*4 out.
#include "rbf_common.cuh"
#include "rbf_kernels.cuh"
#include "rbf_ptx.cuh"

namespace rbf {

__global__ void __launch_bounds__(256) prep_split_kernel(
    const float* __restrict__ X, const float* __restrict__ Y, int64_t N, int64_t M, int64_t D,
    int64_t Dp, float* __restrict__ xn, float* __restrict__ yn, float* __restrict__ xhi,
    float* __restrict__ xlo, float* __restrict__ yhi, float* __restrict__ ylo,
    int* __restrict__ status) {
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();
  if (blockIdx.x == 0 && threadIdx.x == 0) *status = RBF_OK;  // fresh workspace: no error yet
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (warp >= N + M) return;
  const bool is_x = warp < N;
  const int64_t r = is_x ? warp : warp - N;
  const float* src = (is_x ? X : Y) + r * D;
  float* hi = (is_x ? xhi : yhi) + r * Dp;
  float* lo = (is_x ? xlo : ylo) + r * Dp;
  float s = 0.f;
  for (int64_t d = lane; d < Dp; d += 32) {
    const float v = d < D ? __ldg(src + d) : 0.f;
    s = fmaf(v, v, s);
    float h, l;
    tf32_split(v, h, l);
    hi[d] = h;
    lo[d] = l;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) (is_x ? xn : yn)[r] = s;
}

cudaError_t launch_prep(const float* X, const float* Y, int64_t N, int64_t M, int64_t D,
                        void* ws, cudaStream_t stream) {
  const PrepLayout L = prep_layout(N, M, D);
  const int64_t rows = N + M;
  if (rows == 0) return cudaSuccess;
  const int warps_per_block = 8;
  const int64_t blocks = ceil_div(rows, warps_per_block);
  const cudaError_t e = launch_kernel(
      prep_split_kernel, dim3((unsigned)blocks), dim3(32 * warps_per_block), 0, stream, X, Y, N,
      M, D, L.Dp, ws_at<float>(ws, L.xn), ws_at<float>(ws, L.yn), ws_at<float>(ws, L.xhi),
      ws_at<float>(ws, L.xlo), ws_at<float>(ws, L.yhi), ws_at<float>(ws, L.ylo),
      ws_at<int>(ws, L.status));
  if (e != cudaSuccess) return e;
  note_launches(1);
  return cudaGetLastError();
}

}  // namespace rbf
