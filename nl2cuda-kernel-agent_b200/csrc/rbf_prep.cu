// rbf_prep.cu -- the split pass shared by forward and backward.
//
// For every row r of X and of Y it writes
//   norm[r]        = sum_d x[r,d]^2                        (fp32, fixed warp-tree order)
//   hi[r, 0..Dp)   = TF32-exact high part of x[r,:], zero padded from D to Dp
//   lo[r, 0..Dp)   = x[r,:] - hi[r,:]                       (exact in fp32)
// hi/lo are the operands of the 3xTF32 tensor-core products (hi*hi + hi*lo + lo*hi), which
// keep fp32-level accuracy on TF32 hardware.  HBM-bound, (N+M)*D*4 bytes in and
// (N+M)*(2*Dp+1)*4 out.
//
// The normalising variant (cosine similarity) splits the unit rows instead:
//   norm[r] = ||x_r||  (not squared),  hi + lo = x_r / (||x_r|| + eps)  (an IEEE division, as
// the reference's  A / (A.norm(dim=-1, keepdim=True) + eps),  reference
// cases/cosine_sim/reference.py:17-18); hi + lo is the unit row exactly, so the backward reads
// the saved rows back from the split.
#include <algorithm>

#include "rbf_common.cuh"
#include "rbf_kernels.cuh"
#include "rbf_ptx.cuh"

namespace rbf {

// Row r is handled by a group of G lanes (G = 8, 16 or 32: Dp / 4 rounded up to a power of two,
// at most 32), each lane 4 consecutive features per step (float4 loads when D % 4 == 0), so a
// warp covers 32 / G rows at D <= 64 and every load and store is 16 bytes wide.
template <bool NORM>
__global__ void __launch_bounds__(256) prep_split_kernel(
    const float* __restrict__ X, const float* __restrict__ Y, int64_t N, int64_t M, int64_t D,
    int64_t Dp, int G, float eps, float* __restrict__ xn, float* __restrict__ yn, float* __restrict__ xhi,
    float* __restrict__ xlo, float* __restrict__ yhi, float* __restrict__ ylo,
    int* __restrict__ status, ZeroSpec zero) {
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();
  if (blockIdx.x == 0 && threadIdx.x == 0) *status = RBF_OK;  // fresh workspace: no error yet
  const int lane = threadIdx.x & 31;
  const int sub = lane / G, l = lane % G;
  const int64_t warp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t row = warp * (32 / G) + sub;
  const bool valid = row < N + M;
  const bool is_x = row < N;
  const int64_t r = is_x ? row : row - N;
  const float* src = (is_x ? X : Y) + r * D;
  float* hi = (is_x ? xhi : yhi) + r * Dp;
  float* lo = (is_x ? xlo : ylo) + r * Dp;
  const bool vec = (D & 3) == 0;
  auto load4 = [&](int64_t d, float (&v)[4]) {
    if (vec && d + 4 <= D) {
      const float4 f = __ldg(reinterpret_cast<const float4*>(src + d));
      v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) v[e] = d + e < D ? __ldg(src + d + e) : 0.f;
    }
  };
  // Sum over the row's lane group (G is a power of two, so xor partners stay in the group).
  auto group_sum = [&](float s) {
    for (int o = G >> 1; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    return s;
  };
  float den = 1.f, s = 0.f;
  if (NORM) {  // first pass: the row's norm (the second pass re-reads the row from L1 / L2)
    for (int64_t d = 4 * (int64_t)l; valid && d < Dp; d += 4 * (int64_t)G) {
      float v[4];
      load4(d, v);
#pragma unroll
      for (int e = 0; e < 4; ++e) s = fmaf(v[e], v[e], s);
    }
    s = sqrtf(group_sum(s));
    den = s + eps;
  }
  for (int64_t d = 4 * (int64_t)l; valid && d < Dp; d += 4 * (int64_t)G) {
    float v[4];
    load4(d, v);
    float h[4], o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (NORM) v[e] = d + e < D ? v[e] / den : 0.f;  // the padding stays 0 even if den is
      else s = fmaf(v[e], v[e], s);
      tf32_split(v[e], h[e], o[e]);
    }
    *reinterpret_cast<float4*>(hi + d) = make_float4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<float4*>(lo + d) = make_float4(o[0], o[1], o[2], o[3]);
  }
  if (!NORM) s = group_sum(s);
  if (valid && l == 0) (is_x ? xn : yn)[r] = s;
  // Ranges the caller asked to have zeroed (the backward's accumulation targets), grid-stride.
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
#pragma unroll
  for (int z = 0; z < 3; ++z)
    for (int64_t k = tid; k < zero.n[z]; k += stride) zero.p[z][k] = 0.f;
}

cudaError_t launch_prep(const float* X, const float* Y, int64_t N, int64_t M, int64_t D,
                        void* ws, cudaStream_t stream, const float* normalize_eps,
                        const ZeroSpec* zero) {
  const PrepLayout L = prep_layout(N, M, D);
  const int64_t rows = N + M;
  if (rows == 0 && (zero == nullptr || zero->n[0] + zero->n[1] + zero->n[2] == 0)) return cudaSuccess;
  const int64_t q = L.Dp / 4;  // float4 steps per row (Dp is a multiple of 32)
  const int G = q <= 8 ? 8 : (q <= 16 ? 16 : 32);
  const int rows_per_block = 8 * (32 / G);
  const int64_t blocks = std::max<int64_t>(ceil_div(rows, rows_per_block), 1);
  const cudaError_t e = launch_kernel(
      normalize_eps != nullptr ? prep_split_kernel<true> : prep_split_kernel<false>,
      dim3((unsigned)blocks), dim3(256), 0, stream, X, Y, N, M, D, L.Dp, G,
      normalize_eps != nullptr ? *normalize_eps : 0.f, ws_at<float>(ws, L.xn), ws_at<float>(ws, L.yn), ws_at<float>(ws, L.xhi),
      ws_at<float>(ws, L.xlo), ws_at<float>(ws, L.yhi), ws_at<float>(ws, L.ylo),
      ws_at<int>(ws, L.status), zero != nullptr ? *zero : ZeroSpec{});
  if (e != cudaSuccess) return e;
  note_launches(1);
  return cudaGetLastError();
}

}  // namespace rbf
