// rbf_common.cuh -- shared definitions of the sm_100a RBF library: workspace layout, launch
// helpers and small device utilities.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

#include "../../include/rbf_sm100.h"

namespace rbf {

constexpr int kSmCount = 148;             // B200: 2 dies x 74 SMs
constexpr size_t kAlign = 1024;           // every workspace section starts on 1 KiB
constexpr int kDPad = 32;                 // feature dim padded to 32 fp32 = one 128 B TMA row

__host__ __device__ inline int64_t round_up(int64_t a, int64_t b) { return (a + b - 1) / b * b; }
__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// -------------------------------------------------------------------------------------------
// Workspace ("prep") layout, shared by forward and backward.
//
//   [status]  64 B: int32 status word written by bounded device waits (RBF_OK / TIMEOUT)
//   [xn]      N  fp32   ||x_i||^2 (fp32, summed in a fixed order)
//   [yn]      M  fp32   ||y_j||^2
//   [xhi,xlo] N x Dp    X split into a TF32-exact high part and the fp32 remainder
//   [yhi,ylo] M x Dp    same for Y               (Dp = D rounded up to 32, zero padded)
//   [bwd]     backward-only scratch (partial dX / dY sums), see rbf_bwd_layout
// -------------------------------------------------------------------------------------------
struct PrepLayout {
  int64_t Dp;
  size_t status, xn, yn, xhi, xlo, yhi, ylo, end;
};

inline PrepLayout prep_layout(int64_t N, int64_t M, int64_t D) {
  PrepLayout L;
  L.Dp = round_up(D > 0 ? D : 1, kDPad);
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off = (size_t)round_up((int64_t)(off + bytes), kAlign); return o; };
  L.status = take(64);
  L.xn = take(sizeof(float) * (size_t)N);
  L.yn = take(sizeof(float) * (size_t)M);
  L.xhi = take(sizeof(float) * (size_t)N * L.Dp);
  L.xlo = take(sizeof(float) * (size_t)N * L.Dp);
  L.yhi = take(sizeof(float) * (size_t)M * L.Dp);
  L.ylo = take(sizeof(float) * (size_t)M * L.Dp);
  L.end = off;
  return L;
}

template <typename T>
inline T* ws_at(void* ws, size_t off) { return reinterpret_cast<T*>(static_cast<char*>(ws) + off); }

// Count of kernels enqueued by this library (rbf_sm100_launch_count).
void note_launches(int n);

// -------------------------------------------------------------------------------------------
// Device helpers
// -------------------------------------------------------------------------------------------

// TF32 split: hi keeps the sign, exponent and top 10 mantissa bits (exactly representable in
// TF32, so the tensor core reads it without rounding); lo = x - hi is exact in fp32.
__device__ __forceinline__ void tf32_split(float x, float& hi, float& lo) {
  hi = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
  lo = x - hi;
}

// exp(-gamma * d) for d >= 0, as 2^(d * (-gamma*log2 e)) on the MUFU ex2 unit.  The scale
// -gamma*log2(e) is rounded once on the host; the product's rounding adds at most
// |d*scale| * 2^-24 * ln 2 relative error (< 1e-6 for K > 1e-30), ex2.approx.ftz adds
// ~2 ulp.  Results below 2^-126 flush to zero (K that small is 0 to every tolerance used).
__device__ __forceinline__ float exp2_approx(float t) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(t));
  return r;
}

}  // namespace rbf
