// rbf_kernels.cuh -- host-side launchers of the kernels in this directory (C++ linkage,
// internal to the library; the public C ABI is include/rbf_sm100.h).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace rbf {

// rbf_prep.cu: norms + TF32 hi/lo split of X and Y into the workspace.
cudaError_t launch_prep(const float* X, const float* Y, int64_t N, int64_t M, int64_t D,
                        void* ws, cudaStream_t stream);

// rbf_simt.cu: fp32 CUDA-core kernels (bring-up path).
cudaError_t launch_forward_simt(const float* X, const float* Y, float* K, int64_t N, int64_t M,
                                int64_t D, float gamma, const void* ws, cudaStream_t stream);
cudaError_t launch_backward_simt(const float* X, const float* Y, const float* G, const float* K,
                                 float* dX, float* dY, int64_t N, int64_t M, int64_t D,
                                 float gamma, cudaStream_t stream);

}  // namespace rbf
