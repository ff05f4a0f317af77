// rbf_kernels.cuh -- host-side launchers of the kernels in this directory (C++ linkage,
// internal to the library; the public C ABI is include/rbf_sm100.h).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

namespace rbf {

// Programmatic dependent launch of the library's kernels (on unless RBF_NO_PDL=1): each launch
// carries cudaLaunchAttributeProgrammaticStreamSerialization, so its prologue may overlap the
// tail of the previous kernel in the stream; the kernels wait (griddepcontrol.wait) before
// touching global memory, so stream order is kept for every byte they read or write.
bool pdl_enabled();

template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Same, launched as clusters of `cluster_x` CTAs along x (gridDim.x a multiple of it).
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                  unsigned cluster_x, cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster_x;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Bound of every device-side mbarrier wait, and the test hook that makes one wait run out.
// Read from the environment at each call: RBF_WAIT_TIMEOUT_MS (default 2000) and
// RBF_DEBUG_SKIP_FIRST_LOAD (default 0; 1 = CTA 0 of the tensor-core kernels never fills its
// first pipeline stage, so the consumer's wait times out and the status word reports it).
struct WaitConfig {
  unsigned long long timeout_ns;
  int debug_skip_first_load;
  int fwd_pair;  // RBF_FWD_PAIR (default 0): 1 runs the D <= 64 forward on two-CTA clusters
  int deterministic;  // RBF_DETERMINISTIC (default 0): 1 makes the backward bit-reproducible
};
WaitConfig wait_config_from_env();
// RBF_DETERMINISTIC set to a non-zero integer (read at every call): the backward stores each
// tile's partials into its own workspace slot and sums the slots in a fixed order.
bool deterministic_backward();

// Row-sharded dY reduction without a library collective: every rank's backward accumulates its
// dY partial into slot (*ctr % kDySlots) of its own buffer bufs[rank] (peer-visible memory, e.g.
// CUDA symmetric memory; bufs[r] is rank r's buffer mapped in this process), and the exchange
// kernel (rbf_exchange.cu) reduces and gathers over NVLink.  world == 0: the caller's dY.
constexpr int kMaxRanks = 8;
constexpr int kDySlots = 2;
struct DyRoute {
  float* bufs[kMaxRanks];
  const int* ctr;
  int world, rank;
};

// What the tensor-core kernels compute from the X.Y^T contraction:
//   kRbf: the forward stores exp(-gamma * (|x|^2 + |y|^2 - 2 x.y)); the backward's W = G o K
//         and it adds the row / column sum terms (the Gaussian RBF case);
//   kDot: the forward stores x.y; the backward's W = G (no K) and it adds nothing else, so
//         dX = G Y and dY = G^T X (the cosine-similarity case, on rows the split pass
//         normalised; cos_finalize_kernel turns these into the gradients of the raw rows).
enum class Epi { kRbf, kDot };

// rbf_fwd_tc.cu: the tcgen05 3xTF32 forward (workspace must hold the split pass output).
cudaError_t launch_forward_tc(const float* X, const float* Y, float* K, int64_t N, int64_t M,
                              int64_t D, float gamma, void* ws, const WaitConfig& wc,
                              cudaStream_t stream, Epi epi = Epi::kRbf);

// rbf_prep.cu: norms + TF32 hi/lo split of X and Y into the workspace.  normalize_eps != NULL:
// the rows are first divided by (||row|| + *normalize_eps) and the norms (not squared) stored.
// Up to three fp32 ranges that a pass zeroes besides its own work (n = 0: unused).
struct ZeroSpec {
  float* p[3] = {nullptr, nullptr, nullptr};
  int64_t n[3] = {0, 0, 0};
};
// zero != NULL: the split pass also zeroes those ranges (the backward's accumulation targets when
// forward and backward run as one call), so the backward needs no zeroing launch of its own.
cudaError_t launch_prep(const float* X, const float* Y, int64_t N, int64_t M, int64_t D,
                        void* ws, cudaStream_t stream, const float* normalize_eps = nullptr,
                        const ZeroSpec* zero = nullptr);

// rbf_fwd_tc.cu host helpers shared by the tensor-core kernels.
bool make_tmap_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                  uint64_t pitch_elems, uint32_t box_cols, uint32_t box_rows,
                  int swizzle = CU_TENSOR_MAP_SWIZZLE_128B);
int device_sm_count();

// rbf_bwd_tc.cu: the fused tcgen05 3xTF32 backward (zeroes dX, dY, then accumulates into
// them).  Needs M % 4 == 0 (16-byte pitched rows of G and K for TMA).
bool backward_tc_supported(int64_t N, int64_t M, int64_t D);
// Workspace bytes the tensor-core backward needs after the split-pass layout (rowsum vector).
size_t backward_scratch_bytes(int64_t N, int64_t M, int64_t D);
// Epi::kDot: K is not read (may be NULL) and gamma is ignored.
// pre_zeroed: the ranges of backward_zero_spec were zeroed earlier in stream order (by the split
// pass of a one-call forward + backward), so the zeroing launch is skipped.
cudaError_t launch_backward_tc(const float* X, const float* Y, const float* G, const float* K,
                               float* dX, float* dY, int64_t N, int64_t M, int64_t D,
                               float gamma, void* ws, const WaitConfig& wc, cudaStream_t stream,
                               const DyRoute* route = nullptr, Epi epi = Epi::kRbf,
                               bool pre_zeroed = false);
// The ranges the tensor-core backward (caller's dY, no route) zeroes before it accumulates.
ZeroSpec backward_zero_spec(int64_t N, int64_t M, int64_t D, void* ws, float* dX, float* dY,
                            const WaitConfig& wc);

// rbf_exchange.cu: completes a routed step -- barrier, owners reduce their j-blocks over every
// rank's slot, barrier, every rank gathers dY from the owners, the step counter advances.
// flags[r] is rank r's int[world] signal array (peer memory).
struct ExchangeArgs {
  float* dY;
  int64_t M, D;
  DyRoute route;
  int* flags[kMaxRanks];
  int* ctr;
  unsigned* tickets;  // two zeroed counters reused across steps, then the sticky failure flag
  int one_phase_max;  // up to this many ranks: one barrier, every rank sums all partials
  int* status;
  unsigned long long timeout_ns;
};
cudaError_t launch_dy_exchange(const ExchangeArgs& a, cudaStream_t stream);

// rbf_simt.cu: fp32 CUDA-core backward for M % 4 != 0.  Epi::kDot: W = G, K unused, and the
// rows multiplied are the normalised ones of the split workspace `ws`.
cudaError_t launch_backward_simt(const float* X, const float* Y, const float* G, const float* K,
                                 float* dX, float* dY, int64_t N, int64_t M, int64_t D,
                                 float gamma, cudaStream_t stream, Epi epi = Epi::kRbf,
                                 const void* ws = nullptr);

// cos_finalize.cu: turns gA = dS Bh and gB = dS^T Ah (in dA, dB, in place) into the gradients of
// the raw rows, dA = gA / (|a| + eps) - (Ah . gA) Ah / |a|  (the second term 0 for a zero row),
// reading Ah = hi + lo and |a| from a workspace the normalising split pass filled.
cudaError_t launch_cos_finalize(float* dA, float* dB, int64_t N, int64_t M, int64_t D, float eps,
                                const void* ws, cudaStream_t stream);

}  // namespace rbf
