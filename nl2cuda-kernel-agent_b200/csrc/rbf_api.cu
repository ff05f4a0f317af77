// rbf_api.cu -- the C ABI (include/rbf_sm100.h): argument validation, workspace carving and
// kernel dispatch.  Every check that can fail on bad arguments runs on the host before any CUDA
// call, so invalid calls return an rbf_status without touching the device.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <mutex>

#include "../../include/cos_sm100.h"
#include "rbf_common.cuh"
#include "rbf_kernels.cuh"

namespace rbf {

static std::atomic<uint64_t> g_launches{0};
void note_launches(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

bool pdl_enabled() {
  static const bool on = [] {
    const char* s = std::getenv("RBF_NO_PDL");
    return !(s != nullptr && std::atoi(s) != 0);
  }();
  return on;
}

bool deterministic_backward() {
  const char* s = std::getenv("RBF_DETERMINISTIC");
  return s != nullptr && std::atoi(s) != 0;
}

WaitConfig wait_config_from_env() {
  WaitConfig w;
  w.timeout_ns = 2000ull * 1000000ull;
  w.debug_skip_first_load = 0;
  w.fwd_pair = 0;
  w.deterministic = deterministic_backward() ? 1 : 0;
  if (const char* s = std::getenv("RBF_FWD_PAIR")) w.fwd_pair = std::atoi(s) != 0;
  if (const char* s = std::getenv("RBF_WAIT_TIMEOUT_MS")) {
    const long long ms = std::atoll(s);
    if (ms > 0) w.timeout_ns = (unsigned long long)ms * 1000000ull;
  }
  if (const char* s = std::getenv("RBF_DEBUG_SKIP_FIRST_LOAD")) w.debug_skip_first_load = std::atoi(s) != 0;
  return w;
}

namespace {

thread_local char g_detail[512] = "";

int set_detail(int status, const char* what, cudaError_t e = cudaSuccess) {
  if (e != cudaSuccess) {
    std::snprintf(g_detail, sizeof(g_detail), "%s: %s (%s)", what, cudaGetErrorName(e),
                  cudaGetErrorString(e));
  } else {
    std::snprintf(g_detail, sizeof(g_detail), "%s", what);
  }
  return status;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Pointer rule: NULL is allowed only for an empty operand; non-NULL must be 16-byte aligned.
int check_ptr(const void* p, int64_t elems, const char* name) {
  if (elems == 0) return RBF_OK;
  if (p == nullptr) {
    char b[96];
    std::snprintf(b, sizeof(b), "%s is NULL but has %lld elements", name, (long long)elems);
    return set_detail(RBF_ERR_INVALID_ARGUMENT, b);
  }
  if (!aligned16(p)) {
    char b[96];
    std::snprintf(b, sizeof(b), "%s is not 16-byte aligned", name);
    return set_detail(RBF_ERR_MISALIGNED, b);
  }
  return RBF_OK;
}

constexpr int64_t kMaxDim = int64_t(1) << 31;  // rows / cols of one call
constexpr int64_t kMaxD = 4096;

int check_shape(int64_t N, int64_t M, int64_t D, float gamma, bool is_eps = false) {
  if (N < 0 || M < 0 || D < 0) return set_detail(RBF_ERR_INVALID_ARGUMENT, "negative size");
  if (N >= kMaxDim || M >= kMaxDim) return set_detail(RBF_ERR_UNSUPPORTED, "N or M >= 2^31");
  if (D > kMaxD) return set_detail(RBF_ERR_UNSUPPORTED, "D > 4096");
  if (!std::isfinite(gamma))
    return set_detail(RBF_ERR_INVALID_ARGUMENT, is_eps ? "eps is not finite" : "gamma is not finite");
  return RBF_OK;
}

// The current device must be an sm_100 part (B200).  Cached per device ordinal.
int check_device() {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_detail(RBF_ERR_NO_DEVICE, "cudaGetDevice", e);
  static std::mutex mu;
  static int cached[64];
  static bool init = false;
  std::lock_guard<std::mutex> lock(mu);
  if (!init) {
    for (int& c : cached) c = -1;
    init = true;
  }
  if (dev >= 0 && dev < 64 && cached[dev] >= 0) return cached[dev];
  int major = 0, minor = 0;
  e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (e != cudaSuccess) return set_detail(RBF_ERR_CUDA, "cudaDeviceGetAttribute", e);
  const int st = (major == 10 && minor == 0)
                     ? RBF_OK
                     : set_detail(RBF_ERR_NO_DEVICE, "current device is not sm_100 (B200)");
  if (dev >= 0 && dev < 64) cached[dev] = st;
  return st;
}

size_t backward_extra_bytes(int64_t N, int64_t M, int64_t D) {
  return backward_scratch_bytes(N, M, D);
}

int cuda_status(cudaError_t e, const char* what) {
  return e == cudaSuccess ? RBF_OK : set_detail(RBF_ERR_CUDA, what, e);
}

int forward_impl(const float* X, const float* Y, float* K, int64_t N, int64_t M, int64_t D,
                 float gamma, void* ws, size_t ws_bytes, cudaStream_t stream) {
  int st = check_shape(N, M, D, gamma);
  if (st) return st;
  if ((st = check_ptr(X, N * D, "X"))) return st;
  if ((st = check_ptr(Y, M * D, "Y"))) return st;
  if ((st = check_ptr(K, N * M, "K"))) return st;
  const PrepLayout L = prep_layout(N, M, D);
  if (ws == nullptr || ws_bytes < L.end) return set_detail(RBF_ERR_WORKSPACE, "forward workspace too small");
  if (!aligned16(ws)) return set_detail(RBF_ERR_MISALIGNED, "workspace is not 16-byte aligned");
  if ((st = check_device())) return st;
  if ((st = cuda_status(launch_prep(X, Y, N, M, D, ws, stream), "split pass launch"))) return st;
  return cuda_status(launch_forward_tc(X, Y, K, N, M, D, gamma, ws, wait_config_from_env(), stream),
                     "forward launch");
}

int backward_impl(const float* X, const float* Y, const float* G, const float* K, float* dX,
                  float* dY, int64_t N, int64_t M, int64_t D, float gamma, void* ws,
                  size_t ws_bytes, cudaStream_t stream, bool prepared,
                  const DyRoute* route = nullptr, bool pre_zeroed = false) {
  int st = check_shape(N, M, D, gamma);
  if (st) return st;
  if ((st = check_ptr(X, N * D, "X"))) return st;
  if ((st = check_ptr(Y, M * D, "Y"))) return st;
  if ((st = check_ptr(G, N * M, "G"))) return st;
  if ((st = check_ptr(K, N * M, "K"))) return st;
  if ((st = check_ptr(dX, N * D, "dX"))) return st;
  if (route == nullptr && (st = check_ptr(dY, M * D, "dY"))) return st;
  const PrepLayout L = prep_layout(N, M, D);
  const size_t need = L.end + backward_extra_bytes(N, M, D);
  if (ws == nullptr || ws_bytes < need) return set_detail(RBF_ERR_WORKSPACE, "backward workspace too small");
  if (!aligned16(ws)) return set_detail(RBF_ERR_MISALIGNED, "workspace is not 16-byte aligned");
  if ((st = check_device())) return st;
  if (!prepared) {
    if ((st = cuda_status(launch_prep(X, Y, N, M, D, ws, stream), "split pass launch"))) return st;
  }
  if (route != nullptr && !backward_tc_supported(N, M, D))
    return set_detail(RBF_ERR_UNSUPPORTED, "routed dY needs M % 4 == 0 (tensor-core backward)");
  if (backward_tc_supported(N, M, D))
    return cuda_status(launch_backward_tc(X, Y, G, K, dX, dY, N, M, D, gamma, ws,
                                          wait_config_from_env(), stream, route, Epi::kRbf,
                                          pre_zeroed),
                       "backward launch");
  return cuda_status(launch_backward_simt(X, Y, G, K, dX, dY, N, M, D, gamma, stream),
                     "backward launch");
}

// ---- cosine similarity (include/cos_sm100.h): the same split workspace, normalised rows ----

int cos_forward_impl(const float* A, const float* B, float* S, int64_t N, int64_t M, int64_t D,
                     float eps, void* ws, size_t ws_bytes, cudaStream_t stream) {
  int st = check_shape(N, M, D, eps, true);
  if (st) return st;
  if ((st = check_ptr(A, N * D, "A"))) return st;
  if ((st = check_ptr(B, M * D, "B"))) return st;
  if ((st = check_ptr(S, N * M, "S"))) return st;
  const PrepLayout L = prep_layout(N, M, D);
  if (ws == nullptr || ws_bytes < L.end) return set_detail(RBF_ERR_WORKSPACE, "forward workspace too small");
  if (!aligned16(ws)) return set_detail(RBF_ERR_MISALIGNED, "workspace is not 16-byte aligned");
  if ((st = check_device())) return st;
  if ((st = cuda_status(launch_prep(A, B, N, M, D, ws, stream, &eps), "normalising split launch")))
    return st;
  return cuda_status(launch_forward_tc(A, B, S, N, M, D, 0.f, ws, wait_config_from_env(), stream,
                                       Epi::kDot),
                     "forward launch");
}

// A, B: only when !prepared (the normalising split pass runs first).
int cos_backward_impl(const float* A, const float* B, const float* dS, float* dA, float* dB,
                      int64_t N, int64_t M, int64_t D, float eps, void* ws, size_t ws_bytes,
                      cudaStream_t stream, bool prepared) {
  int st = check_shape(N, M, D, eps, true);
  if (st) return st;
  if (!prepared) {
    if ((st = check_ptr(A, N * D, "A"))) return st;
    if ((st = check_ptr(B, M * D, "B"))) return st;
  }
  if ((st = check_ptr(dS, N * M, "dS"))) return st;
  if ((st = check_ptr(dA, N * D, "dA"))) return st;
  if ((st = check_ptr(dB, M * D, "dB"))) return st;
  const PrepLayout L = prep_layout(N, M, D);
  const size_t need = L.end + backward_extra_bytes(N, M, D);
  if (ws == nullptr || ws_bytes < need) return set_detail(RBF_ERR_WORKSPACE, "backward workspace too small");
  if (!aligned16(ws)) return set_detail(RBF_ERR_MISALIGNED, "workspace is not 16-byte aligned");
  if ((st = check_device())) return st;
  if (!prepared) {
    if ((st = cuda_status(launch_prep(A, B, N, M, D, ws, stream, &eps), "normalising split launch")))
      return st;
  }
  // gA = dS Bh, gB = dS^T Ah on the tensor cores (or CUDA cores when M % 4 != 0) ...
  if (backward_tc_supported(N, M, D))
    st = cuda_status(launch_backward_tc(nullptr, nullptr, dS, nullptr, dA, dB, N, M, D, 0.f, ws,
                                        wait_config_from_env(), stream, nullptr, Epi::kDot),
                     "backward launch");
  else
    st = cuda_status(launch_backward_simt(nullptr, nullptr, dS, nullptr, dA, dB, N, M, D, 0.f,
                                          stream, Epi::kDot, ws),
                     "backward launch");
  if (st) return st;
  // ... then through the normalisation, row by row.
  return cuda_status(launch_cos_finalize(dA, dB, N, M, D, eps, ws, stream), "finalize launch");
}

}  // namespace
}  // namespace rbf

using namespace rbf;

extern "C" {

const char* rbf_sm100_strerror(int status) {
  switch (status) {
    case RBF_OK: return "success";
    case RBF_ERR_INVALID_ARGUMENT: return "invalid argument";
    case RBF_ERR_MISALIGNED: return "pointer not 16-byte aligned";
    case RBF_ERR_WORKSPACE: return "workspace missing or too small";
    case RBF_ERR_UNSUPPORTED: return "unsupported shape";
    case RBF_ERR_CUDA: return "CUDA error";
    case RBF_ERR_NO_DEVICE: return "no sm_100 device is current";
    case RBF_ERR_TIMEOUT: return "device-side wait timed out";
    case RBF_ERR_TOO_LARGE: return "size exceeds the entry point's fixed capacity";
    default: return "unknown rbf status";
  }
}

const char* rbf_sm100_last_error_detail(void) { return g_detail; }

int rbf_sm100_version(void) { return 100; }

uint64_t rbf_sm100_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

size_t rbf_sm100_forward_workspace_bytes(int64_t N, int64_t M, int64_t D) {
  if (N < 0 || M < 0 || D < 0) return 0;
  return prep_layout(N, M, D).end;
}

size_t rbf_sm100_backward_workspace_bytes(int64_t N, int64_t M, int64_t D) {
  if (N < 0 || M < 0 || D < 0) return 0;
  return prep_layout(N, M, D).end + backward_extra_bytes(N, M, D);
}

int rbf_sm100_forward(const float* X, const float* Y, float* K, int64_t N, int64_t M, int64_t D,
                      float gamma, void* workspace, size_t workspace_bytes, rbf_stream_t stream) {
  return forward_impl(X, Y, K, N, M, D, gamma, workspace, workspace_bytes,
                      reinterpret_cast<cudaStream_t>(stream));
}

int rbf_sm100_backward(const float* X, const float* Y, const float* G, const float* K, float* dX,
                       float* dY, int64_t N, int64_t M, int64_t D, float gamma, void* workspace,
                       size_t workspace_bytes, rbf_stream_t stream) {
  return backward_impl(X, Y, G, K, dX, dY, N, M, D, gamma, workspace, workspace_bytes,
                       reinterpret_cast<cudaStream_t>(stream), false);
}

int rbf_sm100_backward_prepared(const float* X, const float* Y, const float* G, const float* K,
                                float* dX, float* dY, int64_t N, int64_t M, int64_t D,
                                float gamma, void* workspace, size_t workspace_bytes,
                                rbf_stream_t stream) {
  return backward_impl(X, Y, G, K, dX, dY, N, M, D, gamma, workspace, workspace_bytes,
                       reinterpret_cast<cudaStream_t>(stream), true);
}

int rbf_sm100_forward_backward(const float* X, const float* Y, const float* G, float* K,
                               float* dX, float* dY, int64_t N, int64_t M, int64_t D, float gamma,
                               void* workspace, size_t workspace_bytes, rbf_stream_t stream) {
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // Every backward operand is checked before the forward runs, so a refused call writes nothing.
  int st = check_shape(N, M, D, gamma);
  if (st) return st;
  if ((st = check_ptr(G, N * M, "G"))) return st;
  if ((st = check_ptr(dX, N * D, "dX"))) return st;
  if ((st = check_ptr(dY, M * D, "dY"))) return st;
  if (workspace == nullptr || workspace_bytes < rbf_sm100_backward_workspace_bytes(N, M, D))
    return set_detail(RBF_ERR_WORKSPACE, "forward-backward needs the backward workspace");
  if (!backward_tc_supported(N, M, D)) {
    if ((st = forward_impl(X, Y, K, N, M, D, gamma, workspace, workspace_bytes, s))) return st;
    return backward_impl(X, Y, G, K, dX, dY, N, M, D, gamma, workspace, workspace_bytes, s, true);
  }
  // The split pass also zeroes the backward's accumulation targets (one launch fewer).
  if ((st = check_ptr(X, N * D, "X"))) return st;
  if ((st = check_ptr(Y, M * D, "Y"))) return st;
  if ((st = check_ptr(K, N * M, "K"))) return st;
  if (!aligned16(workspace)) return set_detail(RBF_ERR_MISALIGNED, "workspace is not 16-byte aligned");
  if ((st = check_device())) return st;
  const WaitConfig wc = wait_config_from_env();
  const ZeroSpec zero = backward_zero_spec(N, M, D, workspace, dX, dY, wc);
  if ((st = cuda_status(launch_prep(X, Y, N, M, D, workspace, s, nullptr, &zero), "split pass launch")))
    return st;
  if ((st = cuda_status(launch_forward_tc(X, Y, K, N, M, D, gamma, workspace, wc, s), "forward launch")))
    return st;
  return backward_impl(X, Y, G, K, dX, dY, N, M, D, gamma, workspace, workspace_bytes, s, true,
                       nullptr, true);
}

int rbf_sm100_backward_shard(const float* X_local, const float* Y, const float* G_local,
                             const float* K_local, float* dX_local, float* dY_partial,
                             int64_t N_local, int64_t M, int64_t D, float gamma, void* workspace,
                             size_t workspace_bytes, rbf_stream_t stream) {
  return backward_impl(X_local, Y, G_local, K_local, dX_local, dY_partial, N_local, M, D, gamma,
                       workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream), false);
}

int rbf_sm100_backward_shard_routed(const float* X_local, const float* Y, const float* G_local,
                                    const float* K_local, float* dX_local, int64_t N_local,
                                    int64_t M, int64_t D, float gamma, void* workspace,
                                    size_t workspace_bytes, float* const* dy_buffers, int world,
                                    int rank, const int* step_counter, rbf_stream_t stream) {
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
    return set_detail(RBF_ERR_INVALID_ARGUMENT, "world must be in [1, 8] and rank < world");
  if (dy_buffers == nullptr || step_counter == nullptr)
    return set_detail(RBF_ERR_INVALID_ARGUMENT, "NULL dY buffers or step counter");
  DyRoute route{};
  for (int r = 0; r < world; ++r) {
    if (dy_buffers[r] == nullptr || !aligned16(dy_buffers[r]))
      return set_detail(RBF_ERR_MISALIGNED, "dY buffer NULL or not 16-byte aligned");
    route.bufs[r] = dy_buffers[r];
  }
  route.world = world;
  route.rank = rank;
  route.ctr = step_counter;
  return backward_impl(X_local, Y, G_local, K_local, dX_local, nullptr, N_local, M, D, gamma,
                       workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream), true,
                       &route);
}

int rbf_sm100_dy_exchange(float* dY, int64_t M, int64_t D, float* const* dy_buffers,
                          int* const* flag_arrays, int world, int rank, int* step_counter,
                          unsigned* tickets, void* workspace, size_t workspace_bytes,
                          rbf_stream_t stream) {
  if (M < 0 || D < 0) return set_detail(RBF_ERR_INVALID_ARGUMENT, "negative size");
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
    return set_detail(RBF_ERR_INVALID_ARGUMENT, "world must be in [1, 8] and rank < world");
  if (dy_buffers == nullptr || flag_arrays == nullptr || step_counter == nullptr ||
      tickets == nullptr || (dY == nullptr && M * D > 0))
    return set_detail(RBF_ERR_INVALID_ARGUMENT, "NULL argument");
  if (D % 4 != 0) return set_detail(RBF_ERR_UNSUPPORTED, "the dY exchange needs D % 4 == 0");
  if (workspace == nullptr || workspace_bytes < sizeof(int))
    return set_detail(RBF_ERR_WORKSPACE, "exchange needs the workspace's status word");
  int st = check_device();
  if (st) return st;
  ExchangeArgs a{};
  a.dY = dY;
  a.M = M;
  a.D = D;
  for (int r = 0; r < world; ++r) {
    if (dy_buffers[r] == nullptr || flag_arrays[r] == nullptr)
      return set_detail(RBF_ERR_INVALID_ARGUMENT, "NULL peer pointer");
    a.route.bufs[r] = dy_buffers[r];
    a.flags[r] = flag_arrays[r];
  }
  a.route.world = world;
  a.route.rank = rank;
  a.route.ctr = step_counter;
  a.ctr = step_counter;
  a.tickets = tickets;
  a.status = ws_at<int>(workspace, prep_layout(0, 0, 0).status);
  a.timeout_ns = wait_config_from_env().timeout_ns;
  // Up to RBF_XCHG_ONE_PHASE_MAX ranks (default 8, i.e. always) every rank sums all partials
  // after one barrier; beyond, owners reduce, then a second barrier and a gather.  At 8 ranks
  // and c1 the one-phase read is ~7 MB per rank over NVLink (~9 us), about the cost of the
  // second barrier the two-phase form needs (measured +8 us at 2 ranks).
  a.one_phase_max = 8;
  if (const char* s = std::getenv("RBF_XCHG_ONE_PHASE_MAX")) a.one_phase_max = std::atoi(s);
  return cuda_status(launch_dy_exchange(a, reinterpret_cast<cudaStream_t>(stream)),
                     "exchange launch");
}

size_t cos_sm100_forward_workspace_bytes(int64_t N, int64_t M, int64_t D) {
  return rbf_sm100_forward_workspace_bytes(N, M, D);
}

size_t cos_sm100_backward_workspace_bytes(int64_t N, int64_t M, int64_t D) {
  return rbf_sm100_backward_workspace_bytes(N, M, D);
}

int cos_sm100_forward(const float* A, const float* B, float* S, int64_t N, int64_t M, int64_t D,
                      float eps, void* workspace, size_t workspace_bytes, rbf_stream_t stream) {
  return cos_forward_impl(A, B, S, N, M, D, eps, workspace, workspace_bytes,
                          reinterpret_cast<cudaStream_t>(stream));
}

int cos_sm100_backward_prepared(const float* dS, float* dA, float* dB, int64_t N, int64_t M,
                                int64_t D, float eps, void* workspace, size_t workspace_bytes,
                                rbf_stream_t stream) {
  return cos_backward_impl(nullptr, nullptr, dS, dA, dB, N, M, D, eps, workspace,
                           workspace_bytes, reinterpret_cast<cudaStream_t>(stream), true);
}

int cos_sm100_backward(const float* A, const float* B, const float* dS, float* dA, float* dB,
                       int64_t N, int64_t M, int64_t D, float eps, void* workspace,
                       size_t workspace_bytes, rbf_stream_t stream) {
  return cos_backward_impl(A, B, dS, dA, dB, N, M, D, eps, workspace, workspace_bytes,
                           reinterpret_cast<cudaStream_t>(stream), false);
}

int rbf_sm100_read_status(void* workspace, rbf_stream_t stream, int* device_status) {
  if (workspace == nullptr || device_status == nullptr)
    return set_detail(RBF_ERR_INVALID_ARGUMENT, "NULL workspace or output");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int st = cuda_status(cudaStreamSynchronize(s), "cudaStreamSynchronize");
  if (st) return st;
  int v = 0;
  const PrepLayout L = prep_layout(0, 0, 0);
  if ((st = cuda_status(cudaMemcpy(&v, ws_at<int>(workspace, L.status), sizeof(int),
                                   cudaMemcpyDeviceToHost), "status copy")))
    return st;
  if ((st = cuda_status(cudaMemsetAsync(ws_at<int>(workspace, L.status), 0, sizeof(int), s),
                        "status reset")))
    return st;
  *device_status = v;
  return cuda_status(cudaStreamSynchronize(s), "cudaStreamSynchronize");
}

// ---- legacy host-pointer ABI (reference cases/rbf/delivery/rbf_kernels.cu:168-220) --------

static void legacy_check(int st, const char* what) {
  if (st != RBF_OK) {
    std::fprintf(stderr, "rbf: %s failed: %s (%s)\n", what, rbf_sm100_strerror(st), g_detail);
    std::abort();
  }
}

static void legacy_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) legacy_check(set_detail(RBF_ERR_CUDA, what, e), what);
}

void rbf_forward_cuda(const float* hX, const float* hY, float* hK, int N, int M, int D,
                      float gamma) {
  const size_t sx = sizeof(float) * (size_t)N * D, sy = sizeof(float) * (size_t)M * D,
               sk = sizeof(float) * (size_t)N * M;
  const size_t sw = rbf_sm100_forward_workspace_bytes(N, M, D);
  float *dX = nullptr, *dY = nullptr, *dK = nullptr;
  void* ws = nullptr;
  legacy_cuda(cudaMalloc(&dX, sx ? sx : 16), "cudaMalloc");
  legacy_cuda(cudaMalloc(&dY, sy ? sy : 16), "cudaMalloc");
  legacy_cuda(cudaMalloc(&dK, sk ? sk : 16), "cudaMalloc");
  legacy_cuda(cudaMalloc(&ws, sw), "cudaMalloc");
  legacy_cuda(cudaMemcpy(dX, hX, sx, cudaMemcpyHostToDevice), "cudaMemcpy H2D");
  legacy_cuda(cudaMemcpy(dY, hY, sy, cudaMemcpyHostToDevice), "cudaMemcpy H2D");
  legacy_check(rbf_sm100_forward(dX, dY, dK, N, M, D, gamma, ws, sw, nullptr), "rbf_sm100_forward");
  legacy_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  legacy_cuda(cudaMemcpy(hK, dK, sk, cudaMemcpyDeviceToHost), "cudaMemcpy D2H");
  cudaFree(dX); cudaFree(dY); cudaFree(dK); cudaFree(ws);
}

void rbf_backward_cuda(const float* hX, const float* hY, const float* hG, const float* hK,
                       float* hdX, float* hdY, int N, int M, int D, float gamma) {
  const size_t sx = sizeof(float) * (size_t)N * D, sy = sizeof(float) * (size_t)M * D,
               snm = sizeof(float) * (size_t)N * M;
  const size_t sw = rbf_sm100_backward_workspace_bytes(N, M, D);
  float *dX = nullptr, *dY = nullptr, *dG = nullptr, *dK = nullptr, *ddX = nullptr, *ddY = nullptr;
  void* ws = nullptr;
  legacy_cuda(cudaMalloc(&dX, sx ? sx : 16), "cudaMalloc");
  legacy_cuda(cudaMalloc(&dY, sy ? sy : 16), "cudaMalloc");
  legacy_cuda(cudaMalloc(&dG, snm ? snm : 16), "cudaMalloc");
  legacy_cuda(cudaMalloc(&dK, snm ? snm : 16), "cudaMalloc");
  legacy_cuda(cudaMalloc(&ddX, sx ? sx : 16), "cudaMalloc");
  legacy_cuda(cudaMalloc(&ddY, sy ? sy : 16), "cudaMalloc");
  legacy_cuda(cudaMalloc(&ws, sw), "cudaMalloc");
  legacy_cuda(cudaMemcpy(dX, hX, sx, cudaMemcpyHostToDevice), "cudaMemcpy H2D");
  legacy_cuda(cudaMemcpy(dY, hY, sy, cudaMemcpyHostToDevice), "cudaMemcpy H2D");
  legacy_cuda(cudaMemcpy(dG, hG, snm, cudaMemcpyHostToDevice), "cudaMemcpy H2D");
  legacy_cuda(cudaMemcpy(dK, hK, snm, cudaMemcpyHostToDevice), "cudaMemcpy H2D");
  legacy_check(rbf_sm100_backward(dX, dY, dG, dK, ddX, ddY, N, M, D, gamma, ws, sw, nullptr),
               "rbf_sm100_backward");
  legacy_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  legacy_cuda(cudaMemcpy(hdX, ddX, sx, cudaMemcpyDeviceToHost), "cudaMemcpy D2H");
  legacy_cuda(cudaMemcpy(hdY, ddY, sy, cudaMemcpyDeviceToHost), "cudaMemcpy D2H");
  cudaFree(dX); cudaFree(dY); cudaFree(dG); cudaFree(dK); cudaFree(ddX); cudaFree(ddY);
  cudaFree(ws);
}

}  // extern "C"

// ---- allocation-free forward ------------------------------------------------------------
//
// Some callers cannot allocate device memory: a host runtime whose allocator owns the whole
// device heap, an embedding that forbids cudaMalloc on its hot path, or a plugin with no
// workspace argument to pass through.  rbf_sm100_forward_noalloc serves them with a workspace
// that lives in this file-scope device array instead of a caller buffer.  Every GPU that loads
// the library reserves these bytes until the process exits.
namespace rbf {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // 16 MiB
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

// The current driver context (cuCtxGetCurrent, reached through the runtime's driver entry-point
// table so that the library does not link libcuda directly).
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<CtxGetCurrentFn>(nullptr);
    return reinterpret_cast<CtxGetCurrentFn>(p);
  }();
  return fn;
}

// Device address of g_noalloc_scratch in the current context, looked up once per context.  In
// host code the array's name is only a stand-in, never a device address, so the address must
// come from cudaGetSymbolAddress with that device current.  The cache is keyed by the driver
// context, not the device ordinal: a caller that runs its own (non-primary) context, or that
// reset the device, gets the address that belongs to the context it is using.
int noalloc_scratch(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_detail(RBF_ERR_NO_DEVICE, "cudaGetDevice", e);
  CtxGetCurrentFn get = ctx_get_current();
  CUcontext ctx = nullptr;
  if (get == nullptr || get(&ctx) != CUDA_SUCCESS)
    return set_detail(RBF_ERR_NO_DEVICE, "cuCtxGetCurrent");
  if (ctx == nullptr) {
    // No context bound to this thread yet: the runtime binds the primary context of `dev` on its
    // first call that needs one (this lookup), then the context is read again.
    void* p = nullptr;
    if ((e = cudaGetSymbolAddress(&p, g_noalloc_scratch)) != cudaSuccess)
      return set_detail(RBF_ERR_CUDA, "cudaGetSymbolAddress(scratch)", e);
    if (get(&ctx) != CUDA_SUCCESS || ctx == nullptr)
      return set_detail(RBF_ERR_NO_DEVICE, "no current CUDA context");
  }
  static std::mutex mu;
  constexpr int kSlots = 64;
  static CUcontext keys[kSlots] = {};
  static void* addr[kSlots] = {};
  static int next = 0;
  std::lock_guard<std::mutex> lock(mu);
  for (int k = 0; k < kSlots; ++k)
    if (keys[k] == ctx) {
      *out = addr[k];
      return RBF_OK;
    }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || p == nullptr)
    return set_detail(RBF_ERR_CUDA, "cudaGetSymbolAddress(scratch)", e);
  // A context handle can be reused after its context is destroyed; the slot is then looked up
  // again above and overwritten here (round robin), never read stale for a live context other
  // than the one that created it.
  keys[next] = ctx;
  addr[next] = p;
  next = (next + 1) % kSlots;
  *out = p;
  return RBF_OK;
}

}  // namespace
}  // namespace rbf

extern "C" size_t rbf_sm100_forward_noalloc_capacity(void) { return rbf::kNoAllocScratchBytes; }

extern "C" int rbf_sm100_forward_noalloc(const float* X, const float* Y, float* K, int64_t N,
                                         int64_t M, int64_t D, float gamma,
                                         rbf_stream_t stream) {
  using namespace rbf;
  int st = check_shape(N, M, D, gamma);
  if (st) return st;
  if ((st = check_ptr(X, N * D, "X"))) return st;
  if ((st = check_ptr(Y, M * D, "Y"))) return st;
  if ((st = check_ptr(K, N * M, "K"))) return st;
  const PrepLayout L = prep_layout(N, M, D);
  if (L.end > kNoAllocScratchBytes) {
    char b[256];
    std::snprintf(b, sizeof(b),
                  "needs %zu bytes of scratch for N=%lld M=%lld D=%lld; the allocation-free "
                  "forward holds %zu (use rbf_sm100_forward with a workspace)",
                  L.end, (long long)N, (long long)M, (long long)D, kNoAllocScratchBytes);
    return set_detail(RBF_ERR_TOO_LARGE, b);
  }
  if ((st = check_device())) return st;
  void* ws = nullptr;
  if ((st = noalloc_scratch(&ws))) return st;
  // The split pass rewrites every scratch byte the forward reads (norms, hi/lo splits) and
  // resets the status word, so nothing left by an earlier call leaks into this one.  The status
  // word stays readable through rbf_sm100_forward_noalloc_read_status until the next call.
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if ((st = cuda_status(launch_prep(X, Y, N, M, D, ws, s), "split pass launch"))) return st;
  return cuda_status(launch_forward_tc(X, Y, K, N, M, D, gamma, ws, wait_config_from_env(), s),
                     "forward launch");
}

extern "C" int rbf_sm100_forward_noalloc_read_status(rbf_stream_t stream, int* device_status) {
  using namespace rbf;
  if (device_status == nullptr) return set_detail(RBF_ERR_INVALID_ARGUMENT, "NULL output");
  int st = check_device();
  if (st) return st;
  void* ws = nullptr;
  if ((st = noalloc_scratch(&ws))) return st;
  return rbf_sm100_read_status(ws, stream, device_status);
}
