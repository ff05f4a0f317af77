// rbf_selftest.cpp -- standalone C++ self-test of the sm_100a RBF library (no PyTorch).
//
// Replaces the reference delivery's harness (cases/rbf/delivery/rbf_test.cu): random X, Y, G;
// the GPU results through the reference's host-pointer ABI (rbf_forward_cuda /
// rbf_backward_cuda, delivery/README.md:37-41) and through the stream-ordered device-pointer ABI
// (rbf_sm100_forward / rbf_sm100_backward_prepared); a CPU reference in double precision; PASS
// when every element of K, dX, dY is within 1e-3 + 1e-3*|ref| and the two ABIs agree.
//
//   usage: rbf_selftest [N M D gamma seed]      (default 128 128 64 1/64 1234)
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <random>
#include <vector>

#include "rbf_sm100.h"

namespace {

// K = exp(-gamma * ||x_i - y_j||^2) and the backward of sum(G o K), in double precision.
void cpu_reference(const std::vector<float>& X, const std::vector<float>& Y,
                   const std::vector<float>& G, int N, int M, int D, double gamma,
                   std::vector<double>& K, std::vector<double>& dX, std::vector<double>& dY) {
  K.assign((size_t)N * M, 0.0);
  dX.assign((size_t)N * D, 0.0);
  dY.assign((size_t)M * D, 0.0);
  for (int i = 0; i < N; ++i)
    for (int j = 0; j < M; ++j) {
      double s = 0.0;
      for (int d = 0; d < D; ++d) {
        const double t = (double)X[(size_t)i * D + d] - (double)Y[(size_t)j * D + d];
        s += t * t;
      }
      const double k = std::exp(-gamma * s);
      K[(size_t)i * M + j] = k;
      // d/dx_i of G*K = -2 gamma G K (x_i - y_j); d/dy_j is the negative.
      const double w = -2.0 * gamma * (double)G[(size_t)i * M + j] * k;
      for (int d = 0; d < D; ++d) {
        const double t = (double)X[(size_t)i * D + d] - (double)Y[(size_t)j * D + d];
        dX[(size_t)i * D + d] += w * t;
        dY[(size_t)j * D + d] -= w * t;
      }
    }
}

struct Check {
  double max_abs = 0.0, max_rel = 0.0;
  size_t bad = 0;
  void add(double got, double ref) {
    const double e = std::fabs(got - ref);
    max_abs = std::max(max_abs, e);
    if (std::fabs(ref) > 1e-12) max_rel = std::max(max_rel, e / std::fabs(ref));
    if (!(e <= 1e-3 + 1e-3 * std::fabs(ref))) ++bad;  // NaN counts as bad
  }
};

Check compare(const std::vector<float>& got, const std::vector<double>& ref) {
  Check c;
  for (size_t k = 0; k < ref.size(); ++k) c.add(got[k], ref[k]);
  return c;
}

bool cuda_ok(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return true;
  std::fprintf(stderr, "%s: %s\n", what, cudaGetErrorString(e));
  return false;
}

}  // namespace

int main(int argc, char** argv) {
  const int N = argc > 1 ? std::atoi(argv[1]) : 128;
  const int M = argc > 2 ? std::atoi(argv[2]) : 128;
  const int D = argc > 3 ? std::atoi(argv[3]) : 64;
  const float gamma = argc > 4 ? (float)std::atof(argv[4]) : 1.0f / (float)(D > 0 ? D : 1);
  const unsigned seed = argc > 5 ? (unsigned)std::atoi(argv[5]) : 1234u;
  if (N <= 0 || M <= 0 || D <= 0) {
    std::fprintf(stderr, "N, M, D must be positive\n");
    return 2;
  }
  std::printf("rbf_selftest: N=%d M=%d D=%d gamma=%g seed=%u (library %d)\n", N, M, D, gamma,
              seed, rbf_sm100_version());

  std::mt19937 rng(seed);
  std::normal_distribution<float> normal(0.f, 1.f);
  std::vector<float> X((size_t)N * D), Y((size_t)M * D), G((size_t)N * M);
  for (float& v : X) v = normal(rng);
  for (float& v : Y) v = normal(rng);
  for (float& v : G) v = normal(rng);

  // 1. The reference delivery's host-pointer ABI.
  std::vector<float> K((size_t)N * M), dX((size_t)N * D), dY((size_t)M * D);
  rbf_forward_cuda(X.data(), Y.data(), K.data(), N, M, D, gamma);
  rbf_backward_cuda(X.data(), Y.data(), G.data(), K.data(), dX.data(), dY.data(), N, M, D, gamma);

  // 2. The stream-ordered device-pointer ABI (forward fills the workspace, the prepared backward
  //    reuses it).
  std::vector<float> K2(K.size()), dX2(dX.size()), dY2(dY.size());
  {
    float *dXp, *dYp, *dGp, *dKp, *ddX, *ddY;
    void* ws;
    const size_t wsb = std::max(rbf_sm100_forward_workspace_bytes(N, M, D),
                                rbf_sm100_backward_workspace_bytes(N, M, D));
    cudaStream_t s;
    if (!cuda_ok(cudaStreamCreate(&s), "cudaStreamCreate") ||
        !cuda_ok(cudaMalloc(&dXp, X.size() * 4), "cudaMalloc") ||
        !cuda_ok(cudaMalloc(&dYp, Y.size() * 4), "cudaMalloc") ||
        !cuda_ok(cudaMalloc(&dGp, G.size() * 4), "cudaMalloc") ||
        !cuda_ok(cudaMalloc(&dKp, K.size() * 4), "cudaMalloc") ||
        !cuda_ok(cudaMalloc(&ddX, dX.size() * 4), "cudaMalloc") ||
        !cuda_ok(cudaMalloc(&ddY, dY.size() * 4), "cudaMalloc") ||
        !cuda_ok(cudaMalloc(&ws, wsb), "cudaMalloc"))
      return 1;
    cudaMemcpy(dXp, X.data(), X.size() * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(dYp, Y.data(), Y.size() * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(dGp, G.data(), G.size() * 4, cudaMemcpyHostToDevice);
    int st = rbf_sm100_forward(dXp, dYp, dKp, N, M, D, gamma, ws, wsb, s);
    if (st == RBF_OK)
      st = rbf_sm100_backward_prepared(dXp, dYp, dGp, dKp, ddX, ddY, N, M, D, gamma, ws, wsb, s);
    if (st != RBF_OK) {
      std::fprintf(stderr, "rbf_sm100 call failed: %s (%s)\n", rbf_sm100_strerror(st),
                   rbf_sm100_last_error_detail());
      return 1;
    }
    int dev_status = RBF_OK;
    st = rbf_sm100_read_status(ws, s, &dev_status);
    if (st != RBF_OK || dev_status != RBF_OK) {
      std::fprintf(stderr, "device status: %s\n", rbf_sm100_strerror(st != RBF_OK ? st : dev_status));
      return 1;
    }
    cudaMemcpy(K2.data(), dKp, K.size() * 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(dX2.data(), ddX, dX.size() * 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(dY2.data(), ddY, dY.size() * 4, cudaMemcpyDeviceToHost);
    for (void* p : {(void*)dXp, (void*)dYp, (void*)dGp, (void*)dKp, (void*)ddX, (void*)ddY, ws})
      cudaFree(p);
    cudaStreamDestroy(s);
  }

  std::vector<double> Kr, dXr, dYr;
  cpu_reference(X, Y, G, N, M, D, gamma, Kr, dXr, dYr);
  bool pass = true;
  const char* names[3] = {"K", "dX", "dY"};
  const std::vector<float>* got[2][3] = {{&K, &dX, &dY}, {&K2, &dX2, &dY2}};
  const std::vector<double>* ref[3] = {&Kr, &dXr, &dYr};
  for (int abi = 0; abi < 2; ++abi)
    for (int t = 0; t < 3; ++t) {
      const Check c = compare(*got[abi][t], *ref[t]);
      std::printf("  %-13s %-2s max_abs %.3e max_rel %.3e  %s\n",
                  abi == 0 ? "host-pointer" : "stream-order", names[t], c.max_abs, c.max_rel,
                  c.bad == 0 ? "ok" : "FAIL");
      pass = pass && c.bad == 0;
    }
  std::printf("%s\n", pass ? "PASS" : "FAIL");
  return pass ? 0 : 1;
}
