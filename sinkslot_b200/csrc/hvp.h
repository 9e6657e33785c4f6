// hvp.h -- Hessian-vector product of grad_X SLOT_eps on a frozen support
// (implicit differentiation of the Sinkhorn fixed point, MINRES on device).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace sinkslot {

struct HvpArgs {
  const float* x = nullptr;  // (n, d)
  const float* y = nullptr;  // (m, d)
  const float* v = nullptr;  // (n, d) direction
  const float* a = nullptr;  // (n) diagonal weights of the u block
  const float* b = nullptr;  // (m) diagonal weights of the w block
  int d = 0;
  // the plan on its support, by rows (CSR) and by columns (CSC)
  const int32_t* r_ptr = nullptr;
  const void* r_idx = nullptr;
  const float* r_T = nullptr;
  const int32_t* c_ptr = nullptr;
  const void* c_idx = nullptr;
  const float* c_T = nullptr;
  int idx_bytes = 4;
  int64_t n = 0, m = 0;
  double eps = 0, tau2 = 0, tol = 0;
  int64_t max_iter = 0;
  void* ws = nullptr;
  size_t ws_bytes = 0;
  float* out = nullptr;      // (n, d)
  float* sol_out = nullptr;  // optional (n + m): the solved (u, w)
  int64_t* iters_host = nullptr;
  double* resid_host = nullptr;
};

size_t hvp_workspace_bytes(int64_t n, int64_t m);
int hvp(const HvpArgs& h, cudaStream_t st);

}  // namespace sinkslot
