// export.h -- cost / lam, plan values, barycentric map, small reductions.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace sinkslot {

int cost_lam(const float* x, const float* y, int d, const int64_t* rows, const int64_t* cols,
             const float* S, int64_t nnz, double eps, float* lam, float* cost, cudaStream_t st);
int plan_values(const float* phi, const float* psi, const int64_t* rows, const int64_t* cols,
                const float* S, const float* x, const float* y, int d, int64_t nnz, double eps,
                int grad_form, float* out, cudaStream_t st);
size_t bary_workspace_bytes(int64_t nnz, int64_t n, int64_t m, int d);
int barycentric(const float* T, const int64_t* rows, const int64_t* cols, int64_t nnz,
                const float* x, const float* y, int64_t n, int64_t m, int d, const float* a,
                float* Tx, float* Ty, float* grad, void* ws, size_t ws_bytes, cudaStream_t st);
int max_index(const int64_t* v, int64_t n, void* ws, int64_t* out_host, cudaStream_t st);
int dual_value(const float* phi, const float* a, int64_t n, const float* psi, const float* b,
               int64_t m, double* dev_out, cudaStream_t st);

}  // namespace sinkslot
