// export.cu -- per-entry cost / lam, plan values and the barycentric map.
//
//   cost_lam_kernel     solver.py:346 + sinkhorn_solvers.py:700:
//                       cost = sum_j (x_rj - y_cj)^2 (each op rounded, as torch's
//                       sub / square / sum), lam = log(max(S, tiny)) - cost / eps
//   plan_values_kernel  sinkhorn_solvers.py:757-758 (plan) and gradient.py:95-97
//                       (T_vals): exp of the potentials plus lam, cost recomputed
//   bary_rows_kernel    gradient.py:52-59 for row-sorted COO: per-row sums in COO
//                       order (the order of the reference's CPU index_add_), then
//                       Tx = sum(T y) / max(sum T, tiny) and grad = 2 a (x - Tx)
//   bary_atomic_kernel  the same sums for unsorted COO and for the column side
#include <cfloat>

#include "common.cuh"
#include "export.h"

namespace sinkslot {

static unsigned grid_for_e(int64_t work, int threads) {
  int64_t g = ceil_div64(work, threads);
  const int64_t cap = (int64_t)num_sms() * 8;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (unsigned)g;
}

__device__ __forceinline__ float sq_cost(const float* __restrict__ x, const float* __restrict__ y,
                                         int d, int64_t r, int64_t c) {
  const float* xr = x + r * d;
  const float* yc = y + c * d;
  float s = 0.0f;
  for (int j = 0; j < d; ++j) {
    const float t = __fsub_rn(xr[j], yc[j]);
    s = __fadd_rn(s, __fmul_rn(t, t));
  }
  return s;
}

__global__ void cost_lam_kernel(const float* __restrict__ x, const float* __restrict__ y, int d,
                                const int64_t* __restrict__ rows, const int64_t* __restrict__ cols,
                                const float* __restrict__ S, int64_t nnz, float eps,
                                float* __restrict__ lam, float* __restrict__ cost_out) {
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < nnz;
       k += (int64_t)gridDim.x * blockDim.x) {
    const float c = sq_cost(x, y, d, rows[k], cols[k]);
    if (cost_out) cost_out[k] = c;
    if (lam) lam[k] = __fsub_rn(logf(fmaxf(S[k], FLT_MIN)), __fdiv_rn(c, eps));
  }
}

int cost_lam(const float* x, const float* y, int d, const int64_t* rows, const int64_t* cols,
             const float* S, int64_t nnz, double eps, float* lam, float* cost, cudaStream_t st) {
  SINKSLOT_REQUIRE(d >= 1 && nnz >= 0, "cost: bad sizes");
  SINKSLOT_REQUIRE(lam == nullptr || S != nullptr, "lam: S is required");
  if (nnz == 0) return kOk;
  cost_lam_kernel<<<grid_for_e(nnz, 256), 256, 0, st>>>(x, y, d, rows, cols, S, nnz, (float)eps, lam,
                                                        cost);
  SINKSLOT_CHECK_LAUNCH();
  return kOk;
}

__global__ void plan_values_kernel(const float* __restrict__ phi, const float* __restrict__ psi,
                                   const int64_t* __restrict__ rows,
                                   const int64_t* __restrict__ cols, const float* __restrict__ S,
                                   const float* __restrict__ x, const float* __restrict__ y, int d,
                                   int64_t nnz, float eps, int grad_form, float* __restrict__ out) {
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < nnz;
       k += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = rows[k], c = cols[k];
    const float ce = __fdiv_rn(sq_cost(x, y, d, r, c), eps);
    const float ls = logf(fmaxf(S[k], FLT_MIN));
    const float pp = __fadd_rn(phi[r], psi[c]);
    const float v = grad_form ? __fadd_rn(pp, __fsub_rn(ls, ce)) : __fsub_rn(__fadd_rn(pp, ls), ce);
    out[k] = expf(v);
  }
}

int plan_values(const float* phi, const float* psi, const int64_t* rows, const int64_t* cols,
                const float* S, const float* x, const float* y, int d, int64_t nnz, double eps,
                int grad_form, float* out, cudaStream_t st) {
  SINKSLOT_REQUIRE(d >= 1 && nnz >= 0, "plan_values: bad sizes");
  if (nnz == 0) return kOk;
  plan_values_kernel<<<grid_for_e(nnz, 256), 256, 0, st>>>(phi, psi, rows, cols, S, x, y, d, nnz,
                                                           (float)eps, grad_form, out);
  SINKSLOT_CHECK_LAUNCH();
  return kOk;
}

// row boundaries of a row-sorted COO: ptr[i] = #{rows < i}
__global__ void row_ptr_kernel(const int64_t* __restrict__ rows, int64_t nnz, int64_t n,
                               int64_t* __restrict__ ptr) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i <= n;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t lo = 0, hi = nnz;
    while (lo < hi) {
      const int64_t mid = (lo + hi) >> 1;
      if (rows[mid] < i) lo = mid + 1; else hi = mid;
    }
    ptr[i] = lo;
  }
}

__global__ void rows_sorted_kernel(const int64_t* __restrict__ r, int64_t nnz, int* flag) {
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x + 1; k < nnz;
       k += (int64_t)gridDim.x * blockDim.x)
    if (r[k] < r[k - 1]) {
      *flag = 1;
      return;
    }
}

constexpr int kMaxD = 16;

__global__ void bary_rows_kernel(const float* __restrict__ T, const int64_t* __restrict__ cols,
                                 const int64_t* __restrict__ ptr, const float* __restrict__ x,
                                 const float* __restrict__ y, int64_t n, int d,
                                 const float* __restrict__ a, float* __restrict__ Tx,
                                 float* __restrict__ grad) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float acc[kMaxD];
    for (int j = 0; j < d; ++j) acc[j] = 0.0f;
    float r = 0.0f;
    for (int64_t k = ptr[i]; k < ptr[i + 1]; ++k) {
      const float t = T[k];
      const float* yc = y + cols[k] * d;
      r = __fadd_rn(r, t);
      for (int j = 0; j < d; ++j) acc[j] = __fadd_rn(acc[j], __fmul_rn(t, yc[j]));
    }
    const float den = fmaxf(r, FLT_MIN);
    for (int j = 0; j < d; ++j) {
      const float tx = __fdiv_rn(acc[j], den);
      if (Tx) Tx[i * d + j] = tx;
      if (grad) grad[i * d + j] = __fmul_rn(__fmul_rn(2.0f, a[i]), __fsub_rn(x[i * d + j], tx));
    }
  }
}

// accumulate sums for one side with atomics: tot[seg] += T, acc[seg, j] += T * pts[other, j]
__global__ void bary_atomic_kernel(const float* __restrict__ T, const int64_t* __restrict__ seg,
                                   const int64_t* __restrict__ oth, const float* __restrict__ pts,
                                   int64_t nnz, int d, float* __restrict__ tot,
                                   float* __restrict__ acc) {
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < nnz;
       k += (int64_t)gridDim.x * blockDim.x) {
    const float t = T[k];
    const int64_t s = seg[k];
    const float* p = pts + oth[k] * d;
    atomicAdd(tot + s, t);
    for (int j = 0; j < d; ++j) atomicAdd(acc + s * d + j, __fmul_rn(t, p[j]));
  }
}

__global__ void bary_finish_kernel(const float* __restrict__ tot, const float* __restrict__ acc,
                                   const float* __restrict__ x, const float* __restrict__ a,
                                   int64_t n, int d, float* __restrict__ Tx,
                                   float* __restrict__ grad) {
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < n * d;
       q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = q / d;
    const float tx = __fdiv_rn(acc[q], fmaxf(tot[i], FLT_MIN));
    if (Tx) Tx[q] = tx;
    if (grad) grad[q] = __fmul_rn(__fmul_rn(2.0f, a[i]), __fsub_rn(x[q], tx));
  }
}

size_t bary_workspace_bytes(int64_t n, int64_t m, int d) {
  Carver cv(nullptr, 0);
  cv.take<int64_t>(n + 1);
  cv.take<float>(n > m ? n : m);
  cv.take<float>((n > m ? n : m) * d);
  cv.take<int>(4);
  return cv.used;
}

int barycentric(const float* T, const int64_t* rows, const int64_t* cols, int64_t nnz,
                const float* x, const float* y, int64_t n, int64_t m, int d, const float* a,
                float* Tx, float* Ty, float* grad, void* ws, size_t ws_bytes, cudaStream_t st) {
  SINKSLOT_REQUIRE(d >= 1 && d <= kMaxD, "barycentric: d must be in [1, 16]");
  SINKSLOT_REQUIRE(grad == nullptr || a != nullptr, "barycentric: grad needs a");
  Carver cv(ws, ws_bytes);
  int64_t* ptr = cv.take<int64_t>(n + 1);
  float* tot = cv.take<float>(n > m ? n : m);
  float* acc = cv.take<float>((n > m ? n : m) * d);
  int* flag = cv.take<int>(4);
  if (!cv.ok) {
    set_error("barycentric: workspace too small");
    return kWorkspaceTooSmall;
  }
  int unsorted = 0;
  if (nnz > 1) {
    SINKSLOT_CUDA_TRY(cudaMemsetAsync(flag, 0, sizeof(int), st));
    rows_sorted_kernel<<<grid_for_e(nnz, 256), 256, 0, st>>>(rows, nnz, flag);
    SINKSLOT_CHECK_LAUNCH();
    SINKSLOT_CUDA_TRY(cudaMemcpyAsync(&unsorted, flag, sizeof(int), cudaMemcpyDeviceToHost, st));
    SINKSLOT_CUDA_TRY(cudaStreamSynchronize(st));
  }
  if (Tx || grad) {
    if (!unsorted) {
      row_ptr_kernel<<<grid_for_e(n + 1, 256), 256, 0, st>>>(rows, nnz, n, ptr);
      SINKSLOT_CHECK_LAUNCH();
      bary_rows_kernel<<<grid_for_e(n, 128), 128, 0, st>>>(T, cols, ptr, x, y, n, d, a, Tx, grad);
      SINKSLOT_CHECK_LAUNCH();
    } else {
      SINKSLOT_CUDA_TRY(cudaMemsetAsync(tot, 0, n * sizeof(float), st));
      SINKSLOT_CUDA_TRY(cudaMemsetAsync(acc, 0, n * d * sizeof(float), st));
      if (nnz > 0) {
        bary_atomic_kernel<<<grid_for_e(nnz, 256), 256, 0, st>>>(T, rows, cols, y, nnz, d, tot, acc);
        SINKSLOT_CHECK_LAUNCH();
      }
      bary_finish_kernel<<<grid_for_e(n * d, 256), 256, 0, st>>>(tot, acc, x, a, n, d, Tx, grad);
      SINKSLOT_CHECK_LAUNCH();
    }
  }
  if (Ty) {
    SINKSLOT_CUDA_TRY(cudaMemsetAsync(tot, 0, m * sizeof(float), st));
    SINKSLOT_CUDA_TRY(cudaMemsetAsync(acc, 0, m * d * sizeof(float), st));
    if (nnz > 0) {
      bary_atomic_kernel<<<grid_for_e(nnz, 256), 256, 0, st>>>(T, cols, rows, x, nnz, d, tot, acc);
      SINKSLOT_CHECK_LAUNCH();
    }
    bary_finish_kernel<<<grid_for_e(m * d, 256), 256, 0, st>>>(tot, acc, nullptr, nullptr, m, d, Ty,
                                                              nullptr);
    SINKSLOT_CHECK_LAUNCH();
  }
  return kOk;
}

__global__ void max_index_kernel(const int64_t* __restrict__ v, int64_t n,
                                 unsigned long long* out) {
  unsigned long long best = 0;
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < n;
       k += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = v[k];
    const unsigned long long u = t < 0 ? 0ull : (unsigned long long)t;
    if (u > best) best = u;
  }
  for (int o = 16; o >= 1; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
    if (t > best) best = t;
  }
  if ((threadIdx.x & 31) == 0) atomicMax(out, best);
}

int max_index(const int64_t* v, int64_t n, void* ws, int64_t* out_host, cudaStream_t st) {
  unsigned long long* d = static_cast<unsigned long long*>(ws);
  SINKSLOT_CUDA_TRY(cudaMemsetAsync(d, 0, sizeof(unsigned long long), st));
  if (n > 0) {
    max_index_kernel<<<grid_for_e(n, 256), 256, 0, st>>>(v, n, d);
    SINKSLOT_CHECK_LAUNCH();
  }
  unsigned long long h = 0;
  SINKSLOT_CUDA_TRY(cudaMemcpyAsync(&h, d, sizeof(h), cudaMemcpyDeviceToHost, st));
  SINKSLOT_CUDA_TRY(cudaStreamSynchronize(st));
  *out_host = (int64_t)h;
  return kOk;
}

// dual value eps * (<phi, a> + <psi, b>) in fp32 partial sums, fp64 across blocks
__global__ void dual_kernel(const float* __restrict__ p, const float* __restrict__ w, int64_t n,
                            double* out) {
  double s = 0.0;
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < n;
       k += (int64_t)gridDim.x * blockDim.x)
    s += (double)__fmul_rn(p[k], w[k]);
  for (int o = 16; o >= 1; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) atomicAdd(out, s);
}

int dual_value(const float* phi, const float* a, int64_t n, const float* psi, const float* b,
               int64_t m, double* dev_out, cudaStream_t st) {
  SINKSLOT_CUDA_TRY(cudaMemsetAsync(dev_out, 0, sizeof(double), st));
  if (n > 0) {
    dual_kernel<<<grid_for_e(n, 256), 256, 0, st>>>(phi, a, n, dev_out);
    SINKSLOT_CHECK_LAUNCH();
  }
  if (m > 0) {
    dual_kernel<<<grid_for_e(m, 256), 256, 0, st>>>(psi, b, m, dev_out);
    SINKSLOT_CHECK_LAUNCH();
  }
  return kOk;
}

}  // namespace sinkslot
