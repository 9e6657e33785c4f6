// export.cu -- per-entry cost / lam, plan values and the barycentric map.
//
//   cost_lam_kernel     solver.py:346 + sinkhorn_solvers.py:700:
//                       cost = sum_j (x_rj - y_cj)^2 (each op rounded, as torch's
//                       sub / square / sum), lam = log(max(S, tiny)) - cost / eps
//   plan_values_kernel  sinkhorn_solvers.py:757-758 (plan) and gradient.py:95-97
//                       (T_vals): exp of the potentials plus lam, cost recomputed
//   seg_bary_kernel     gradient.py:52-59: per-row (and per-column) sums of the
//                       plan in COO order -- the order of the reference's CPU
//                       index_add_, so results are deterministic -- then
//                       Tx = sum(T y) / max(sum T, tiny) and grad = 2 a (x - Tx)
#include <cfloat>

#include "common.cuh"
#include "export.h"
#include "primitives.h"

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

// Per-segment sums of a sparse plan in COO order (the order of the reference's
// CPU index_add_): the entries are grouped by `seg` with a stable sort (skipped
// when `seg` is already non-decreasing), then one thread per segment sums
//   tot = sum T,  acc_j = sum T * pts[oth, j]
// and writes Tout = acc / max(tot, tiny) and, optionally, grad = 2 a (x - Tout).
constexpr int kMaxD = 16;

__global__ void seg_sorted_check_kernel(const int64_t* __restrict__ r, int64_t nnz, int* flag) {
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x + 1; k < nnz;
       k += (int64_t)gridDim.x * blockDim.x)
    if (r[k] < r[k - 1]) {
      *flag = 1;
      return;
    }
}

__global__ void seg_key32_kernel(const int64_t* __restrict__ r, int64_t nnz,
                                 uint32_t* __restrict__ k) {
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < nnz;
       q += (int64_t)gridDim.x * blockDim.x)
    k[q] = (uint32_t)r[q];
}

// ptr[i] = #{keys < i} over sorted keys (int64 COO indices or uint32 sort keys)
template <typename KT>
__global__ void seg_ptr_kernel(const KT* __restrict__ keys, int64_t nnz, int64_t nseg,
                               int64_t* __restrict__ ptr) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i <= nseg;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t lo = 0, hi = nnz;
    while (lo < hi) {
      const int64_t mid = (lo + hi) >> 1;
      if ((int64_t)keys[mid] < i) lo = mid + 1; else hi = mid;
    }
    ptr[i] = lo;
  }
}

__global__ void seg_bary_kernel(const float* __restrict__ T, const int64_t* __restrict__ oth,
                                const uint32_t* __restrict__ perm, const int64_t* __restrict__ ptr,
                                const float* __restrict__ pts, int64_t nseg, int d,
                                const float* __restrict__ self_pts, const float* __restrict__ a,
                                float* __restrict__ Tout, float* __restrict__ grad) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nseg;
       i += (int64_t)gridDim.x * blockDim.x) {
    float acc[kMaxD];
    for (int j = 0; j < d; ++j) acc[j] = 0.0f;
    float tot = 0.0f;
    for (int64_t q = ptr[i]; q < ptr[i + 1]; ++q) {
      const int64_t k = perm ? (int64_t)perm[q] : q;
      const float t = T[k];
      const float* p = pts + oth[k] * d;
      tot = __fadd_rn(tot, t);
      for (int j = 0; j < d; ++j) acc[j] = __fadd_rn(acc[j], __fmul_rn(t, p[j]));
    }
    const float den = fmaxf(tot, FLT_MIN);
    for (int j = 0; j < d; ++j) {
      const float tx = __fdiv_rn(acc[j], den);
      if (Tout) Tout[i * d + j] = tx;
      if (grad)
        grad[i * d + j] = __fmul_rn(__fmul_rn(2.0f, a[i]), __fsub_rn(self_pts[i * d + j], tx));
    }
  }
}

struct BaryWs {
  uint32_t *k1, *v1, *k2, *v2;
  int64_t *hist, *stmp, *ptr;
  int* flag;
};

static void carve_bary(Carver& cv, BaryWs& w, int64_t nnz, int64_t n, int64_t m) {
  const int64_t e = nnz > 0 ? nnz : 1;
  w.k1 = cv.take<uint32_t>(e); w.v1 = cv.take<uint32_t>(e);
  w.k2 = cv.take<uint32_t>(e); w.v2 = cv.take<uint32_t>(e);
  const int64_t nh = radix_hist_elems(1, e);
  w.hist = cv.take<int64_t>(nh);
  w.stmp = cv.take<int64_t>(scan_tmp_elems(nh));
  w.ptr = cv.take<int64_t>((n > m ? n : m) + 1);
  w.flag = cv.take<int>(4);
}

size_t bary_workspace_bytes(int64_t nnz, int64_t n, int64_t m, int d) {
  (void)d;
  Carver cv(nullptr, 0);
  BaryWs w;
  carve_bary(cv, w, nnz, n, m);
  return cv.used;
}

static int side_sums(const float* T, const int64_t* seg, const int64_t* oth, int64_t nnz,
                     const float* pts, int64_t nseg, int d, const float* self_pts, const float* a,
                     float* Tout, float* grad, BaryWs& w, cudaStream_t st) {
  int unsorted = 0;
  if (nnz > 1) {
    SINKSLOT_CUDA_TRY(cudaMemsetAsync(w.flag, 0, sizeof(int), st));
    seg_sorted_check_kernel<<<grid_for_e(nnz, 256), 256, 0, st>>>(seg, nnz, w.flag);
    SINKSLOT_CHECK_LAUNCH();
    SINKSLOT_CUDA_TRY(cudaMemcpyAsync(&unsorted, w.flag, sizeof(int), cudaMemcpyDeviceToHost, st));
    SINKSLOT_CUDA_TRY(cudaStreamSynchronize(st));
  }
  const uint32_t* perm = nullptr;
  if (!unsorted) {
    seg_ptr_kernel<int64_t><<<grid_for_e(nseg + 1, 256), 256, 0, st>>>(seg, nnz, nseg, w.ptr);
  } else {
    seg_key32_kernel<<<grid_for_e(nnz, 256), 256, 0, st>>>(seg, nnz, w.k1);
    SINKSLOT_CHECK_LAUNCH();
    bool alt = false;
    SINKSLOT_TRY(radix_sort_pairs<uint32_t>(w.k1, w.v1, w.k2, w.v2, true, 1, nnz,
                                            bits_for((uint64_t)(nseg > 1 ? nseg : 1)), w.hist,
                                            w.stmp, &alt, st));
    perm = alt ? w.v2 : w.v1;
    seg_ptr_kernel<uint32_t><<<grid_for_e(nseg + 1, 256), 256, 0, st>>>(alt ? w.k2 : w.k1, nnz,
                                                                        nseg, w.ptr);
  }
  SINKSLOT_CHECK_LAUNCH();
  if (nseg > 0) {
    seg_bary_kernel<<<grid_for_e(nseg, 128), 128, 0, st>>>(T, oth, perm, w.ptr, pts, nseg, d,
                                                          self_pts, a, Tout, grad);
    SINKSLOT_CHECK_LAUNCH();
  }
  return kOk;
}

int barycentric(const float* T, const int64_t* rows, const int64_t* cols, int64_t nnz,
                const float* x, const float* y, int64_t n, int64_t m, int d, const float* a,
                float* Tx, float* Ty, float* grad, void* ws, size_t ws_bytes, cudaStream_t st) {
  SINKSLOT_REQUIRE(d >= 1 && d <= kMaxD, "barycentric: d must be in [1, 16]");
  SINKSLOT_REQUIRE(grad == nullptr || a != nullptr, "barycentric: grad needs a");
  SINKSLOT_REQUIRE(nnz < (int64_t(1) << 32) && n < (int64_t(1) << 31) && m < (int64_t(1) << 31),
                   "barycentric: sizes too large");
  Carver cv(ws, ws_bytes);
  BaryWs w;
  carve_bary(cv, w, nnz, n, m);
  if (!cv.ok) {
    set_error("barycentric: workspace too small");
    return kWorkspaceTooSmall;
  }
  if (Tx || grad)
    SINKSLOT_TRY(side_sums(T, rows, cols, nnz, y, n, d, x, a, Tx, grad, w, st));
  if (Ty)
    SINKSLOT_TRY(side_sums(T, cols, rows, nnz, x, m, d, nullptr, nullptr, Ty, nullptr, w, st));
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
