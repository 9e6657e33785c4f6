// hvp.cu -- Hessian-vector product H(X) v of grad_X SLOT_eps by implicit
// differentiation of the Sinkhorn fixed point on a frozen support
// (reference: sinkslot/hvp.py:34-113, hvp_x_sqeuclid_from_potentials).
//
// With the plan P (T_k on the support entries (r_k, c_k)) at the converged
// potentials and dlam_k = -(2/eps) <x_{r_k} - y_{c_k}, v_{r_k}> (hvp.py:88):
//
//   rhs_u[i] = -sum_{k in row i} T_k dlam_k,   rhs_w[j] = -sum_{k in col j} T_k dlam_k
//   [ diag(a + tau)  P             ] [u]   [rhs_u]
//   [ P^T            diag(b + tau) ] [w] = [rhs_w]          (hvp.py:90-108)
//   H v = 2 a v - 2 sum_{k in row i} T_k (u_i + w_{c_k} + dlam_k) y_{c_k}   (hvp.py:110-113)
//
// The symmetric system is solved by MINRES (Paige & Saunders, 1975), the
// method the reference reaches through torchsparsegradutils' `minres`:
// Lanczos vectors v_k, the tridiagonal's QR by Givens rotations, direction
// vectors w_k, x_k = x_{k-1} + c_k eta w_k, |eta| the residual norm; it stops
// when |eta| <= tol * ||rhs|| or after max_iter iterations.  Everything stays on
// the device: one iteration is three launches (the operator applied to v_k
// with the alpha dot product, the beta norm, the rotation and vector updates);
// the scalars live in a two-slot device state that every block reads and block
// 0 writes for the next iteration.  All sums run in a fixed order, so a solve
// is deterministic.  Every segmented sum (rows over the CSR of P, columns over
// its CSC) uses G lanes per segment and a fixed shuffle tree.
#include <cfloat>
#include <cmath>

#include "common.cuh"
#include "hvp.h"

namespace sinkslot {

namespace {

constexpr int kHvpThreads = 256;
constexpr int kHvpG = 8;  // lanes per segment
constexpr int kMaxHvpD = 16;

struct Minres {
  double beta;      // beta_k
  double c1, s1;    // rotation k-1
  double c2, s2;    // rotation k-2
  double eta;
  double beta1;     // ||rhs||
  double resid;     // |eta| after the last iteration
  long long iters;
  int done;
};

unsigned blocks_for(int64_t segs) {
  int64_t g = ceil_div64(segs * kHvpG, kHvpThreads);
  const int64_t cap = (int64_t)num_sms() * 4;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (unsigned)g;
}

__device__ __forceinline__ float dlam_of(const float* __restrict__ x, const float* __restrict__ y,
                                         const float* __restrict__ v, int d, int64_t i,
                                         int64_t j, float two_over_eps) {
  float s = 0.0f;
  for (int q = 0; q < d; ++q)
    s = __fadd_rn(s, __fmul_rn(__fsub_rn(x[i * d + q], y[j * d + q]), v[i * d + q]));
  return -__fmul_rn(two_over_eps, s);
}

// segment s of the operator's 2-block layout: rows [0, n) through the CSR,
// columns [n, n + m) through the CSC
template <typename IT>
struct Side {
  const int32_t* ptr;
  const IT* idx;
  const float* T;
};

template <typename IT>
struct Op {
  Side<IT> row, col;
  int64_t n, m;
};

// sum over the group's lanes in a fixed tree
__device__ __forceinline__ double group_sum(double v) {
#pragma unroll
  for (int o = kHvpG / 2; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o, kHvpG);
  return v;
}

// Block sum of one double per thread into part[blockIdx.x] (fixed order).
__device__ __forceinline__ void block_partial(double v, double* part) {
  __shared__ double red[kHvpThreads / 32];
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < kHvpThreads / 32; ++w) t += red[w];
    part[blockIdx.x] = t;
  }
}

// Sum of the nb block partials (every thread, same order: the same value).
__device__ __forceinline__ double all_partials(const double* part, int nb) {
  double t = 0.0;
  for (int b = 0; b < nb; ++b) t += part[b];
  return t;
}

// Generic segmented pass over both sides: f(seg, lane-strided entry sum) per
// segment; `term(k, s, other)` gives the entry's contribution.
template <typename IT, typename Term, typename Fin>
__device__ __forceinline__ void both_sides(const Op<IT>& op, Term term, Fin fin) {
  const int lane = threadIdx.x & (kHvpG - 1);
  const int64_t groups = (int64_t)gridDim.x * kHvpThreads / kHvpG;
  const int64_t total = op.n + op.m;
  const int64_t gw = ((int64_t)blockIdx.x * kHvpThreads + (threadIdx.x & ~31)) / kHvpG;
  const int gin = (threadIdx.x & 31) / kHvpG;
  for (int64_t base = gw; base < total; base += groups) {
    const int64_t s = base + gin;
    const bool act = s < total;
    const bool isrow = s < op.n;
    const Side<IT>& sd = isrow ? op.row : op.col;
    const int64_t seg = isrow ? s : s - op.n;
    const int64_t b0 = act ? sd.ptr[seg] : 0, b1 = act ? sd.ptr[seg + 1] : 0;
    double acc = 0.0;
    for (int64_t k = b0 + lane; k < b1; k += kHvpG)
      acc += (double)term(isrow, seg, (int64_t)sd.idx[k], sd.T[k]);
    acc = group_sum(acc);
    fin(act && lane == 0, s, acc);
  }
}

// rhs[s] = -sum T_k dlam_k over the segment
template <typename IT>
__global__ void __launch_bounds__(kHvpThreads) rhs_kernel(const Op<IT> op,
                                                          const float* __restrict__ x,
                                                          const float* __restrict__ y,
                                                          const float* __restrict__ v, int d,
                                                          float two_over_eps,
                                                          float* __restrict__ rhs,
                                                          double* __restrict__ part) {
  double sq = 0.0;
  both_sides(
      op,
      [&](bool isrow, int64_t seg, int64_t oth, float t) {
        const int64_t i = isrow ? seg : oth, j = isrow ? oth : seg;
        return -__fmul_rn(t, dlam_of(x, y, v, d, i, j, two_over_eps));
      },
      [&](bool store, int64_t s, double acc) {
        if (store) {
          const float r = (float)acc;
          rhs[s] = r;
          sq += (double)r * (double)r;
        }
      });
  block_partial(sq, part);
}

// v1 = rhs / beta1, x = 0, w buffers = 0, v0 = 0; the state's first slot
__global__ void minres_init_kernel(const float* __restrict__ rhs, int64_t N,
                                   const double* __restrict__ part, int nb, double tol,
                                   float* __restrict__ v0, float* __restrict__ v1,
                                   float* __restrict__ w0, float* __restrict__ w1,
                                   float* __restrict__ xsol, Minres* st) {
  const double beta1 = sqrt(all_partials(part, nb));
  const float inv = beta1 > 0.0 ? (float)(1.0 / beta1) : 0.0f;
  for (int64_t s = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; s < N;
       s += (int64_t)gridDim.x * blockDim.x) {
    v0[s] = 0.0f;
    v1[s] = __fmul_rn(rhs[s], inv);
    w0[s] = 0.0f;
    w1[s] = 0.0f;
    xsol[s] = 0.0f;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    Minres m{};
    m.beta = beta1;
    m.c1 = m.c2 = 1.0;
    m.s1 = m.s2 = 0.0;
    m.eta = beta1;
    m.beta1 = beta1;
    m.resid = beta1;
    m.iters = 0;
    m.done = (beta1 <= 0.0 || !(beta1 == beta1)) ? 1 : 0;
    (void)tol;
    st[0] = m;
  }
}

// p = M v_k - beta_k v_{k-1}; partial of <v_k, p>
template <typename IT>
__global__ void __launch_bounds__(kHvpThreads) minres_apply_kernel(
    const Op<IT> op, const float* __restrict__ diag, const float* __restrict__ vk,
    const float* __restrict__ vkm1, float* __restrict__ p, double* __restrict__ part,
    const Minres* __restrict__ st) {
  const Minres S = *st;
  if (S.done) return;
  const float beta = (float)S.beta;
  double dot = 0.0;
  both_sides(
      op,
      [&](bool isrow, int64_t, int64_t oth, float t) {
        return __fmul_rn(t, vk[isrow ? op.n + oth : oth]);
      },
      [&](bool store, int64_t s, double acc) {
        if (store) {
          const float ps = __fsub_rn(__fadd_rn(__fmul_rn(diag[s], vk[s]), (float)acc),
                                     __fmul_rn(beta, vkm1[s]));
          p[s] = ps;
          dot += (double)vk[s] * (double)ps;
        }
      });
  block_partial(dot, part);
}

// alpha = sum of the partials; p -= alpha v_k; partial of ||p||^2
__global__ void __launch_bounds__(kHvpThreads) minres_orth_kernel(
    int64_t N, const float* __restrict__ vk, float* __restrict__ p,
    const double* __restrict__ part_alpha, int nb, double* __restrict__ part_beta,
    const Minres* __restrict__ st) {
  if (st->done) return;
  const float alpha = (float)all_partials(part_alpha, nb);
  double sq = 0.0;
  for (int64_t s = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; s < N;
       s += (int64_t)gridDim.x * blockDim.x) {
    const float ps = __fsub_rn(p[s], __fmul_rn(alpha, vk[s]));
    p[s] = ps;
    sq += (double)ps * (double)ps;
  }
  block_partial(sq, part_beta);
}

// beta_{k+1}, the rotations, v_{k+1} (over v_{k-1}), w_k (over w_{k-2}), x
__global__ void __launch_bounds__(kHvpThreads) minres_update_kernel(
    int64_t N, const float* __restrict__ vk, const float* __restrict__ p,
    float* __restrict__ vnext, float* __restrict__ wkm2, const float* __restrict__ wkm1,
    float* __restrict__ xsol, const double* __restrict__ part_alpha,
    const double* __restrict__ part_beta, int nb, double tol, long long max_iter,
    const Minres* __restrict__ st_in, Minres* __restrict__ st_out) {
  const Minres S = *st_in;
  if (S.done) {
    if (blockIdx.x == 0 && threadIdx.x == 0) *st_out = S;
    return;
  }
  const double alpha = (double)(float)all_partials(part_alpha, nb);
  const double beta_next = sqrt(all_partials(part_beta, nb));
  const double eps_k = S.s2 * S.beta;
  const double dbar = S.c2 * S.beta;
  const double delta = S.c1 * dbar + S.s1 * alpha;
  const double gbar = -S.s1 * dbar + S.c1 * alpha;
  const double gamma = hypot(gbar, beta_next);
  const bool ok = gamma > 0.0;
  const double c = ok ? gbar / gamma : 1.0;
  const double s = ok ? beta_next / gamma : 0.0;
  const float f_eps = (float)eps_k, f_delta = (float)delta;
  const float inv_g = ok ? (float)(1.0 / gamma) : 0.0f;
  const float step = (float)(c * S.eta);
  const float inv_b = beta_next > 0.0 ? (float)(1.0 / beta_next) : 0.0f;
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < N;
       q += (int64_t)gridDim.x * blockDim.x) {
    const float w = __fmul_rn(
        __fsub_rn(__fsub_rn(vk[q], __fmul_rn(f_eps, wkm2[q])), __fmul_rn(f_delta, wkm1[q])),
        inv_g);
    wkm2[q] = w;
    xsol[q] = __fadd_rn(xsol[q], __fmul_rn(step, w));
    vnext[q] = __fmul_rn(p[q], inv_b);
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    Minres m = S;
    m.beta = beta_next;
    m.c2 = S.c1;
    m.s2 = S.s1;
    m.c1 = c;
    m.s1 = s;
    m.eta = -s * S.eta;
    m.resid = fabs(m.eta);
    m.iters = S.iters + 1;
    m.done = (!ok || beta_next <= 0.0 || m.resid <= tol * S.beta1 || m.iters >= max_iter ||
              !(m.resid == m.resid))
                 ? 1
                 : 0;
    *st_out = m;
  }
}

// out[i, :] = 2 a_i v_i - 2 sum_{k in row i} T_k (u_i + w_{c_k} + dlam_k) y_{c_k}
template <typename IT>
__global__ void __launch_bounds__(kHvpThreads) hvp_out_kernel(
    const Side<IT> row, int64_t n, const float* __restrict__ x, const float* __restrict__ y,
    const float* __restrict__ v, const float* __restrict__ a, int d, float two_over_eps,
    const float* __restrict__ sol, float* __restrict__ out) {
  const int lane = threadIdx.x & (kHvpG - 1);
  const int64_t groups = (int64_t)gridDim.x * kHvpThreads / kHvpG;
  const int64_t gw = ((int64_t)blockIdx.x * kHvpThreads + (threadIdx.x & ~31)) / kHvpG;
  const int gin = (threadIdx.x & 31) / kHvpG;
  for (int64_t base = gw; base < n; base += groups) {
    const int64_t i = base + gin;
    const bool act = i < n;
    const int64_t b0 = act ? row.ptr[i] : 0, b1 = act ? row.ptr[i + 1] : 0;
    double acc[kMaxHvpD];
    for (int q = 0; q < d; ++q) acc[q] = 0.0;
    const float ui = act ? sol[i] : 0.0f;
    for (int64_t k = b0 + lane; k < b1; k += kHvpG) {
      const int64_t j = (int64_t)row.idx[k];
      const float wgt = __fmul_rn(
          row.T[k], __fadd_rn(__fadd_rn(ui, sol[n + j]), dlam_of(x, y, v, d, i, j, two_over_eps)));
      for (int q = 0; q < d; ++q) acc[q] += (double)__fmul_rn(wgt, y[j * d + q]);
    }
    for (int q = 0; q < d; ++q) {
      const double t = group_sum(acc[q]);
      if (act && lane == 0)
        out[i * d + q] = __fsub_rn(__fmul_rn(__fmul_rn(2.0f, a[i]), v[i * d + q]),
                                   __fmul_rn(2.0f, (float)t));
    }
  }
}

__global__ void diag_kernel(const float* __restrict__ a, int64_t n, const float* __restrict__ b,
                            int64_t m, float tau, float* __restrict__ diag) {
  for (int64_t s = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; s < n + m;
       s += (int64_t)gridDim.x * blockDim.x)
    diag[s] = __fadd_rn(s < n ? a[s] : b[s - n], tau);
}

struct HvpWs {
  float *diag, *rhs, *p, *x;
  float* v[3];
  float* w[2];
  double *pa, *pb;
  Minres* st;  // two slots
};

void carve_hvp(Carver& cv, HvpWs& w, int64_t N) {
  w.diag = cv.take<float>(N);
  w.rhs = cv.take<float>(N);
  w.p = cv.take<float>(N);
  w.x = cv.take<float>(N);
  for (auto& t : w.v) t = cv.take<float>(N);
  for (auto& t : w.w) t = cv.take<float>(N);
  const int64_t nb = (int64_t)num_sms() * 4;
  w.pa = cv.take<double>(nb);
  w.pb = cv.take<double>(nb);
  w.st = cv.take<Minres>(2);
}

template <typename IT>
int hvp_run(const HvpArgs& h, cudaStream_t st) {
  const int64_t n = h.n, m = h.m, N = n + m;
  Carver cv(h.ws, h.ws_bytes);
  HvpWs w;
  carve_hvp(cv, w, N);
  if (!cv.ok) {
    set_error("hvp: workspace too small");
    return kWorkspaceTooSmall;
  }
  Op<IT> op;
  op.row = Side<IT>{h.r_ptr, static_cast<const IT*>(h.r_idx), h.r_T};
  op.col = Side<IT>{h.c_ptr, static_cast<const IT*>(h.c_idx), h.c_T};
  op.n = n;
  op.m = m;
  const float toe = (float)(2.0 / h.eps);
  const unsigned gs = blocks_for(N);         // segment kernels
  const unsigned ge = blocks_for(N / kHvpG + 1);  // elementwise kernels (one element per thread)
  diag_kernel<<<ge, kHvpThreads, 0, st>>>(h.a, n, h.b, m, (float)h.tau2, w.diag);
  SINKSLOT_CHECK_LAUNCH();
  rhs_kernel<IT><<<gs, kHvpThreads, 0, st>>>(op, h.x, h.y, h.v, h.d, toe, w.rhs, w.pb);
  SINKSLOT_CHECK_LAUNCH();
  // v_0 = 0 in v[0], v_1 in v[1]; w_{-1} in w[1], w_0 in w[0]
  minres_init_kernel<<<ge, kHvpThreads, 0, st>>>(w.rhs, N, w.pb, (int)gs, h.tol, w.v[0], w.v[1],
                                                 w.w[0], w.w[1], w.x, w.st);
  SINKSLOT_CHECK_LAUNCH();
  // Iteration k (1-based): v_{k-1} = v[(k-1)%3], v_k = v[k%3], v_{k+1} -> v[(k+1)%3]
  // (over v_{k-2}); w_{k-2} = w[k%2] (overwritten by w_k), w_{k-1} = w[(k+1)%2];
  // state slot k%2... slot 0 holds the state entering iteration 1.
  const int64_t check_every = 64;
  for (int64_t k = 1; k <= h.max_iter; ++k) {
    const Minres* s_in = w.st + ((k - 1) & 1);
    Minres* s_out = w.st + (k & 1);
    float* vkm1 = w.v[(k - 1) % 3];
    float* vk = w.v[k % 3];
    float* vnext = w.v[(k + 1) % 3];
    float* wkm2 = w.w[k & 1];
    float* wkm1 = w.w[(k + 1) & 1];
    minres_apply_kernel<IT><<<gs, kHvpThreads, 0, st>>>(op, w.diag, vk, vkm1, w.p, w.pa, s_in);
    minres_orth_kernel<<<gs, kHvpThreads, 0, st>>>(N, vk, w.p, w.pa, (int)gs, w.pb, s_in);
    minres_update_kernel<<<gs, kHvpThreads, 0, st>>>(N, vk, w.p, vnext, wkm2, wkm1, w.x, w.pa,
                                                     w.pb, (int)gs, h.tol,
                                                     (long long)h.max_iter, s_in, s_out);
    SINKSLOT_CHECK_LAUNCH();
    if (k % check_every == 0 || k == h.max_iter) {
      Minres hs;
      SINKSLOT_CUDA_TRY(cudaMemcpyAsync(&hs, s_out, sizeof(Minres), cudaMemcpyDeviceToHost, st));
      SINKSLOT_CUDA_TRY(cudaStreamSynchronize(st));
      if (hs.done || k == h.max_iter) {
        *h.iters_host = hs.iters;
        *h.resid_host = hs.beta1 > 0.0 ? hs.resid / hs.beta1 : 0.0;
        break;
      }
    }
  }
  if (h.max_iter <= 0) {
    *h.iters_host = 0;
    *h.resid_host = 1.0;
  }
  hvp_out_kernel<IT><<<blocks_for(n), kHvpThreads, 0, st>>>(op.row, n, h.x, h.y, h.v, h.a, h.d,
                                                             toe, w.x, h.out);
  SINKSLOT_CHECK_LAUNCH();
  if (h.sol_out)
    SINKSLOT_CUDA_TRY(cudaMemcpyAsync(h.sol_out, w.x, N * sizeof(float), cudaMemcpyDeviceToDevice,
                                      st));
  return kOk;
}

}  // namespace

size_t hvp_workspace_bytes(int64_t n, int64_t m) {
  Carver cv(nullptr, 0);
  HvpWs w;
  carve_hvp(cv, w, n + m);
  return cv.used;
}

int hvp(const HvpArgs& h, cudaStream_t st) {
  SINKSLOT_REQUIRE(h.idx_bytes == 2 || h.idx_bytes == 4, "hvp: idx_bytes must be 2 or 4");
  SINKSLOT_REQUIRE(h.d >= 1 && h.d <= kMaxHvpD, "hvp: d must be in [1, 16]");
  SINKSLOT_REQUIRE(h.n >= 1 && h.m >= 1 && h.eps != 0.0, "hvp: bad sizes or eps");
  SINKSLOT_REQUIRE(h.iters_host && h.resid_host && h.out, "hvp: null argument");
  return h.idx_bytes == 2 ? hvp_run<int16_t>(h, st) : hvp_run<int32_t>(h, st);
}

}  // namespace sinkslot
