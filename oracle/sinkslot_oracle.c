/*
 * sinkslot_oracle.c -- CPU restatement of the SinkSLOT sparse-Sinkhorn path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity oracle for the sm_100a
 * kernels in sinkslot_b200/csrc.  Only the test suite, the smoke check and the
 * CPU-baseline / reference arm of bench.py may load it, and only as the
 * checker or as the timed CPU reference -- never as the product path.
 *
 * It restates, in plain C, the algorithm of the reference package
 * (cai4cai/SinkSLOT, torch-ext/sinkslot/), following each torch op's
 * arithmetic:
 *
 *   orc_project            solver.py:221          PX = X @ theta^T   (sequential FMA chain over d)
 *   orc_ot1d_*             solver.py:55-150       1-D north-west-corner couplings, C slices
 *   orc_coalesce           solver.py:194-232      key = r*m + c, unique + index_add_, / L
 *   orc_sqeuclid_cost      solver.py:346          (x[rows]-y[cols]).square().sum(1)
 *   orc_seg_lse_*          sinkhorn_solvers.py:427-440  _seg_lse_coo (amax, index_add_ of exp)
 *   orc_solve              sinkhorn_solvers.py:443-588  torch-backend loops, all stop modes
 *   orc_plan_values        sinkhorn_solvers.py:755-760
 *   orc_barycentric        gradient.py:50-61
 *
 * Sort semantics: the reference's CUDA builder sorts with CUB radix sort
 * (stable; -0.0 and +0.0 compare equal).  The oracle sorts stably with the
 * same tie rule.  Cumsum: two association orders are restated --
 *   CUMSUM_TORCH_CUDA: torch's innermost-dim Sklansky scan (chunks of
 *     2*2^k elements, k from get_log_num_threads_x_inner_scan(C, n)),
 *     ATen/native/cuda/ScanUtils.cuh (torch 2.11 headers);
 *   CUMSUM_TORCH_CPU:  double accumulator rounded to float per element
 *     (torch CPU cumsum, the reference's naive builder on CPU tensors).
 *
 * The Sinkhorn loops are parallel over segments (OpenMP).  Each segment is
 * summed sequentially in COO order, which is exactly the order of the
 * reference's CPU index_add_, so the thread count does not change results.
 */
#include <math.h>
#include <float.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define CUMSUM_TORCH_CUDA 0
#define CUMSUM_TORCH_CPU 1

#define EMIT_SLICE_MAJOR 0 /* _ot_1d_coo_batched_cuda: (C, n+m) flattened */
#define EMIT_POSITION_MAJOR 1 /* _ot_1d_coo_batched: (n+m, C)[keep] row-major */

/* ------------------------------------------------------------------------ */
/* projection: solver.py:221  PX = X @ th.T                                  */
/* The product is the sequential FMA chain fma(x_{d-1},t_{d-1},...fma(x1,t1, */
/* x0*t0)); MKL (CPU) and cuBLAS (K=d) produce the same bits.                 */
/* ------------------------------------------------------------------------ */
void orc_project(const float *X, int64_t n, int d, const float *theta, int L,
                 float *out /* (L, n) */) {
#pragma omp parallel for schedule(static)
  for (int c = 0; c < L; ++c) {
    const float *t = theta + (int64_t)c * d;
    float *o = out + (int64_t)c * n;
    for (int64_t i = 0; i < n; ++i) {
      const float *x = X + i * d;
      float acc = x[0] * t[0];
      for (int j = 1; j < d; ++j) acc = fmaf(x[j], t[j], acc);
      o[i] = acc;
    }
  }
}

/* ------------------------------------------------------------------------ */
/* stable argsort, ascending, -0.0 == +0.0 (CUB radix-sort semantics)        */
/* ------------------------------------------------------------------------ */
static void merge_sort_idx(const float *v, int32_t *idx, int32_t *tmp, int64_t n) {
  /* bottom-up stable merge sort on indices */
  int32_t *src = idx, *dst = tmp;
  for (int64_t w = 1; w < n; w *= 2) {
    for (int64_t lo = 0; lo < n; lo += 2 * w) {
      int64_t mid = lo + w < n ? lo + w : n;
      int64_t hi = lo + 2 * w < n ? lo + 2 * w : n;
      int64_t i = lo, j = mid, k = lo;
      while (i < mid && j < hi) {
        /* take right only if strictly smaller: stability */
        if (v[src[j]] < v[src[i]]) dst[k++] = src[j++];
        else dst[k++] = src[i++];
      }
      while (i < mid) dst[k++] = src[i++];
      while (j < hi) dst[k++] = src[j++];
    }
    int32_t *t = src; src = dst; dst = t;
  }
  if (src != idx) memcpy(idx, src, (size_t)n * sizeof(int32_t));
}

void orc_stable_argsort_f32(const float *v, int64_t n, int32_t *idx) {
  int32_t *tmp = (int32_t *)malloc((size_t)(n > 0 ? n : 1) * sizeof(int32_t));
  for (int64_t i = 0; i < n; ++i) idx[i] = (int32_t)i;
  merge_sort_idx(v, idx, tmp, n);
  free(tmp);
}

/* ------------------------------------------------------------------------ */
/* cumsum association orders                                                 */
/* ------------------------------------------------------------------------ */
/* ATen get_log_num_threads_x_inner_scan<uint32_t>(num_rows, row_size),
 * unsigned arithmetic included (the wrap when rows >> row_size). */
uint32_t orc_torch_inner_scan_log_tx(uint32_t num_rows, uint32_t row_size) {
  uint32_t lx = 0, ly = 0;
  while (((uint32_t)1 << lx) < row_size) ++lx;
  while (((uint32_t)1 << ly) < num_rows) ++ly;
  uint32_t diff = lx - ly;
  lx = ((uint32_t)9 + diff) / (uint32_t)2;
  if (lx < 4) lx = 4;
  if (lx > 9) lx = 9;
  return lx;
}

/* torch CUDA inclusive scan along the innermost dim (Sklansky per chunk of
 * 2*2^log_tx elements, running total folded into the chunk's first element). */
static void cumsum_torch_cuda(const float *w, int64_t n, uint32_t log_tx, float *out,
                              float *buf) {
  const int64_t tx = (int64_t)1 << log_tx;
  const int64_t chunk = 2 * tx;
  float total = 0.0f;
  for (int64_t base = 0; base < n; base += chunk) {
    for (int64_t t = 0; t < chunk; ++t) buf[t] = (base + t < n) ? w[base + t] : 0.0f;
    buf[0] = buf[0] + total;
    for (uint32_t mm = 0; mm <= log_tx; ++mm) {
      const uint32_t s = 1u << mm;
      for (uint32_t th = 0; th < (uint32_t)tx; ++th) {
        uint32_t a = ((th >> mm) << (mm + 1)) | s;
        uint32_t ti = a + (th % s);
        uint32_t si = a - 1;
        buf[ti] = buf[ti] + buf[si];
      }
    }
    for (int64_t t = 0; t < chunk && base + t < n; ++t) out[base + t] = buf[t];
    total = buf[chunk - 1];
  }
}

static void cumsum_torch_cpu(const float *w, int64_t n, float *out) {
  double acc = 0.0;
  for (int64_t i = 0; i < n; ++i) {
    acc += (double)w[i];
    out[i] = (float)acc;
  }
}

/* scan of one slice's gathered weights; C = number of slices in the call
 * (torch picks the CUDA block shape from it; C == 1 takes CUB's device scan,
 * whose order is not restated here -- a sequential fp32 scan stands in). */
static void slice_cumsum(const float *w, int64_t n, int C, int mode, float *out, float *buf) {
  if (mode == CUMSUM_TORCH_CPU) {
    cumsum_torch_cpu(w, n, out);
  } else if (C == 1) {
    float acc = 0.0f;
    for (int64_t i = 0; i < n; ++i) { acc = acc + w[i]; out[i] = acc; }
  } else {
    cumsum_torch_cuda(w, n, orc_torch_inner_scan_log_tx((uint32_t)C, (uint32_t)n), out, buf);
  }
}

void orc_cumsum(const float *w, int64_t n, int C, int mode, float *out) {
  float *buf = (float *)malloc(1024 * sizeof(float));
  slice_cumsum(w, n, C, mode, out, buf);
  free(buf);
}

/* searchsorted on a non-decreasing array: left = #{s < v}, right = #{s <= v} */
static int64_t ss_left(const float *s, int64_t n, float v) {
  int64_t lo = 0, hi = n;
  while (lo < hi) { int64_t mid = (lo + hi) >> 1; if (s[mid] < v) lo = mid + 1; else hi = mid; }
  return lo;
}
static int64_t ss_right(const float *s, int64_t n, float v) {
  int64_t lo = 0, hi = n;
  while (lo < hi) { int64_t mid = (lo + hi) >> 1; if (s[mid] <= v) lo = mid + 1; else hi = mid; }
  return lo;
}

/* ------------------------------------------------------------------------ */
/* 1-D couplings for C slices (solver.py:107-150 / 55-104)                   */
/* PXt: (C, n), PYt: (C, m) projections (slice-major).  Writes the kept      */
/* (R, Cc, mass) triples in the requested emission order and returns their   */
/* count.  Capacity of the outputs: C * (n + m).                             */
/* ------------------------------------------------------------------------ */
int64_t orc_ot1d(const float *PXt, const float *PYt, int64_t n, int64_t m, int C,
                 const float *a, const float *b, int cum_mode, int emit_order,
                 int64_t *R, int64_t *Cc, float *mass_out, int scan_rows) {
  const int64_t nm = n + m;
  /* the cumsum association of a batch of scan_rows slices (0: this call's C) */
  const int scan_c = scan_rows > 0 ? scan_rows : C;
  /* per-slice full arrays (position-major emission needs them all) */
  int64_t *allR = (int64_t *)malloc((size_t)C * nm * sizeof(int64_t));
  int64_t *allC = (int64_t *)malloc((size_t)C * nm * sizeof(int64_t));
  float *allM = (float *)malloc((size_t)C * nm * sizeof(float));

#pragma omp parallel
  {
    int32_t *ix = (int32_t *)malloc((size_t)n * sizeof(int32_t));
    int32_t *iy = (int32_t *)malloc((size_t)m * sizeof(int32_t));
    float *wa = (float *)malloc((size_t)n * sizeof(float));
    float *wb = (float *)malloc((size_t)m * sizeof(float));
    float *ca = (float *)malloc((size_t)n * sizeof(float));
    float *cb = (float *)malloc((size_t)m * sizeof(float));
    float *bounds = (float *)malloc((size_t)nm * sizeof(float));
    float *buf = (float *)malloc(1024 * sizeof(float));
#pragma omp for schedule(dynamic, 1)
    for (int c = 0; c < C; ++c) {
      orc_stable_argsort_f32(PXt + (int64_t)c * n, n, ix);
      orc_stable_argsort_f32(PYt + (int64_t)c * m, m, iy);
      for (int64_t i = 0; i < n; ++i) wa[i] = a[ix[i]];
      for (int64_t j = 0; j < m; ++j) wb[j] = b[iy[j]];
      slice_cumsum(wa, n, scan_c, cum_mode, ca, buf);
      slice_cumsum(wb, m, scan_c, cum_mode, cb, buf);
      /* rank_a = i + searchsorted(cb, ca, right=True); rank_b = j + searchsorted(ca, cb, left) */
      for (int64_t i = 0; i < n; ++i) bounds[i + ss_right(cb, m, ca[i])] = ca[i];
      for (int64_t j = 0; j < m; ++j) bounds[j + ss_left(ca, n, cb[j])] = cb[j];
      float prev = 0.0f;
      for (int64_t k = 0; k < nm; ++k) {
        const float bnd = bounds[k];
        const float ms = bnd - prev;
        const float mid = 0.5f * (prev + bnd);
        int64_t ii = ss_left(ca, n, mid);
        int64_t jj = ss_left(cb, m, mid);
        if (ii > n - 1) ii = n - 1;
        if (jj > m - 1) jj = m - 1;
        allR[(int64_t)c * nm + k] = ix[ii];
        allC[(int64_t)c * nm + k] = iy[jj];
        allM[(int64_t)c * nm + k] = ms;
        prev = bnd;
      }
    }
    free(ix); free(iy); free(wa); free(wb); free(ca); free(cb); free(bounds); free(buf);
  }

  int64_t cnt = 0;
  if (emit_order == EMIT_SLICE_MAJOR) {
    for (int c = 0; c < C; ++c)
      for (int64_t k = 0; k < nm; ++k) {
        const int64_t q = (int64_t)c * nm + k;
        if (allM[q] > 0.0f) { R[cnt] = allR[q]; Cc[cnt] = allC[q]; mass_out[cnt] = allM[q]; ++cnt; }
      }
  } else {
    for (int64_t k = 0; k < nm; ++k)
      for (int c = 0; c < C; ++c) {
        const int64_t q = (int64_t)c * nm + k;
        if (allM[q] > 0.0f) { R[cnt] = allR[q]; Cc[cnt] = allC[q]; mass_out[cnt] = allM[q]; ++cnt; }
      }
  }
  free(allR); free(allC); free(allM);
  return cnt;
}

/* ------------------------------------------------------------------------ */
/* coalesce (solver.py:196-206, 228-232): sort by key r*m+c (stable), sum    */
/* duplicates in raw order (CPU index_add_ order), then divide by L.         */
/* div_mode 0: v / L (CPU true division); 1: v * (1/L) (CUDA scalar div).    */
/* Returns the unique count; outputs sized >= nraw.                          */
/* ------------------------------------------------------------------------ */
static void radix_sort_keys_idx(uint64_t *key, int64_t *idx, int64_t n) {
  uint64_t *k2 = (uint64_t *)malloc((size_t)(n ? n : 1) * sizeof(uint64_t));
  int64_t *i2 = (int64_t *)malloc((size_t)(n ? n : 1) * sizeof(int64_t));
  uint64_t maxk = 0;
  for (int64_t i = 0; i < n; ++i) if (key[i] > maxk) maxk = key[i];
  for (int shift = 0; shift < 64 && (shift == 0 || (maxk >> shift)); shift += 16) {
    int64_t *cnt = (int64_t *)calloc(65537, sizeof(int64_t));
    for (int64_t i = 0; i < n; ++i) cnt[((key[i] >> shift) & 0xFFFF) + 1]++;
    for (int t = 0; t < 65536; ++t) cnt[t + 1] += cnt[t];
    for (int64_t i = 0; i < n; ++i) {
      int64_t p = cnt[(key[i] >> shift) & 0xFFFF]++;
      k2[p] = key[i]; i2[p] = idx[i];
    }
    memcpy(key, k2, (size_t)n * sizeof(uint64_t));
    memcpy(idx, i2, (size_t)n * sizeof(int64_t));
    free(cnt);
  }
  free(k2); free(i2);
}

int64_t orc_coalesce(const int64_t *R, const int64_t *Cc, const float *v, int64_t nraw,
                     int64_t m, int L, int div_mode, int64_t *rows, int64_t *cols, float *S) {
  uint64_t *key = (uint64_t *)malloc((size_t)(nraw ? nraw : 1) * sizeof(uint64_t));
  int64_t *idx = (int64_t *)malloc((size_t)(nraw ? nraw : 1) * sizeof(int64_t));
  for (int64_t i = 0; i < nraw; ++i) { key[i] = (uint64_t)(R[i] * m + Cc[i]); idx[i] = i; }
  radix_sort_keys_idx(key, idx, nraw); /* LSD radix: stable */
  int64_t u = -1;
  for (int64_t i = 0; i < nraw; ++i) {
    if (i == 0 || key[i] != key[i - 1]) {
      ++u;
      rows[u] = (int64_t)(key[i] / (uint64_t)m);
      cols[u] = (int64_t)(key[i] % (uint64_t)m);
      S[u] = 0.0f;
    }
    S[u] = S[u] + v[idx[i]];
  }
  const int64_t nu = u + 1;
  const float Lf = (float)L;
  const float invL = 1.0f / Lf;
  for (int64_t i = 0; i < nu; ++i) S[i] = div_mode ? S[i] * invL : S[i] / Lf;
  free(key); free(idx);
  return nu;
}

/* ------------------------------------------------------------------------ */
/* cost: solver.py:346  (x[rows]-y[cols]).square().sum(1)                   */
/* ------------------------------------------------------------------------ */
void orc_sqeuclid_cost(const float *x, const float *y, int d, const int64_t *rows,
                       const int64_t *cols, int64_t nnz, float *out) {
#pragma omp parallel for schedule(static)
  for (int64_t k = 0; k < nnz; ++k) {
    const float *xr = x + rows[k] * d, *yc = y + cols[k] * d;
    float s = 0.0f;
    for (int j = 0; j < d; ++j) {
      const float t = xr[j] - yc[j];
      const float sq = t * t;
      s = s + sq;
    }
    out[k] = s;
  }
}

/* lam = log(S.clamp_min(tiny)) - cost / eps   (sinkhorn_solvers.py:700) */
void orc_lam(const float *S, const float *cost, int64_t nnz, double eps, float *lam) {
  const float e = (float)eps;
#pragma omp parallel for schedule(static)
  for (int64_t k = 0; k < nnz; ++k) {
    const float s = S[k] < FLT_MIN ? FLT_MIN : S[k];
    lam[k] = logf(s) - cost[k] / e;
  }
}

/* ------------------------------------------------------------------------ */
/* segmented LSE over a COO axis, sequential within a segment in COO order  */
/* (sinkhorn_solvers.py:427-440).  seg_ptr/seg_ent: the COO entries grouped */
/* by segment, preserving COO order (a stable grouping).                    */
/*   out[s] = base[s] - LSE_{k in s}(lam[k] + other[oidx[k]])               */
/* ------------------------------------------------------------------------ */
static void seg_half_step(const int64_t *seg_ptr, const int64_t *seg_ent, const float *lam,
                          const int64_t *oidx, const float *other, const float *base,
                          int64_t nseg, float *out) {
#pragma omp parallel for schedule(dynamic, 256)
  for (int64_t s = 0; s < nseg; ++s) {
    const int64_t lo = seg_ptr[s], hi = seg_ptr[s + 1];
    float mx = -INFINITY;
    for (int64_t t = lo; t < hi; ++t) {
      const int64_t k = seg_ent[t];
      const float v = lam[k] + other[oidx[k]];
      if (!isnan(mx) && (isnan(v) || v > mx)) mx = v;
    }
    float acc = 0.0f;
    for (int64_t t = lo; t < hi; ++t) {
      const int64_t k = seg_ent[t];
      const float v = lam[k] + other[oidx[k]];
      acc = acc + expf(v - mx);
    }
    float lse;
    if (acc > 0.0f) lse = mx + logf(acc < FLT_MIN ? FLT_MIN : acc);
    else lse = -INFINITY;
    out[s] = base[s] - lse;
  }
}

/* stable grouping of COO entries by an index array (counting sort) */
static void group_by(const int64_t *key, int64_t nnz, int64_t nseg, int64_t *ptr, int64_t *ent) {
  memset(ptr, 0, (size_t)(nseg + 1) * sizeof(int64_t));
  for (int64_t k = 0; k < nnz; ++k) ptr[key[k] + 1]++;
  for (int64_t s = 0; s < nseg; ++s) ptr[s + 1] += ptr[s];
  int64_t *fill = (int64_t *)malloc((size_t)(nseg + 1) * sizeof(int64_t));
  memcpy(fill, ptr, (size_t)(nseg + 1) * sizeof(int64_t));
  for (int64_t k = 0; k < nnz; ++k) ent[fill[key[k]]++] = k;
  free(fill);
}

typedef struct {
  int64_t *rptr, *rent, *cptr, *cent;
} orc_layout;

static void layout_build(orc_layout *lo, const int64_t *rows, const int64_t *cols, int64_t nnz,
                         int64_t n, int64_t m) {
  lo->rptr = (int64_t *)malloc((size_t)(n + 1) * sizeof(int64_t));
  lo->cptr = (int64_t *)malloc((size_t)(m + 1) * sizeof(int64_t));
  lo->rent = (int64_t *)malloc((size_t)(nnz ? nnz : 1) * sizeof(int64_t));
  lo->cent = (int64_t *)malloc((size_t)(nnz ? nnz : 1) * sizeof(int64_t));
  group_by(rows, nnz, n, lo->rptr, lo->rent);
  group_by(cols, nnz, m, lo->cptr, lo->cent);
}
static void layout_free(orc_layout *lo) {
  free(lo->rptr); free(lo->rent); free(lo->cptr); free(lo->cent);
}

/* phi <- log_a - LSE(lam + psi[cols]) by rows; psi likewise by cols */
void orc_seg_lse_coo(const int64_t *idx_self, const int64_t *idx_other, const float *lam,
                     int64_t nnz, const float *other, const float *base, int64_t nseg,
                     float *out) {
  int64_t *ptr = (int64_t *)malloc((size_t)(nseg + 1) * sizeof(int64_t));
  int64_t *ent = (int64_t *)malloc((size_t)(nnz ? nnz : 1) * sizeof(int64_t));
  group_by(idx_self, nnz, nseg, ptr, ent);
  seg_half_step(ptr, ent, lam, idx_other, other, base, nseg, out);
  free(ptr); free(ent);
}

static float max_abs_diff(const float *p, const float *q, int64_t n) {
  float r = 0.0f; int seen = 0;
  for (int64_t i = 0; i < n; ++i) {
    const float d = fabsf(p[i] - q[i]);
    if (isnan(d)) return NAN;
    if (!seen || d > r) { r = d; seen = 1; }
  }
  return r;
}

/* max |a*exp(old-new) - a| in fp32 (sinkhorn_solvers.py:577-580) */
static float marg_viol(const float *a, const float *oldp, const float *newp, int64_t n) {
  float r = 0.0f; int seen = 0;
  for (int64_t i = 0; i < n; ++i) {
    const float t = a[i] * expf(oldp[i] - newp[i]);
    const float d = fabsf(t - a[i]);
    if (isnan(d)) return NAN;
    if (!seen || d > r) { r = d; seen = 1; }
  }
  return r;
}

static double fmax_nan(double x, double y) {
  if (isnan(x) || isnan(y)) return NAN;
  return x > y ? x : y;
}

/* ------------------------------------------------------------------------ */
/* torch-backend solve loops (sinkhorn_solvers.py:443-588)                   */
/* variant: 0 alternating, 1 symmetric.  mode: 0 fixed, 1 potential,         */
/* 2 marginal.  Returns iterations run; *converged: -1 none, 0/1; *viol:     */
/* NAN when not defined (fixed mode).                                        */
/* ------------------------------------------------------------------------ */
int64_t orc_solve(const int64_t *rows, const int64_t *cols, const float *lam, int64_t nnz,
                  const float *log_a, const float *log_b, int64_t n, int64_t m, int variant,
                  int mode, int64_t n_iters, int64_t max_iter, int64_t check_every, double tol,
                  double eps, double alpha, float *phi, float *psi, int *converged,
                  double *viol) {
  orc_layout lo;
  layout_build(&lo, rows, cols, nnz, n, m);
  float *pc = (float *)malloc((size_t)(n ? n : 1) * sizeof(float));
  float *qc = (float *)malloc((size_t)(m ? m : 1) * sizeof(float));
  float *p0 = (float *)malloc((size_t)(n ? n : 1) * sizeof(float));
  float *q0 = (float *)malloc((size_t)(m ? m : 1) * sizeof(float));
  float *ea = (float *)malloc((size_t)(n ? n : 1) * sizeof(float));
  float *eb = (float *)malloc((size_t)(m ? m : 1) * sizeof(float));
  for (int64_t i = 0; i < n; ++i) phi[i] = 0.0f;
  for (int64_t j = 0; j < m; ++j) psi[j] = 0.0f;
  for (int64_t i = 0; i < n; ++i) ea[i] = expf(log_a[i]);
  for (int64_t j = 0; j < m; ++j) eb[j] = expf(log_b[j]);
  const float w_old = (float)(1.0 - alpha), w_new = (float)alpha;
  int64_t it = 0;
  *converged = -1;
  *viol = NAN;

#define ROW_STEP(dst, psrc) seg_half_step(lo.rptr, lo.rent, lam, cols, psrc, log_a, n, dst)
#define COL_STEP(dst, psrc) seg_half_step(lo.cptr, lo.cent, lam, rows, psrc, log_b, m, dst)
#define BLEND()                                                                       \
  do {                                                                                \
    for (int64_t i = 0; i < n; ++i) phi[i] = w_old * phi[i] + w_new * pc[i];          \
    for (int64_t j = 0; j < m; ++j) psi[j] = w_old * psi[j] + w_new * qc[j];          \
  } while (0)

  if (mode == 0) {
    for (it = 0; it < n_iters; ++it) {
      if (variant == 0) {
        ROW_STEP(pc, psi); memcpy(phi, pc, (size_t)n * sizeof(float));
        COL_STEP(qc, phi); memcpy(psi, qc, (size_t)m * sizeof(float));
      } else {
        ROW_STEP(pc, psi); COL_STEP(qc, phi); BLEND();
      }
    }
    it = n_iters;
  } else if (mode == 1) {
    memcpy(p0, phi, (size_t)n * sizeof(float));
    memcpy(q0, psi, (size_t)m * sizeof(float));
    double change = INFINITY;
    *converged = 0;
    const double thr = variant == 0 ? tol : alpha * tol;
    while (it < max_iter) {
      if (variant == 0) {
        ROW_STEP(pc, psi); memcpy(phi, pc, (size_t)n * sizeof(float));
        COL_STEP(qc, phi); memcpy(psi, qc, (size_t)m * sizeof(float));
      } else {
        ROW_STEP(pc, psi); COL_STEP(qc, phi); BLEND();
      }
      ++it;
      if (it % check_every == 0) {
        change = eps * fmax_nan((double)max_abs_diff(phi, p0, n), (double)max_abs_diff(psi, q0, m));
        if (change < thr) { *converged = 1; break; }
        memcpy(p0, phi, (size_t)n * sizeof(float));
        memcpy(q0, psi, (size_t)m * sizeof(float));
      }
    }
    *viol = change;
  } else {
    double v = INFINITY;
    *converged = 0;
    while (it < max_iter) {
      if (variant == 0) {
        memcpy(p0, phi, (size_t)n * sizeof(float));
        memcpy(q0, psi, (size_t)m * sizeof(float));
        ROW_STEP(pc, psi); memcpy(phi, pc, (size_t)n * sizeof(float));
        COL_STEP(qc, phi); memcpy(psi, qc, (size_t)m * sizeof(float));
      } else {
        ROW_STEP(pc, psi); COL_STEP(qc, phi); BLEND();
      }
      ++it;
      if (it % check_every == 0 || it == max_iter) {
        if (variant == 0) {
          v = fmax_nan((double)marg_viol(ea, p0, phi, n), (double)marg_viol(eb, q0, psi, m));
        } else {
          ROW_STEP(pc, psi); COL_STEP(qc, phi);
          v = fmax_nan((double)marg_viol(ea, phi, pc, n), (double)marg_viol(eb, psi, qc, m));
        }
        if (v <= tol) { *converged = 1; break; }
      }
    }
    *viol = v;
  }
#undef ROW_STEP
#undef COL_STEP
#undef BLEND
  free(pc); free(qc); free(p0); free(q0); free(ea); free(eb);
  layout_free(&lo);
  return it;
}

/* Prebuilt layout + fixed-mode alternating iterations, for timing the
 * iteration alone (the CPU baseline): same arithmetic as orc_solve. */
void *orc_layout_new(const int64_t *rows, const int64_t *cols, int64_t nnz, int64_t n, int64_t m) {
  orc_layout *lo = (orc_layout *)malloc(sizeof(orc_layout));
  layout_build(lo, rows, cols, nnz, n, m);
  return lo;
}
void orc_layout_free(void *h) {
  if (!h) return;
  layout_free((orc_layout *)h);
  free(h);
}
void orc_iterate_alternating(void *h, const int64_t *rows, const int64_t *cols, const float *lam,
                             const float *log_a, const float *log_b, int64_t n, int64_t m,
                             int64_t iters, float *phi, float *psi) {
  orc_layout *lo = (orc_layout *)h;
  for (int64_t it = 0; it < iters; ++it) {
    seg_half_step(lo->rptr, lo->rent, lam, cols, psi, log_a, n, phi);
    seg_half_step(lo->cptr, lo->cent, lam, rows, phi, log_b, m, psi);
  }
}

/* ------------------------------------------------------------------------ */
/* plan values, sinkhorn_solvers.py:757-758:                                 */
/*   exp(phi[r] + psi[c] + log_S - cost/eps)                                  */
/* and the gradient's T_vals, gradient.py:95-97:                              */
/*   exp(phi[r] + psi[c] + (log_S - cost/eps))                                */
/* ------------------------------------------------------------------------ */
void orc_plan_values(const float *phi, const float *psi, const int64_t *rows,
                     const int64_t *cols, const float *S, const float *cost, int64_t nnz,
                     double eps, int grad_form, float *out) {
  const float e = (float)eps;
#pragma omp parallel for schedule(static)
  for (int64_t k = 0; k < nnz; ++k) {
    const float s = S[k] < FLT_MIN ? FLT_MIN : S[k];
    const float ls = logf(s);
    const float ce = cost[k] / e;
    float v;
    if (grad_form) v = (phi[rows[k]] + psi[cols[k]]) + (ls - ce);
    else v = ((phi[rows[k]] + psi[cols[k]]) + ls) - ce;
    out[k] = expf(v);
  }
}

/* barycentric map Tx (gradient.py:52-59), sums in COO order per row;
 * grad = 2*a*(x - Tx) (gradient.py:99).  Tx and grad are (n, d). */
void orc_barycentric(const float *T, const int64_t *rows, const int64_t *cols, int64_t nnz,
                     const float *x, const float *y, int64_t n, int64_t m, int d,
                     const float *a, float *Tx, float *grad) {
  int64_t *ptr = (int64_t *)malloc((size_t)(n + 1) * sizeof(int64_t));
  int64_t *ent = (int64_t *)malloc((size_t)(nnz ? nnz : 1) * sizeof(int64_t));
  group_by(rows, nnz, n, ptr, ent);
  (void)m;
#pragma omp parallel for schedule(dynamic, 256)
  for (int64_t i = 0; i < n; ++i) {
    float r = 0.0f;
    float acc[64];
    for (int j = 0; j < d && j < 64; ++j) acc[j] = 0.0f;
    for (int64_t t = ptr[i]; t < ptr[i + 1]; ++t) {
      const int64_t k = ent[t];
      r = r + T[k];
      for (int j = 0; j < d; ++j) acc[j] = acc[j] + T[k] * y[cols[k] * d + j];
    }
    const float den = r < FLT_MIN ? FLT_MIN : r;
    for (int j = 0; j < d; ++j) {
      const float tx = acc[j] / den;
      Tx[i * d + j] = tx;
      if (grad) grad[i * d + j] = (2.0f * a[i]) * (x[i * d + j] - tx);
    }
  }
  free(ptr); free(ent);
}

/* column-side barycentric map Ty (gradient.py:54-60) */
void orc_barycentric_cols(const float *T, const int64_t *rows, const int64_t *cols,
                          int64_t nnz, const float *x, int64_t m, int d, float *Ty) {
  int64_t *ptr = (int64_t *)malloc((size_t)(m + 1) * sizeof(int64_t));
  int64_t *ent = (int64_t *)malloc((size_t)(nnz ? nnz : 1) * sizeof(int64_t));
  group_by(cols, nnz, m, ptr, ent);
#pragma omp parallel for schedule(dynamic, 256)
  for (int64_t j = 0; j < m; ++j) {
    float r = 0.0f;
    float acc[64];
    for (int q = 0; q < d && q < 64; ++q) acc[q] = 0.0f;
    for (int64_t t = ptr[j]; t < ptr[j + 1]; ++t) {
      const int64_t k = ent[t];
      r = r + T[k];
      for (int q = 0; q < d; ++q) acc[q] = acc[q] + T[k] * x[rows[k] * d + q];
    }
    const float den = r < FLT_MIN ? FLT_MIN : r;
    for (int q = 0; q < d; ++q) Ty[j * d + q] = acc[q] / den;
  }
  free(ptr); free(ent);
}

int orc_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
