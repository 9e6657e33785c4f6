// sinkhorn.cu -- fused segmented log-sum-exp half-steps and the solve loops.
//
// One half-step (reference: `_seg_lse_online_kernel`, sinkhorn_solvers.py:45-94,
// and `_seg_lse_coo`, :427-440) computes for every segment s of a CSR/CSC:
//
//     res[s] = base[s] - log sum_{k in s} exp(lam[k] + other[idx[k]])
//
// A group of G lanes (G = 4..32, from the mean segment length) owns one segment,
// streams idx/lam once with evict-first loads (they are read once per half-step;
// the gathered potential stays L2-resident), keeps a running (max, sum) per lane
// and merges the G partial pairs with shuffles.  Fused into the same pass:
//   * the write mode: plain store, the symmetric variant's alpha-blend into a
//     second buffer (sinkhorn_solvers.py:361-363), or no store (check only);
//   * the stop-criterion reduction (sinkhorn_solvers.py:246-288, 373-418): the
//     marginal proxy |a*exp(old-new) - a| or the potential change |new - prev|,
//     max-reduced into one device word per side.
#include <cfloat>
#include <cmath>
#include <string>

#include "common.cuh"
#include "epilogue.cuh"
#include "sinkhorn.h"
#include "tiled.h"

namespace sinkslot {

constexpr int kLseThreads = 256;
constexpr int kLseUnroll = 4;

// One half-step over the segments of a CSR side, by the whole grid: G lanes
// per segment, online max / sum, then the epilogue; the check maxima go to acc.
// ZO: the gathered potential is identically zero (`other` is null): the terms
// are lam + p + 0, the same bits as gathering a zero-filled vector, and the
// index stream is not read at all (the first half-step of every solve).
template <typename IT, int G, int OUT, int CHK, bool ZO>
__device__ __forceinline__ void seg_pass(const int32_t* __restrict__ ptr,
                                         const IT* __restrict__ idx,
                                         const float* __restrict__ lam,
                                         const float* __restrict__ other,
                                         const float* __restrict__ selfpot,
                                         const float* __restrict__ base, const float* self_old,
                                         float* out, int64_t nseg, float w_old, float w_new,
                                         float* prev, uint32_t* acc, const int* __restrict__ list,
                                         const int* __restrict__ list_count, const PeerOut& po) {
  // self_old and out alias in the Gauss-Seidel variant (in-place update): no
  // __restrict__ on either, so the old value is read before the store.
  // With `list`, only the segments list[0 .. *list_count) are computed (the rows
  // the tiled pass handed back).
  const int lane = threadIdx.x & (G - 1);
  const int64_t groups = ((int64_t)gridDim.x * kLseThreads) / G;
  uint32_t chk_bits = 0;
  const int64_t nwork = list ? (int64_t)(*list_count) : nseg;
  // The segment loop is warp-uniform (it steps the warp's first segment) so the
  // full-mask shuffles below always see all 32 lanes; idle groups at the tail
  // run with an empty range and store nothing.
  const int64_t warp_first = ((int64_t)blockIdx.x * kLseThreads + (threadIdx.x & ~31)) / G;
  const int group_in_warp = (threadIdx.x & 31) / G;
  for (int64_t wseg = warp_first; wseg < nwork; wseg += groups) {
    const int64_t slot = wseg + group_in_warp;
    const bool active = slot < nwork;
    const int64_t seg = active ? (list ? (int64_t)list[slot] : slot) : 0;
    const int64_t start = active ? ptr[seg] : 0, end = active ? ptr[seg + 1] : 0;
    // term = (lam + p) + other[idx]: the reference kernel's `v + p + q`, with
    // p = 0 in every solve loop (lam + 0 is exact, so the loops see lam + q)
    const float p = (selfpot && active) ? selfpot[seg] : 0.0f;
    float mx = -INFINITY, sm = 0.0f;
    for (int64_t k0 = start; k0 < end; k0 += G * kLseUnroll) {
      float v[kLseUnroll];
      int64_t kk[kLseUnroll];
      IT ci[kLseUnroll];
      float lv[kLseUnroll];
#pragma unroll
      for (int u = 0; u < kLseUnroll; ++u) {
        kk[u] = k0 + u * G + lane;
        ci[u] = (!ZO && kk[u] < end) ? ld_stream(idx + kk[u]) : IT(0);
        lv[u] = kk[u] < end ? ld_stream(lam + kk[u]) : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < kLseUnroll; ++u)
        v[u] = kk[u] < end ? __fadd_rn(__fadd_rn(lv[u], p),
                                       ZO ? 0.0f : __ldg(other + (int64_t)ci[u]))
                           : -INFINITY;
      float bm = v[0];
#pragma unroll
      for (int u = 1; u < kLseUnroll; ++u) bm = fmaxf(bm, v[u]);
      const float nm = fmaxf(mx, bm);
      if (nm == -INFINITY) continue;
      float s2 = 0.0f;
#pragma unroll
      for (int u = 0; u < kLseUnroll; ++u) s2 += __expf(v[u] - nm);
      sm = sm * __expf(mx - nm) + s2;
      mx = nm;
    }
#pragma unroll
    for (int o = G / 2; o >= 1; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, mx, o, G);
      const float os = __shfl_xor_sync(0xffffffffu, sm, o, G);
      const float nm = fmaxf(mx, om);
      if (nm == -INFINITY) {
        sm = 0.0f;
      } else {
        sm = sm * __expf(mx - nm) + os * __expf(om - nm);
      }
      mx = nm;
    }
    if (lane == 0 && active) {
      const float lse = sm > 0.0f ? mx + logf(fmaxf(sm, FLT_MIN)) : -INFINITY;
      segment_epilogue<OUT, CHK>(seg, lse, base, self_old, out, w_old, w_new, prev, chk_bits,
                                 po);
    }
  }
  check_reduce<CHK>(chk_bits, acc);
}

template <typename IT, int G, int OUT, int CHK>
__global__ void __launch_bounds__(kLseThreads) half_step_kernel(
    const int32_t* __restrict__ ptr, const IT* __restrict__ idx, const float* __restrict__ lam,
    const float* __restrict__ other, const float* __restrict__ selfpot,
    const float* __restrict__ base,
    const float* self_old, float* out, int64_t nseg, float w_old, float w_new, float* prev,
    uint32_t* acc, const int* __restrict__ list, const int* __restrict__ list_count,
    const PeerOut po, unsigned int* done) {
  chain_enter();
  if (other != nullptr)
    seg_pass<IT, G, OUT, CHK, false>(ptr, idx, lam, other, selfpot, base, self_old, out, nseg,
                                     w_old, w_new, prev, acc, list, list_count, po);
  else
    seg_pass<IT, G, OUT, CHK, true>(ptr, idx, lam, other, selfpot, base, self_old, out, nseg,
                                    w_old, w_new, prev, acc, list, list_count, po);
  chain_release();
  if (po.n > 0) {
    __syncthreads();
    peer_cta_done(po, done);
  }
}

static int pick_group(int64_t nnz, int64_t nseg) {
  const int64_t mean = nseg > 0 ? (nnz + nseg - 1) / nseg : 1;
  int g = 4;
  while (g < 32 && (int64_t)g * kLseUnroll < mean) g <<= 1;
  return g;
}

template <typename IT, int G>
static unsigned launch_g(const HalfStep& h, int out_mode, int chk, cudaStream_t st) {
  const int64_t want = ceil_div64(h.nseg * G, kLseThreads);
  // a row-list launch does not know its count on the host: a small persistent
  // grid that exits at once when the list is empty
  const int64_t cap = (int64_t)num_sms() * (h.list ? 4 : 16);
  const unsigned grid = (unsigned)(want < 1 ? 1 : (want > cap ? cap : want));
  const IT* idx = static_cast<const IT*>(h.idx);
  // a failed launch leaves its error for SINKSLOT_CHECK_LAUNCH in half_step
#define SINKSLOT_HS(OUTM, CHKM)                                                               \
  (void)launch_chained(half_step_kernel<IT, G, OUTM, CHKM>, dim3(grid), dim3(kLseThreads), 0, \
                       st, h.ptr, idx, h.lam, h.other, h.selfpot, h.base, h.self_old, h.out,  \
                       h.nseg, h.w_old, h.w_new, h.prev, h.acc, h.list, h.list_count, h.peers, \
                       h.done)
  if (out_mode == kOutPlain) {
    if (chk == kChkNone) SINKSLOT_HS(kOutPlain, kChkNone);
    else if (chk == kChkMarg) SINKSLOT_HS(kOutPlain, kChkMarg);
    else SINKSLOT_HS(kOutPlain, kChkPot);
  } else if (out_mode == kOutBlend) {
    if (chk == kChkNone) SINKSLOT_HS(kOutBlend, kChkNone);
    else if (chk == kChkMarg) SINKSLOT_HS(kOutBlend, kChkMarg);
    else SINKSLOT_HS(kOutBlend, kChkPot);
  } else {
    SINKSLOT_HS(kOutNone, kChkMarg);
  }
#undef SINKSLOT_HS
  return grid;
}

template <typename IT>
static unsigned launch_it(const HalfStep& h, int out_mode, int chk, cudaStream_t st) {
  switch (h.group) {
    case 4: return launch_g<IT, 4>(h, out_mode, chk, st);
    case 8: return launch_g<IT, 8>(h, out_mode, chk, st);
    case 16: return launch_g<IT, 16>(h, out_mode, chk, st);
    default: return launch_g<IT, 32>(h, out_mode, chk, st);
  }
}

int half_step(const HalfStep& h0, int out_mode, int chk, cudaStream_t st, unsigned int* ctas) {
  SINKSLOT_REQUIRE(h0.idx_bytes == 2 || h0.idx_bytes == 4, "half step: idx_bytes must be 2 or 4");
  SINKSLOT_REQUIRE(out_mode != kOutNone || chk == kChkMarg, "half step: check-only needs a check");
  SINKSLOT_REQUIRE(h0.peers.n >= 0 && h0.peers.n <= kMaxPeers && (h0.peers.n == 0 || h0.done),
                   "half step: bad peer outputs");
  if (h0.nseg <= 0) return kOk;
  HalfStep h = h0;
  if (h.group == 0) h.group = pick_group(h.nnz, h.nseg);
  const unsigned grid = h.idx_bytes == 2 ? launch_it<int16_t>(h, out_mode, chk, st)
                                         : launch_it<int32_t>(h, out_mode, chk, st);
  SINKSLOT_CHECK_LAUNCH();
  if (ctas) *ctas += grid;
  return kOk;
}

// --------------------------------------------------------------------------
// Solve loops (host logic mirrors sinkhorn_solvers.py:195-419 exactly:
// iteration counting, check cadence, tol comparisons in double).
// --------------------------------------------------------------------------
static int read_acc(const uint32_t* d_acc, double* a0, double* a1, cudaStream_t st) {
  uint32_t h[2];
  SINKSLOT_CUDA_TRY(cudaMemcpyAsync(h, d_acc, sizeof(h), cudaMemcpyDeviceToHost, st));
  SINKSLOT_CUDA_TRY(cudaStreamSynchronize(st));
  float f0, f1;
  memcpy(&f0, &h[0], 4);
  memcpy(&f1, &h[1], 4);
  *a0 = (double)f0;
  *a1 = (double)f1;
  return kOk;
}

static double py_max(double a, double b) { return (b > a) ? b : a; }  // Python's max(a, b)

// sub-buffers start on 16-byte boundaries (the tiled kernel bulk-copies potentials)
static int64_t pad4(int64_t v) { return (v + 3) & ~int64_t(3); }

size_t solve_work_floats(int64_t n, int64_t m) { return (size_t)(3 * (pad4(n) + pad4(m)) + 64); }

static int read_err(const int* d_err, cudaStream_t st) {
  int h = 0;
  SINKSLOT_CUDA_TRY(cudaMemcpyAsync(&h, d_err, sizeof(int), cudaMemcpyDeviceToHost, st));
  SINKSLOT_CUDA_TRY(cudaStreamSynchronize(st));
  if (h != 0) {
    set_error(h == 4 ? std::string("tiled half-step: the layout was built for another kind or "
                                   "geometry (code 4); build and solve under the same tiles kind")
                     : "tiled half-step: a shared-memory pipeline wait timed out (code " +
                           std::to_string(h) + ")");
    return kCudaError;
  }
  return kOk;
}

int solve_loop(const SolveSpec& sp, float* phi, float* psi, float* work, int64_t work_floats,
               int64_t* iters_run, int* converged, double* final_viol, cudaStream_t st) {
  const int64_t n = sp.row.nseg, m = sp.col.nseg;
  SINKSLOT_REQUIRE(sp.variant == 0 || sp.variant == 1, "solve: variant must be 0 or 1");
  SINKSLOT_REQUIRE(sp.mode >= 0 && sp.mode <= 2, "unknown stop.mode");
  SINKSLOT_REQUIRE(sp.mode == 0 || sp.check_every >= 1, "solve: check_every must be >= 1");
  SINKSLOT_REQUIRE(work_floats >= (int64_t)solve_work_floats(n, m), "solve: work buffer too small");
  // work (each part 16-byte aligned): phi_next (n) | psi_next (m) | prev_phi (n) |
  //       prev_psi (m) | 64 words: [0,1] check maxima, [2,3] handed-back row
  //       counts, [4] pipeline error | handed-back row lists (n, m)
  const int64_t n4 = pad4(n), m4 = pad4(m);
  float* phi_next = work;
  float* psi_next = work + n4;
  float* prev_phi = work + n4 + m4;
  float* prev_psi = work + 2 * n4 + m4;
  uint32_t* acc = reinterpret_cast<uint32_t*>(work + 2 * (n4 + m4));
  int* fb_count = reinterpret_cast<int*>(acc + 2);
  int* perr = reinterpret_cast<int*>(acc + 4);
  int* fb_rows = reinterpret_cast<int*>(work + 2 * (n4 + m4) + 64);
  int* fb_cols = fb_rows + n4;
  SINKSLOT_CUDA_TRY(cudaMemsetAsync(phi, 0, n * sizeof(float), st));
  SINKSLOT_CUDA_TRY(cudaMemsetAsync(psi, 0, m * sizeof(float), st));
  SINKSLOT_CUDA_TRY(cudaMemsetAsync(acc, 0, 8 * sizeof(uint32_t), st));
  if (sp.mode == 1) {
    SINKSLOT_CUDA_TRY(cudaMemsetAsync(prev_phi, 0, n * sizeof(float), st));
    SINKSLOT_CUDA_TRY(cudaMemsetAsync(prev_psi, 0, m * sizeof(float), st));
  }
  const float w_old = (float)(1.0 - sp.alpha), w_new = (float)sp.alpha;

  float* phi_cur = phi;
  float* psi_cur = psi;
  float* phi_nx = phi_next;
  float* psi_nx = psi_next;
  int64_t it = 0;

  // One half-step of either side.  Later iterations run the tiled pass (where a
  // side has a tiled layout) plus the exact pass over the rows it hands back,
  // stabilised by each row's previous log-sum-exp.  The first iteration has no
  // previous log-sum-exp:
  //   * a half-step that gathers the zero start potential (the row side, and
  //     both sides of the symmetric variant) runs the exact kernel without
  //     gathering (its terms are lam itself);
  //   * the alternating variant's first column half-step gathers the fresh
  //     row potential: with a tiled layout, a tiled max pass writes each
  //     column's largest term, and the tiled pass uses those as stabilisers
  //     (every term <= 1, every sum >= 1); without one, the exact kernel.
  auto side_step = [&](bool row, int out_mode, int chk, bool first) -> int {
    const HalfStep& side = row ? sp.row : sp.col;
    float* self_cur = row ? phi_cur : psi_cur;
    float* self_nx = row ? phi_nx : psi_nx;
    const float* other = row ? psi_cur : phi_cur;
    const float* base = row ? sp.log_a : sp.log_b;
    float* prev = row ? prev_phi : prev_psi;
    uint32_t* acc_side = acc + (row ? 0 : 1);
    float* out = sp.variant == 0 ? self_cur : self_nx;  // Gauss-Seidel: in place
    const void* tiles = row ? sp.row_tiles : sp.col_tiles;
    const bool zero_other = first && (row || sp.variant == 1);
    if (tiles != nullptr && (it > 0 || (first && !zero_other))) {
      TiledHalfStep t;
      t.g = row ? sp.row_geom : sp.col_geom;
      t.layout = tiles;
      t.ptr = side.ptr;
      t.idx = side.idx;
      t.idx_bytes = side.idx_bytes;
      t.lam = side.lam;
      t.other = other;
      t.base = base;
      t.self_old = self_cur;
      t.out = out;
      t.w_old = w_old;
      t.w_new = w_new;
      t.prev = prev;
      t.acc = acc_side;
      t.fb_count = fb_count + (row ? 0 : 1);
      t.fb_list = row ? fb_rows : fb_cols;
      t.fb_count_reset = fb_count + (row ? 1 : 0);
      // This side's counter is zeroed by the other side's tiled launch; when the
      // other side runs exact, zero it here.
      if ((row ? sp.col_tiles : sp.row_tiles) == nullptr || it == 0)
        SINKSLOT_CUDA_TRY(cudaMemsetAsync(t.fb_count, 0, sizeof(int), st));
      t.err = perr;
      if (it == 0) {
        // the alternating variant's first column half-step: psi_next is unused
        // by that variant and holds the stabilisers
        t.sigma = self_nx;
        SINKSLOT_TRY(tiled_max_pass(t, self_nx, st));
      }
      return tiled_half_step(t, out_mode, chk, st);
    }
    HalfStep h = side;
    h.other = zero_other ? nullptr : other;
    h.base = base;
    h.prev = prev;
    h.acc = acc_side;
    h.w_old = w_old;
    h.w_new = w_new;
    h.self_old = self_cur;
    h.out = out;
    return half_step(h, out_mode, chk, st);
  };
  // `first`: the iteration's own half-step (false for the symmetric variant's
  // check-only half-steps, which read the blended state)
  auto row_step = [&](int out_mode, int chk, bool first = true) {
    return side_step(true, out_mode, chk, first && it == 0);
  };
  auto col_step = [&](int out_mode, int chk, bool first = true) {
    return side_step(false, out_mode, chk, first && it == 0);
  };
  auto swap_sym = [&]() {
    float* t = phi_cur; phi_cur = phi_nx; phi_nx = t;
    t = psi_cur; psi_cur = psi_nx; psi_nx = t;
  };
  const int step_out = sp.variant == 0 ? kOutPlain : kOutBlend;

  *converged = -1;
  *final_viol = NAN;
  if (sp.mode == 0) {
    for (it = 0; it < sp.n_iters; ++it) {
      SINKSLOT_TRY(row_step(step_out, kChkNone));
      SINKSLOT_TRY(col_step(step_out, kChkNone));
      if (sp.variant == 1) swap_sym();
    }
    it = sp.n_iters < 0 ? 0 : sp.n_iters;
  } else if (sp.mode == 1) {
    double change = INFINITY;
    *converged = 0;
    const double thr = sp.variant == 0 ? sp.tol : sp.alpha * sp.tol;
    while (it < sp.max_iter) {
      const bool chk = ((it + 1) % sp.check_every) == 0;
      if (chk) SINKSLOT_CUDA_TRY(cudaMemsetAsync(acc, 0, 2 * sizeof(uint32_t), st));
      SINKSLOT_TRY(row_step(step_out, chk ? kChkPot : kChkNone));
      SINKSLOT_TRY(col_step(step_out, chk ? kChkPot : kChkNone));
      if (sp.variant == 1) swap_sym();
      ++it;
      if (chk) {
        double c0, c1;
        SINKSLOT_TRY(read_acc(acc, &c0, &c1, st));
        change = sp.eps * py_max(c0, c1);
        if (change < thr) {
          *converged = 1;
          break;
        }
      }
    }
    *final_viol = change;
  } else {
    double v = INFINITY;
    *converged = 0;
    while (it < sp.max_iter) {
      const bool chk = ((it + 1) % sp.check_every) == 0 || (it + 1) == sp.max_iter;
      if (chk) SINKSLOT_CUDA_TRY(cudaMemsetAsync(acc, 0, 2 * sizeof(uint32_t), st));
      if (sp.variant == 0) {
        SINKSLOT_TRY(row_step(kOutPlain, chk ? kChkMarg : kChkNone));
        SINKSLOT_TRY(col_step(kOutPlain, chk ? kChkMarg : kChkNone));
      } else {
        SINKSLOT_TRY(row_step(kOutBlend, kChkNone));
        SINKSLOT_TRY(col_step(kOutBlend, kChkNone));
        swap_sym();
        if (chk) {
          SINKSLOT_TRY(row_step(kOutNone, kChkMarg, false));
          SINKSLOT_TRY(col_step(kOutNone, kChkMarg, false));
        }
      }
      ++it;
      if (chk) {
        double c0, c1;
        SINKSLOT_TRY(read_acc(acc, &c0, &c1, st));
        // torch.maximum propagates NaN
        v = (std::isnan(c0) || std::isnan(c1)) ? NAN : (c0 > c1 ? c0 : c1);
        if (v <= sp.tol) {
          *converged = 1;
          break;
        }
      }
    }
    *final_viol = v;
  }
  if (phi_cur != phi)
    SINKSLOT_CUDA_TRY(cudaMemcpyAsync(phi, phi_cur, n * sizeof(float), cudaMemcpyDeviceToDevice, st));
  if (psi_cur != psi)
    SINKSLOT_CUDA_TRY(cudaMemcpyAsync(psi, psi_cur, m * sizeof(float), cudaMemcpyDeviceToDevice, st));
  *iters_run = it;
  if (sp.row_tiles || sp.col_tiles) return read_err(perr, st);
  return kOk;
}

}  // namespace sinkslot
