// support.cu -- sliced-lifted support construction on sm_100a.
//
// Restates the reference's CUDA builder (solver.py:107-150, `_ot_1d_coo_batched_cuda`)
// and coalesce (solver.py:194-232) with hand-written kernels:
//
//   project_keys_kernel    PX = X @ theta^T as the sequential fp32 FMA chain over d
//                          (what cuBLAS computes for K = d), written as radix keys
//   radix_sort_pairs       per-slice stable argsort (CUB semantics: stable, -0 == +0)
//   chunk_*_kernel         cumsum(a[ix]) in torch's CUDA innermost-dim scan order
//                          (Sklansky chunks, ATen/native/cuda/ScanUtils.cuh),
//                          chunks in parallel around a per-row carry chain
//   merge_count/emit       rank merge of the two cumsums + midpoint searchsorted,
//                          as one merge-path walk (replaces 4 searchsorted + 2 scatters)
//   radix_sort_pairs<u64>  stable sort of raw keys r*m+c
//   head/run_sum kernels   unique + in-order duplicate sum, S = sum * (1/L)
//
// Every float operation that decides the support (cumsum adds, bounds - prev,
// 0.5 * (prev + bounds)) is written with explicit round-to-nearest intrinsics so
// no FMA contraction can change a bit.
#include <algorithm>
#include <cfloat>
#include <vector>

#include "common.cuh"
#include "primitives.h"
#include "support.h"

namespace sinkslot {

// --------------------------------------------------------------------------
// projection
// --------------------------------------------------------------------------
template <bool KEYS>
__global__ void project_kernel(const float* __restrict__ X, int64_t n, int d,
                               const float* __restrict__ theta, int C, float* __restrict__ outf,
                               uint32_t* __restrict__ outk) {
  const int64_t total = (int64_t)C * n;
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < total;
       q += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(q / n);
    const int64_t i = q - (int64_t)c * n;
    const float* x = X + i * d;
    const float* t = theta + (int64_t)c * d;
    float acc = __fmul_rn(x[0], t[0]);
    for (int j = 1; j < d; ++j) acc = __fmaf_rn(x[j], t[j], acc);
    if (KEYS)
      outk[q] = float_to_radix(acc);
    else
      outf[q] = acc;
  }
}

static unsigned grid_for(int64_t work, int threads, int waves = 8) {
  int64_t g = ceil_div64(work, threads);
  int64_t cap = (int64_t)num_sms() * waves;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (unsigned)g;
}

int project(const float* X, int64_t n, int d, const float* theta, int C, float* out,
            cudaStream_t stream) {
  SINKSLOT_REQUIRE(n >= 0 && d >= 1 && C >= 0, "project: bad sizes");
  if (n == 0 || C == 0) return kOk;
  project_kernel<false><<<grid_for((int64_t)C * n, 256), 256, 0, stream>>>(X, n, d, theta, C, out,
                                                                           nullptr);
  SINKSLOT_CHECK_LAUNCH();
  return kOk;
}

// Radix keys of slices [start, start + C) of row-major projections P (n, L)
// (the `X @ theta.T` layout), transposed to slice-major (C, n) through a
// 32 x 32 shared-memory tile so both the read and the write are coalesced.
__global__ void transpose_keys_kernel(const float* __restrict__ P, int64_t n, int L, int start,
                                      int C, uint32_t* __restrict__ out) {
  __shared__ float tile[32][33];
  const int64_t i0 = (int64_t)blockIdx.x * 32;
  const int c0 = blockIdx.y * 32;
  for (int r = threadIdx.y; r < 32; r += 8) {
    const int64_t i = i0 + r;
    const int c = c0 + threadIdx.x;
    if (i < n && c < C) tile[r][threadIdx.x] = P[i * L + start + c];
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += 8) {
    const int c = c0 + r;
    const int64_t i = i0 + threadIdx.x;
    if (i < n && c < C) out[(int64_t)c * n + i] = float_to_radix(tile[threadIdx.x][r]);
  }
}

static int slice_keys(const float* X, const float* P, int64_t n, int d, const float* theta, int L,
                      int start, int C, uint32_t* keys, cudaStream_t stream) {
  if (P) {
    dim3 grid((unsigned)ceil_div64(n, 32), (unsigned)ceil_div64(C, 32));
    transpose_keys_kernel<<<grid, dim3(32, 8), 0, stream>>>(P, n, L, start, C, keys);
  } else {
    project_kernel<true><<<grid_for((int64_t)C * n, 256), 256, 0, stream>>>(
        X, n, d, theta + (int64_t)start * d, C, nullptr, keys);
  }
  SINKSLOT_CHECK_LAUNCH();
  return kOk;
}

// radix keys of a float array (for sorting caller-provided projections)
__global__ void float_keys_kernel(const float* __restrict__ v, int64_t total,
                                  uint32_t* __restrict__ k) {
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < total;
       q += (int64_t)gridDim.x * blockDim.x)
    k[q] = float_to_radix(v[q]);
}

// --------------------------------------------------------------------------
// torch-order cumsum of gathered weights
// --------------------------------------------------------------------------
uint32_t torch_inner_scan_log_tx(uint32_t num_rows, uint32_t row_size) {
  uint32_t lx = 0, ly = 0;
  while (((uint32_t)1 << lx) < row_size) ++lx;
  while (((uint32_t)1 << ly) < num_rows) ++ly;
  uint32_t diff = lx - ly;  // unsigned, as in ATen
  lx = ((uint32_t)9 + diff) / (uint32_t)2;
  lx = std::min(std::max((uint32_t)4, lx), (uint32_t)9);
  return lx;
}

// The same scan in three parallel steps with the same fp32 operations.  In a
// chunk of 2*tx elements the carry enters at element 0 (x0 + carry) and reaches
// the chunk's last element through one add per Sklansky level j = 1..L
// (L = log_tx + 1): T_j = R_j + T_{j-1}, where R_j, the tree total of block
// [2^(j-1), 2^j) after levels 0..j-2, does not depend on the carry.  So:
//   1. chunk_parts_kernel: per chunk, x0 and R_1..R_L (all chunks in parallel);
//   2. chunk_carry_kernel: per row, the chain of carries (L + 1 adds per chunk);
//   3. chunk_scan_kernel: per chunk, the full scan with x0 + its carry.
__global__ void chunk_parts_kernel(const uint32_t* __restrict__ order, const float* __restrict__ w,
                                   int64_t len, int log_tx, int64_t nchunks,
                                   float* __restrict__ parts) {
  extern __shared__ float buf[];
  const int tx = 1 << log_tx, L = log_tx + 1;
  const int t = threadIdx.x;
  const int64_t row = blockIdx.y, chunk = blockIdx.x;
  const uint32_t* ord = order + row * len;
  const int64_t c1 = chunk * 2 * tx + t, c2 = c1 + tx;
  buf[t] = c1 < len ? __ldg(w + ord[c1]) : 0.0f;
  buf[tx + t] = c2 < len ? __ldg(w + ord[c2]) : 0.0f;
  float* P = parts + (row * nchunks + chunk) * (L + 1);
  if (t == 0) P[0] = buf[0];
  __syncthreads();
  for (int mm = 0; mm <= log_tx; ++mm) {
    const uint32_t sz = 1u << mm;
    const uint32_t a = ((t >> mm) << (mm + 1)) | sz;
    const uint32_t ti = a + (t % sz);
    const uint32_t si = a - 1;
    if (ti == 2 * sz - 1) P[mm + 1] = buf[ti];  // R_{mm+1}, before this level adds to it
    buf[ti] = __fadd_rn(buf[ti], buf[si]);
    __syncthreads();
  }
}

// One block per row: the row's parts are staged in shared memory a window of
// chunks at a time (coalesced), then thread 0 runs the carry chain -- the same
// adds in the same order -- from registers, so no step of the serial chain
// waits on a global load.
constexpr int kCarryWin = 1024;  // chunks staged at a time
constexpr int kMaxParts = 11;    // L + 1 parts per chunk, L = log_tx + 1 <= 10

__global__ void __launch_bounds__(256) chunk_carry_kernel(const float* __restrict__ parts,
                                                          int64_t nchunks, int L,
                                                          float* __restrict__ carry) {
  __shared__ float sp[kCarryWin * kMaxParts];
  const int np = L + 1;
  const int64_t row = blockIdx.x;
  const float* P = parts + row * nchunks * np;
  float* out = carry + row * nchunks;
  float c = 0.0f;
  for (int64_t k0 = 0; k0 < nchunks; k0 += kCarryWin) {
    const int nk = (int)std::min<int64_t>(kCarryWin, nchunks - k0);
    __syncthreads();  // the previous window is consumed
    for (int i = threadIdx.x; i < nk * np; i += blockDim.x) sp[i] = P[k0 * np + i];
    __syncthreads();
    if (threadIdx.x == 0) {
#pragma unroll 4
      for (int k = 0; k < nk; ++k) {
        const float* q = sp + k * np;
        float v[kMaxParts];
#pragma unroll
        for (int j = 0; j < kMaxParts; ++j) v[j] = j < np ? q[j] : 0.0f;
        out[k0 + k] = c;
        float T = __fadd_rn(v[0], c);
#pragma unroll
        for (int j = 1; j < kMaxParts; ++j)
          if (j < np) T = __fadd_rn(v[j], T);
        c = T;
      }
    }
  }
}

__global__ void chunk_scan_kernel(const uint32_t* __restrict__ order, const float* __restrict__ w,
                                  float* __restrict__ out, int64_t len, int log_tx,
                                  int64_t nchunks, const float* __restrict__ carry) {
  extern __shared__ float buf[];
  const int tx = 1 << log_tx;
  const int t = threadIdx.x;
  const int64_t row = blockIdx.y, chunk = blockIdx.x;
  const uint32_t* ord = order + row * len;
  float* dst = out + row * len;
  const int64_t c1 = chunk * 2 * tx + t, c2 = c1 + tx;
  buf[t] = c1 < len ? __ldg(w + ord[c1]) : 0.0f;
  buf[tx + t] = c2 < len ? __ldg(w + ord[c2]) : 0.0f;
  if (t == 0) buf[0] = __fadd_rn(buf[0], carry[row * nchunks + chunk]);
  __syncthreads();
  for (int mm = 0; mm <= log_tx; ++mm) {
    const uint32_t sz = 1u << mm;
    const uint32_t a = ((t >> mm) << (mm + 1)) | sz;
    const uint32_t ti = a + (t % sz);
    const uint32_t si = a - 1;
    buf[ti] = __fadd_rn(buf[ti], buf[si]);
    __syncthreads();
  }
  if (c1 < len) dst[c1] = buf[t];
  if (c2 < len) dst[c2] = buf[tx + t];
}

// Sequential fp32 scan.  With C == 1 torch scans a 1-D tensor with CUB's
// device-wide scan, whose association order is not restated here; this stands
// in for it (exact for weights whose prefix sums are exact, e.g. uniform 2^-k).
__global__ void slice_cumsum_seq_kernel(const uint32_t* __restrict__ order,
                                        const float* __restrict__ w, float* __restrict__ out,
                                        int64_t len) {
  if (blockIdx.x != 0 || threadIdx.x != 0) return;
  float acc = 0.0f;
  for (int64_t i = 0; i < len; ++i) {
    acc = __fadd_rn(acc, w[order[i]]);
    out[i] = acc;
  }
}

// torch's scan order for C rows of len: chunks of 2*tx elements, tx from
// torch_inner_scan_log_tx(scan_rows, len) -- the order torch uses for a
// (scan_rows, len) tensor, of which these are C rows (scan_rows >= C; a single
// row is scanned sequentially).  `scratch`: C * nchunks * (log_tx + 3) floats,
// less than C * len since 2 * tx >= 32.
static int slice_cumsum(const uint32_t* order, const float* w, float* out, int64_t len, int C,
                        int scan_rows, float* scratch, cudaStream_t stream) {
  if (len == 0 || C == 0) return kOk;
  if (scan_rows == 1) {
    slice_cumsum_seq_kernel<<<1, 32, 0, stream>>>(order, w, out, len);
    SINKSLOT_CHECK_LAUNCH();
    return kOk;
  }
  const int log_tx = (int)torch_inner_scan_log_tx((uint32_t)scan_rows, (uint32_t)len);
  const int tx = 1 << log_tx;
  const int64_t nchunks = ceil_div64(len, (int64_t)2 * tx);
  SINKSLOT_REQUIRE(nchunks <= 0x7fffffff && C <= 65535, "cumsum: too many chunks or rows");
  float* parts = scratch;
  float* carry = scratch + (int64_t)C * nchunks * (log_tx + 2);
  const dim3 grid((unsigned)nchunks, (unsigned)C);
  chunk_parts_kernel<<<grid, tx, 2 * tx * sizeof(float), stream>>>(order, w, len, log_tx, nchunks,
                                                                    parts);
  SINKSLOT_CHECK_LAUNCH();
  SINKSLOT_REQUIRE(log_tx + 2 <= kMaxParts, "cumsum: scan width out of range");
  chunk_carry_kernel<<<(unsigned)C, 256, 0, stream>>>(parts, nchunks, log_tx + 1, carry);
  SINKSLOT_CHECK_LAUNCH();
  chunk_scan_kernel<<<grid, tx, 2 * tx * sizeof(float), stream>>>(order, w, out, len, log_tx,
                                                                   nchunks, carry);
  SINKSLOT_CHECK_LAUNCH();
  return kOk;
}

// --------------------------------------------------------------------------
// merge-path walk over (ca, cb): one merged breakpoint per step
// --------------------------------------------------------------------------
constexpr int kMergeThreads = 256;
constexpr int kMergeItems = 8;
constexpr int kMergeTile = kMergeThreads * kMergeItems;

// #{s[0..hi) < v} on a non-decreasing array
__device__ __forceinline__ int64_t lower_bound_f(const float* s, int64_t hi, float v) {
  int64_t lo = 0;
  while (lo < hi) {
    const int64_t mid = (lo + hi) >> 1;
    if (s[mid] < v) lo = mid + 1; else hi = mid;
  }
  return lo;
}

// number of ca elements among the first k merged elements (cb goes first on ties)
__device__ __forceinline__ int64_t merge_split(const float* ca, int64_t n, const float* cb,
                                               int64_t m, int64_t k) {
  int64_t lo = k - m > 0 ? k - m : 0;
  int64_t hi = k < n ? k : n;
  while (lo < hi) {
    const int64_t mid = (lo + hi) >> 1;
    if (ca[mid] < cb[k - mid - 1]) lo = mid + 1; else hi = mid;
  }
  return lo;
}

struct Walker {
  const float* ca;
  const float* cb;
  int64_t n, m;
  int64_t i, j;
  float prev;
  __device__ void start(int64_t k0) {
    i = merge_split(ca, n, cb, m, k0);
    j = k0 - i;
    if (k0 == 0) {
      prev = 0.0f;
    } else {
      const float pa = i > 0 ? ca[i - 1] : -INFINITY;
      const float pb = j > 0 ? cb[j - 1] : -INFINITY;
      prev = fmaxf(pa, pb);
    }
  }
  // Advance one merged position.  Returns true when the entry is kept (mass > 0)
  // and then sets (ii, jj, mass): the searchsorted(ca/cb, mid) results, clamped.
  __device__ bool step(int64_t& ii, int64_t& jj, float& mass) {
    const bool tb = (j < m) && (i >= n || cb[j] <= ca[i]);
    const float bnd = tb ? cb[j] : ca[i];
    const float ms = __fsub_rn(bnd, prev);
    bool keep = ms > 0.0f;
    if (keep) {
      const float mid = __fmul_rn(0.5f, __fadd_rn(prev, bnd));
      // ca[0..i) <= prev <= mid <= ca[i..): #{ca < mid} = i minus the trailing
      // entries equal to mid.
      int64_t a_ = i;
      if (a_ > 0 && !(ca[a_ - 1] < mid)) a_ = lower_bound_f(ca, a_ - 1, mid);
      int64_t b_ = j;
      if (b_ > 0 && !(cb[b_ - 1] < mid)) b_ = lower_bound_f(cb, b_ - 1, mid);
      ii = a_ < n - 1 ? a_ : n - 1;
      jj = b_ < m - 1 ? b_ : m - 1;
      mass = ms;
    }
    prev = bnd;
    if (tb) ++j; else ++i;
    return keep;
  }
};

__device__ __forceinline__ int64_t block_excl_scan_256(int64_t v, int64_t* total) {
  __shared__ int64_t wsum[kMergeThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int64_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t t = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += t;
  }
  if (lane == 31) wsum[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int64_t w = lane < kMergeThreads / 32 ? wsum[lane] : 0;
    int64_t wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t t = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += t;
    }
    if (lane < kMergeThreads / 32) wsum[lane] = wi - w;
    if (lane == kMergeThreads / 32 - 1) *total = wi;
  }
  __syncthreads();
  const int64_t r = wsum[warp] + x - v;
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kMergeThreads) merge_count_kernel(
    const float* __restrict__ CA, const float* __restrict__ CB, int64_t n, int64_t m, int tps,
    int64_t* __restrict__ counts) {
  const int c = blockIdx.y, tile = blockIdx.x;
  Walker w{CA + (int64_t)c * n, CB + (int64_t)c * m, n, m, 0, 0, 0.0f};
  const int64_t k0 = (int64_t)tile * kMergeTile + (int64_t)threadIdx.x * kMergeItems;
  const int64_t K = n + m;
  int64_t cnt = 0;
  if (k0 < K) {
    w.start(k0);
    int64_t ii, jj;
    float ms;
    for (int p = 0; p < kMergeItems && k0 + p < K; ++p) cnt += w.step(ii, jj, ms) ? 1 : 0;
  }
  __shared__ int64_t total;
  block_excl_scan_256(cnt, &total);
  if (threadIdx.x == 0) counts[(int64_t)c * tps + tile] = total;
}

// Emits kept entries: as (R, C, mass) int64 triples (KEYED = false) or as
// (R*m + C, mass bits) pairs for the coalesce sort (KEYED = true).
template <bool KEYED>
__global__ void __launch_bounds__(kMergeThreads) merge_emit_kernel(
    const float* __restrict__ CA, const float* __restrict__ CB, const uint32_t* __restrict__ IX,
    const uint32_t* __restrict__ IY, int64_t n, int64_t m, int tps,
    const int64_t* __restrict__ offsets, int64_t base_offset, int64_t* __restrict__ outR,
    int64_t* __restrict__ outC, float* __restrict__ outM, uint64_t* __restrict__ outKey,
    uint32_t* __restrict__ outMbits) {
  const int c = blockIdx.y, tile = blockIdx.x;
  const float* ca = CA + (int64_t)c * n;
  const float* cb = CB + (int64_t)c * m;
  const uint32_t* ix = IX + (int64_t)c * n;
  const uint32_t* iy = IY + (int64_t)c * m;
  const int64_t k0 = (int64_t)tile * kMergeTile + (int64_t)threadIdx.x * kMergeItems;
  const int64_t K = n + m;
  Walker w{ca, cb, n, m, 0, 0, 0.0f};
  int64_t cnt = 0;
  if (k0 < K) {
    w.start(k0);
    int64_t ii, jj;
    float ms;
    for (int p = 0; p < kMergeItems && k0 + p < K; ++p) cnt += w.step(ii, jj, ms) ? 1 : 0;
  }
  __shared__ int64_t total;
  int64_t pos = block_excl_scan_256(cnt, &total) + offsets[(int64_t)c * tps + tile] + base_offset;
  if (k0 < K) {
    w.start(k0);
    int64_t ii, jj;
    float ms;
    for (int p = 0; p < kMergeItems && k0 + p < K; ++p) {
      if (w.step(ii, jj, ms)) {
        const int64_t R = ix[ii], Cc = iy[jj];
        if (KEYED) {
          outKey[pos] = (uint64_t)R * (uint64_t)m + (uint64_t)Cc;
          outMbits[pos] = __float_as_uint(ms);
        } else {
          outR[pos] = R;
          outC[pos] = Cc;
          outM[pos] = ms;
        }
        ++pos;
      }
    }
  }
}

// --------------------------------------------------------------------------
// coalesce
// --------------------------------------------------------------------------
__global__ void head_flag_kernel(const uint64_t* __restrict__ key, int64_t nraw,
                                 int64_t* __restrict__ flag) {
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < nraw;
       k += (int64_t)gridDim.x * blockDim.x)
    flag[k] = (k == 0 || key[k] != key[k - 1]) ? 1 : 0;
}

__global__ void run_sum_kernel(const uint64_t* __restrict__ key, const uint32_t* __restrict__ mbits,
                               int64_t nraw, const int64_t* __restrict__ uidx, float invL,
                               uint64_t* __restrict__ ukey, float* __restrict__ S) {
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < nraw;
       k += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t kk = key[k];
    if (k != 0 && key[k - 1] == kk) continue;
    float s = __uint_as_float(mbits[k]);
    for (int64_t t = k + 1; t < nraw && key[t] == kk; ++t) s = __fadd_rn(s, __uint_as_float(mbits[t]));
    const int64_t u = uidx[k];
    ukey[u] = kk;
    S[u] = __fmul_rn(s, invL);
  }
}

__device__ __forceinline__ const float* support_s(const uint32_t* rm, const uint32_t* rm2,
                                                   const int64_t* scal);

__global__ void export_kernel(const uint64_t* __restrict__ ukey, const uint32_t* rm,
                              const uint32_t* rm2, const int64_t* __restrict__ scal,
                              int64_t nnz, int64_t m, int64_t* __restrict__ rows,
                              int64_t* __restrict__ cols, float* __restrict__ S) {
  const float* __restrict__ Sin = support_s(rm, rm2, scal);
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < nnz;
       k += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t kk = ukey[k];
    const uint64_t r = kk / (uint64_t)m;
    rows[k] = (int64_t)r;
    cols[k] = (int64_t)(kk - r * (uint64_t)m);
    S[k] = Sin[k];
  }
}

// --------------------------------------------------------------------------
// workspace layouts
// --------------------------------------------------------------------------
struct SliceBufs {
  uint32_t *kx, *vx, *kx2, *vx2;
  uint32_t *ky, *vy, *ky2, *vy2;
  float *ca, *cb;
  int64_t *counts;
  int64_t *hist, *stmp;
};

static void carve_slices(Carver& cv, SliceBufs& b, int64_t n, int64_t m, int C) {
  const int64_t cn = (int64_t)C * n, cm = (int64_t)C * m;
  b.kx = cv.take<uint32_t>(cn); b.vx = cv.take<uint32_t>(cn);
  b.kx2 = cv.take<uint32_t>(cn); b.vx2 = cv.take<uint32_t>(cn);
  b.ky = cv.take<uint32_t>(cm); b.vy = cv.take<uint32_t>(cm);
  b.ky2 = cv.take<uint32_t>(cm); b.vy2 = cv.take<uint32_t>(cm);
  b.ca = cv.take<float>(cn); b.cb = cv.take<float>(cm);
  const int64_t tps = ceil_div64(n + m, kMergeTile);
  b.counts = cv.take<int64_t>((size_t)C * tps + 1);
  const int64_t nh = std::max(radix_hist_elems(C, n), radix_hist_elems(C, m));
  b.hist = cv.take<int64_t>(std::max<int64_t>(nh, (int64_t)C * tps + 1));
  b.stmp = cv.take<int64_t>(scan_tmp_elems(std::max<int64_t>(nh, (int64_t)C * tps + 1)));
}

// Sort projections of C slices (given as radix keys in b.kx / b.ky), build the
// cumsums and count the kept merge entries per tile (exclusive offsets in
// b.counts, total in *d_total).  Returns the sorted index arrays.
static int slices_prepare(SliceBufs& b, const float* a, const float* bw, int64_t n, int64_t m,
                          int C, int scan_rows, const uint32_t** IX, const uint32_t** IY,
                          int64_t* d_total, cudaStream_t stream) {
  bool alt = false;
  SINKSLOT_TRY(radix_sort_pairs<uint32_t>(b.kx, b.vx, b.kx2, b.vx2, true, C, n, 32, b.hist, b.stmp,
                                          &alt, stream));
  const uint32_t* ix = alt ? b.vx2 : b.vx;
  SINKSLOT_TRY(radix_sort_pairs<uint32_t>(b.ky, b.vy, b.ky2, b.vy2, true, C, m, 32, b.hist, b.stmp,
                                          &alt, stream));
  const uint32_t* iy = alt ? b.vy2 : b.vy;
  // the sort keys are dead once the orders exist: their buffers hold the scan's scratch
  SINKSLOT_TRY(slice_cumsum(ix, a, b.ca, n, C, scan_rows, reinterpret_cast<float*>(b.kx2), stream));
  SINKSLOT_TRY(slice_cumsum(iy, bw, b.cb, m, C, scan_rows, reinterpret_cast<float*>(b.ky2), stream));
  const int tps = (int)ceil_div64(n + m, kMergeTile);
  merge_count_kernel<<<dim3(tps, C), kMergeThreads, 0, stream>>>(b.ca, b.cb, n, m, tps, b.counts);
  SINKSLOT_CHECK_LAUNCH();
  SINKSLOT_TRY(scan_exclusive_i64(b.counts, (int64_t)C * tps, b.stmp, d_total, stream));
  *IX = ix;
  *IY = iy;
  return kOk;
}

static int read_i64(const int64_t* d, int64_t* h, cudaStream_t stream) {
  SINKSLOT_CUDA_TRY(cudaMemcpyAsync(h, d, sizeof(int64_t), cudaMemcpyDeviceToHost, stream));
  SINKSLOT_CUDA_TRY(cudaStreamSynchronize(stream));
  return kOk;
}

// ---- ot1d (one call of the reference's batched 1-D builder) ----
size_t ot1d_workspace_bytes(int64_t n, int64_t m, int C) {
  Carver cv(nullptr, 0);
  SliceBufs b;
  carve_slices(cv, b, n, m, C);
  cv.take<int64_t>(4);
  return cv.used;
}

int ot1d_batched(const float* PXt, const float* PYt, const float* a, const float* b_w, int64_t n,
                 int64_t m, int C, int scan_rows, void* ws, size_t ws_bytes, int64_t* R,
                 int64_t* Cc, float* M, uint32_t* ix_out, uint32_t* iy_out, float* ca_out,
                 float* cb_out, int64_t* count_out, cudaStream_t stream) {
  SINKSLOT_REQUIRE(n >= 1 && m >= 1 && C >= 1, "ot1d: need n >= 1, m >= 1, C >= 1");
  if (scan_rows <= 0) scan_rows = C;
  SINKSLOT_REQUIRE(scan_rows >= C, "ot1d: scan_rows must be 0 or >= C");
  SINKSLOT_REQUIRE(n < (int64_t(1) << 31) && m < (int64_t(1) << 31), "ot1d: n, m must be < 2^31");
  Carver cv(ws, ws_bytes);
  SliceBufs b;
  carve_slices(cv, b, n, m, C);
  int64_t* d_total = cv.take<int64_t>(4);
  if (!cv.ok) {
    set_error("ot1d: workspace too small");
    return kWorkspaceTooSmall;
  }
  float_keys_kernel<<<grid_for((int64_t)C * n, 256), 256, 0, stream>>>(PXt, (int64_t)C * n, b.kx);
  SINKSLOT_CHECK_LAUNCH();
  float_keys_kernel<<<grid_for((int64_t)C * m, 256), 256, 0, stream>>>(PYt, (int64_t)C * m, b.ky);
  SINKSLOT_CHECK_LAUNCH();
  const uint32_t *ix, *iy;
  SINKSLOT_TRY(slices_prepare(b, a, b_w, n, m, C, scan_rows, &ix, &iy, d_total, stream));
  const int tps = (int)ceil_div64(n + m, kMergeTile);
  merge_emit_kernel<false><<<dim3(tps, C), kMergeThreads, 0, stream>>>(
      b.ca, b.cb, ix, iy, n, m, tps, b.counts, 0, R, Cc, M, nullptr, nullptr);
  SINKSLOT_CHECK_LAUNCH();
  if (ix_out) SINKSLOT_CUDA_TRY(cudaMemcpyAsync(ix_out, ix, (size_t)C * n * 4, cudaMemcpyDeviceToDevice, stream));
  if (iy_out) SINKSLOT_CUDA_TRY(cudaMemcpyAsync(iy_out, iy, (size_t)C * m * 4, cudaMemcpyDeviceToDevice, stream));
  if (ca_out) SINKSLOT_CUDA_TRY(cudaMemcpyAsync(ca_out, b.ca, (size_t)C * n * 4, cudaMemcpyDeviceToDevice, stream));
  if (cb_out) SINKSLOT_CUDA_TRY(cudaMemcpyAsync(cb_out, b.cb, (size_t)C * m * 4, cudaMemcpyDeviceToDevice, stream));
  return read_i64(d_total, count_out, stream);
}

// ---- full support (sot_plan_coo) ----
struct SupportBufs {
  SliceBufs s;
  uint64_t *rkey, *rkey2;
  uint32_t *rm, *rm2;
  int64_t *chist, *cstmp;
  uint64_t* ukey;
  // the unique entries' S sits in whichever of rm / rm2 the sort left free
  // (scal[2] = 1: rm2 holds the sorted masses, S is in rm)
  int64_t* scal;  // [0] raw total of a batch, [1] unique count, [2] S buffer selector
};

// the S of the unique entries (see SupportBufs)
__device__ __forceinline__ const float* support_s(const uint32_t* rm, const uint32_t* rm2,
                                                   const int64_t* scal) {
  return reinterpret_cast<const float*>(scal[2] ? rm : rm2);
}

static int chunk_of(int L, int chunk) { return (chunk <= 0 || chunk > L) ? L : chunk; }

static void carve_support(Carver& cv, SupportBufs& b, int64_t n, int64_t m, int L, int chunk) {
  const int C = chunk_of(L, chunk);
  carve_slices(cv, b.s, n, m, C);
  const int64_t cap = (int64_t)L * (n + m);
  b.rkey = cv.take<uint64_t>(cap); b.rkey2 = cv.take<uint64_t>(cap);
  b.rm = cv.take<uint32_t>(cap); b.rm2 = cv.take<uint32_t>(cap);
  const int64_t nh = radix_hist_elems(1, cap);
  b.chist = cv.take<int64_t>(std::max<int64_t>(nh, 1));
  b.cstmp = cv.take<int64_t>(scan_tmp_elems(std::max<int64_t>(nh, cap)));
  b.ukey = cv.take<uint64_t>(cap);
  b.scal = cv.take<int64_t>(8);
}

size_t support_workspace_bytes(int64_t n, int64_t m, int d, int L, int chunk) {
  (void)d;
  Carver cv(nullptr, 0);
  SupportBufs b;
  carve_support(cv, b, n, m, L, chunk);
  return cv.used;
}

int build_support(const float* X, const float* Y, const float* a, const float* bw, int64_t n,
                  int64_t m, int d, const float* theta, const float* PX, const float* PY, int L,
                  int chunk, void* ws, size_t ws_bytes, int64_t* nnz_out, cudaStream_t stream) {
  SINKSLOT_REQUIRE(n >= 1 && m >= 1 && d >= 1 && L >= 1, "build_support: need n, m, d, L >= 1");
  SINKSLOT_REQUIRE(n < (int64_t(1) << 31) && m < (int64_t(1) << 31),
                   "build_support: n, m must be < 2^31");
  SINKSLOT_REQUIRE(L <= 65535, "build_support: L must be <= 65535");
  SINKSLOT_REQUIRE((PX == nullptr) == (PY == nullptr), "build_support: give both PX and PY or neither");
  SINKSLOT_REQUIRE(PX != nullptr || theta != nullptr, "build_support: need theta or projections");
  Carver cv(ws, ws_bytes);
  SupportBufs b;
  carve_support(cv, b, n, m, L, chunk);
  if (!cv.ok) {
    set_error("build_support: workspace too small");
    return kWorkspaceTooSmall;
  }
  const int Cmax = chunk_of(L, chunk);
  const int tps = (int)ceil_div64(n + m, kMergeTile);
  int64_t nraw = 0;
  for (int start = 0; start < L; start += Cmax) {
    const int C = std::min(Cmax, L - start);
    SINKSLOT_TRY(slice_keys(X, PX, n, d, theta, L, start, C, b.s.kx, stream));
    SINKSLOT_TRY(slice_keys(Y, PY, m, d, theta, L, start, C, b.s.ky, stream));
    const uint32_t *ix, *iy;
    SINKSLOT_TRY(slices_prepare(b.s, a, bw, n, m, C, C, &ix, &iy, b.scal, stream));
    merge_emit_kernel<true><<<dim3(tps, C), kMergeThreads, 0, stream>>>(
        b.s.ca, b.s.cb, ix, iy, n, m, tps, b.s.counts, nraw, nullptr, nullptr, nullptr, b.rkey,
        b.rm);
    SINKSLOT_CHECK_LAUNCH();
    int64_t batch = 0;
    SINKSLOT_TRY(read_i64(b.scal, &batch, stream));
    nraw += batch;
  }
  if (nraw == 0) {
    *nnz_out = 0;
    return kOk;
  }
  bool alt = false;
  const int kb = bits_for((uint64_t)n * (uint64_t)m);
  SINKSLOT_TRY(radix_sort_pairs<uint64_t>(b.rkey, b.rm, b.rkey2, b.rm2, false, 1, nraw, kb, b.chist,
                                          b.cstmp, &alt, stream));
  const uint64_t* skey = alt ? b.rkey2 : b.rkey;
  const uint32_t* smass = alt ? b.rm2 : b.rm;
  // the free key buffer holds the head flags / unique positions
  int64_t* uidx = reinterpret_cast<int64_t*>(alt ? b.rkey : b.rkey2);
  head_flag_kernel<<<grid_for(nraw, 256), 256, 0, stream>>>(skey, nraw, uidx);
  SINKSLOT_CHECK_LAUNCH();
  SINKSLOT_TRY(scan_exclusive_i64(uidx, nraw, b.cstmp, b.scal + 1, stream));
  const float invL = 1.0f / (float)L;
  // S of the unique entries goes into the mass buffer the sort left free
  float* S = reinterpret_cast<float*>(alt ? b.rm : b.rm2);
  const int64_t sel = alt ? 1 : 0;  // pageable source: staged before the call returns
  SINKSLOT_CUDA_TRY(cudaMemcpyAsync(b.scal + 2, &sel, sizeof(sel), cudaMemcpyHostToDevice, stream));
  run_sum_kernel<<<grid_for(nraw, 256), 256, 0, stream>>>(skey, smass, nraw, uidx, invL, b.ukey, S);
  SINKSLOT_CHECK_LAUNCH();
  return read_i64(b.scal + 1, nnz_out, stream);
}

int support_export(const void* ws, size_t ws_bytes, int64_t n, int64_t m, int d, int L, int chunk,
                   int64_t nnz, int64_t* rows, int64_t* cols, float* S, cudaStream_t stream) {
  (void)d;
  Carver cv(const_cast<void*>(ws), ws_bytes);
  SupportBufs b;
  carve_support(cv, b, n, m, L, chunk);
  if (!cv.ok) {
    set_error("support_export: workspace too small");
    return kWorkspaceTooSmall;
  }
  SINKSLOT_REQUIRE(nnz >= 0 && nnz <= (int64_t)L * (n + m), "support_export: bad nnz");
  if (nnz == 0) return kOk;
  export_kernel<<<grid_for(nnz, 256), 256, 0, stream>>>(b.ukey, b.rm, b.rm2, b.scal, nnz, m, rows,
                                                        cols, S);
  SINKSLOT_CHECK_LAUNCH();
  return kOk;
}

// --------------------------------------------------------------------------
// COO -> CSR (to_csr, solver.py:235-276)
// --------------------------------------------------------------------------
__global__ void sorted_check_kernel(const int64_t* __restrict__ r, int64_t nnz,
                                    int* __restrict__ unsorted) {
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x + 1; k < nnz;
       k += (int64_t)gridDim.x * blockDim.x)
    if (r[k] < r[k - 1]) {
      *unsorted = 1;
      return;
    }
}

__global__ void key32_kernel(const int64_t* __restrict__ r, int64_t nnz, uint32_t* __restrict__ k) {
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < nnz;
       q += (int64_t)gridDim.x * blockDim.x)
    k[q] = (uint32_t)r[q];
}

// indptr[i] = #{sorted keys < i}, i in [0, nseg]
template <typename T>
__global__ void indptr_kernel(const T* __restrict__ skey, int64_t nnz, int64_t nseg,
                              int32_t* __restrict__ ptr) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i <= nseg;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t lo = 0, hi = nnz;
    while (lo < hi) {
      const int64_t mid = (lo + hi) >> 1;
      if ((int64_t)skey[mid] < i) lo = mid + 1; else hi = mid;
    }
    ptr[i] = (int32_t)lo;
  }
}

// sort key (the segment) and the payload {other index, value bits} of each entry
__global__ void key_payload_kernel(const int64_t* __restrict__ r, const int64_t* __restrict__ idx,
                                   const float* __restrict__ vals, int64_t nnz,
                                   uint32_t* __restrict__ k, uint64_t* __restrict__ pay) {
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < nnz;
       q += (int64_t)gridDim.x * blockDim.x) {
    k[q] = (uint32_t)r[q];
    pay[q] = (uint64_t)(uint32_t)idx[q] | ((uint64_t)__float_as_uint(vals[q]) << 32);
  }
}

template <typename IT>
__global__ void unpack_kernel(const uint64_t* __restrict__ pay, int64_t nnz, IT* __restrict__ oidx,
                              float* __restrict__ ovals) {
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < nnz;
       q += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t v = pay[q];
    oidx[q] = (IT)(int32_t)(uint32_t)v;
    ovals[q] = __uint_as_float((uint32_t)(v >> 32));
  }
}

template <typename IT>
__global__ void permute_kernel(const uint32_t* __restrict__ perm, const int64_t* __restrict__ idx,
                               const float* __restrict__ vals, int64_t nnz, IT* __restrict__ oidx,
                               float* __restrict__ ovals, int64_t* __restrict__ operm) {
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < nnz;
       q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = perm ? (int64_t)perm[q] : q;
    oidx[q] = (IT)idx[p];
    if (vals) ovals[q] = vals[p];
    if (operm) operm[q] = p;
  }
}

size_t csr_workspace_bytes(int64_t nnz, int64_t nseg) {
  Carver cv(nullptr, 0);
  cv.take<uint32_t>(nnz); cv.take<uint64_t>(nnz); cv.take<uint32_t>(nnz); cv.take<uint64_t>(nnz);
  const int64_t nh = radix_hist_elems(1, std::max<int64_t>(nnz, 1));
  cv.take<int64_t>(nh);
  cv.take<int64_t>(scan_tmp_elems(nh));
  cv.take<int>(4);
  (void)nseg;
  return cv.used;
}

int coo_to_csr(const int64_t* seg, const int64_t* idx, const float* vals, int64_t nnz, int64_t nseg,
               int idx_bytes, void* ws, size_t ws_bytes, int32_t* out_ptr, void* out_idx,
               float* out_vals, int64_t* out_perm, int* was_sorted, cudaStream_t stream) {
  SINKSLOT_REQUIRE(idx_bytes == 2 || idx_bytes == 4, "to_csr: idx_bytes must be 2 or 4");
  SINKSLOT_REQUIRE(nseg >= 0 && nseg < (int64_t(1) << 31) && nnz >= 0 && nnz < (int64_t(1) << 31),
                   "to_csr: sizes must be < 2^31");
  Carver cv(ws, ws_bytes);
  // values of the sort: the entry's position (uint32) when the permutation is
  // asked for, else the payload {other index, value bits} (uint64)
  uint32_t* k1 = cv.take<uint32_t>(nnz);
  uint64_t* p1 = cv.take<uint64_t>(nnz);
  uint32_t* k2 = cv.take<uint32_t>(nnz);
  uint64_t* p2 = cv.take<uint64_t>(nnz);
  uint32_t* v1 = reinterpret_cast<uint32_t*>(p1);
  uint32_t* v2 = reinterpret_cast<uint32_t*>(p2);
  const int64_t nh = radix_hist_elems(1, std::max<int64_t>(nnz, 1));
  int64_t* hist = cv.take<int64_t>(nh);
  int64_t* stmp = cv.take<int64_t>(scan_tmp_elems(nh));
  int* flag = cv.take<int>(4);
  if (!cv.ok) {
    set_error("to_csr: workspace too small");
    return kWorkspaceTooSmall;
  }
  int unsorted = 0;
  if (nnz > 1) {
    SINKSLOT_CUDA_TRY(cudaMemsetAsync(flag, 0, sizeof(int), stream));
    sorted_check_kernel<<<grid_for(nnz, 256), 256, 0, stream>>>(seg, nnz, flag);
    SINKSLOT_CHECK_LAUNCH();
    SINKSLOT_CUDA_TRY(cudaMemcpyAsync(&unsorted, flag, sizeof(int), cudaMemcpyDeviceToHost, stream));
    SINKSLOT_CUDA_TRY(cudaStreamSynchronize(stream));
  }
  *was_sorted = unsorted ? 0 : 1;
  if (unsorted && !out_perm && vals && out_vals) {
    // no permutation wanted: the sort carries each entry's index and value, so
    // nothing is gathered from random positions afterwards
    key_payload_kernel<<<grid_for(nnz, 256), 256, 0, stream>>>(seg, idx, vals, nnz, k1, p1);
    SINKSLOT_CHECK_LAUNCH();
    bool alt = false;
    SINKSLOT_TRY((radix_sort_pairs<uint32_t, uint64_t>(
        k1, p1, k2, p2, false, 1, nnz, bits_for((uint64_t)std::max<int64_t>(nseg, 1)), hist,
        stmp, &alt, stream)));
    const uint32_t* sk = alt ? k2 : k1;
    const uint64_t* sp = alt ? p2 : p1;
    indptr_kernel<uint32_t><<<grid_for(nseg + 1, 256), 256, 0, stream>>>(sk, nnz, nseg, out_ptr);
    SINKSLOT_CHECK_LAUNCH();
    if (idx_bytes == 2)
      unpack_kernel<int16_t><<<grid_for(nnz, 256), 256, 0, stream>>>(
          sp, nnz, static_cast<int16_t*>(out_idx), out_vals);
    else
      unpack_kernel<int32_t><<<grid_for(nnz, 256), 256, 0, stream>>>(
          sp, nnz, static_cast<int32_t*>(out_idx), out_vals);
    SINKSLOT_CHECK_LAUNCH();
    return kOk;
  }
  const uint32_t* perm = nullptr;
  if (!unsorted) {
    indptr_kernel<int64_t><<<grid_for(nseg + 1, 256), 256, 0, stream>>>(seg, nnz, nseg, out_ptr);
    SINKSLOT_CHECK_LAUNCH();
  } else {
    key32_kernel<<<grid_for(nnz, 256), 256, 0, stream>>>(seg, nnz, k1);
    SINKSLOT_CHECK_LAUNCH();
    bool alt = false;
    SINKSLOT_TRY(radix_sort_pairs<uint32_t>(k1, v1, k2, v2, true, 1, nnz,
                                            bits_for((uint64_t)std::max<int64_t>(nseg, 1)), hist,
                                            stmp, &alt, stream));
    const uint32_t* sk = alt ? k2 : k1;
    perm = alt ? v2 : v1;
    indptr_kernel<uint32_t><<<grid_for(nseg + 1, 256), 256, 0, stream>>>(sk, nnz, nseg, out_ptr);
    SINKSLOT_CHECK_LAUNCH();
  }
  // Already sorted: the permutation is the identity, `vals` is used as is (the
  // reference aliases it, solver.py:276) and neither out_vals nor out_perm is
  // written.
  const float* pv = unsorted ? vals : nullptr;
  int64_t* pp = unsorted ? out_perm : nullptr;
  if (nnz > 0) {
    if (idx_bytes == 2)
      permute_kernel<int16_t><<<grid_for(nnz, 256), 256, 0, stream>>>(
          perm, idx, pv, nnz, static_cast<int16_t*>(out_idx), out_vals, pp);
    else
      permute_kernel<int32_t><<<grid_for(nnz, 256), 256, 0, stream>>>(
          perm, idx, pv, nnz, static_cast<int32_t*>(out_idx), out_vals, pp);
    SINKSLOT_CHECK_LAUNCH();
  }
  return kOk;
}

}  // namespace sinkslot
