// partition.cu -- the two device steps of a support built across the GPUs of a
// node (one process per GPU, each building a contiguous range of the L slices):
//
//   partition_coo  a stable partition of COO entries by the rank that owns
//                  their segment (row, or column) -- contiguous segment ranges
//                  given by `bounds` -- so each rank's share is one contiguous
//                  run for an all-to-all exchange;
//   coalesce_coo   the reference's coalesce (sot_plan_coo, solver.py:194-232:
//                  unique keys r * m + c, duplicate masses summed, / L) of the
//                  raw entries a rank received, summed in the order received.
//
// Ranks send their runs in rank order and each rank's raw entries are in slice
// order, so the entries a rank receives are in global slice order; the stable
// sort by key then meets the duplicates of a key in slice order, as the
// single-GPU build does (support.cu), and every S is bit-identical to it.
#include <algorithm>

#include "common.cuh"
#include "primitives.h"
#include "support.h"

namespace sinkslot {

namespace {

unsigned grid_for(int64_t work, int threads) {
  int64_t g = ceil_div64(work, threads);
  const int64_t cap = (int64_t)num_sms() * 8;
  return (unsigned)std::max<int64_t>(1, std::min(g, cap));
}

struct Bounds {
  int64_t b[kMaxOwnerParts + 1];
  int parts;
};

// part[k] = the p with bounds[p] <= seg[k] < bounds[p + 1] (entries outside
// [bounds[0], bounds[parts]) go to the nearest end part)
__global__ void part_kernel(const int64_t* __restrict__ seg, int64_t nnz, const Bounds bd,
                            uint32_t* __restrict__ part) {
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < nnz;
       k += (int64_t)gridDim.x * blockDim.x) {
    const int64_t s = seg[k];
    uint32_t p = 0;
    for (int q = 1; q < bd.parts; ++q) p += s >= bd.b[q] ? 1u : 0u;
    part[k] = p;
  }
}

__global__ void gather_coo_kernel(const uint32_t* __restrict__ perm, int64_t nnz,
                                  const int64_t* __restrict__ seg,
                                  const int64_t* __restrict__ other,
                                  const float* __restrict__ vals, int64_t* __restrict__ seg_out,
                                  int64_t* __restrict__ other_out, float* __restrict__ vals_out) {
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < nnz;
       q += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t k = perm[q];
    seg_out[q] = seg[k];
    if (other) other_out[q] = other[k];
    if (vals) vals_out[q] = vals[k];
  }
}

// counts[p] = #{sorted part keys == p}
__global__ void part_counts_kernel(const uint32_t* __restrict__ skey, int64_t nnz, int parts,
                                   int64_t* __restrict__ counts) {
  const int p = threadIdx.x;
  if (p >= parts) return;
  auto lb = [&](uint32_t v) {
    int64_t lo = 0, hi = nnz;
    while (lo < hi) {
      const int64_t mid = (lo + hi) >> 1;
      if (skey[mid] < v) lo = mid + 1; else hi = mid;
    }
    return lo;
  };
  counts[p] = lb((uint32_t)p + 1) - lb((uint32_t)p);
}

__global__ void raw_key_kernel(const int64_t* __restrict__ R, const int64_t* __restrict__ C,
                               const float* __restrict__ mass, int64_t nraw, int64_t m,
                               uint64_t* __restrict__ key, uint32_t* __restrict__ mbits) {
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < nraw;
       k += (int64_t)gridDim.x * blockDim.x) {
    key[k] = (uint64_t)R[k] * (uint64_t)m + (uint64_t)C[k];
    mbits[k] = __float_as_uint(mass[k]);
  }
}

__global__ void flag_kernel(const uint64_t* __restrict__ key, int64_t nraw, int64_t* __restrict__ f) {
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < nraw;
       k += (int64_t)gridDim.x * blockDim.x)
    f[k] = (k == 0 || key[k] != key[k - 1]) ? 1 : 0;
}

// one thread per run of equal keys: the masses summed in order, times 1/L
__global__ void sum_runs_kernel(const uint64_t* __restrict__ key, const uint32_t* __restrict__ mbits,
                                int64_t nraw, const int64_t* __restrict__ uidx, float invL,
                                int64_t m, int64_t* __restrict__ rows, int64_t* __restrict__ cols,
                                float* __restrict__ S) {
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < nraw;
       k += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t kk = key[k];
    if (k != 0 && key[k - 1] == kk) continue;
    float s = __uint_as_float(mbits[k]);
    for (int64_t t = k + 1; t < nraw && key[t] == kk; ++t)
      s = __fadd_rn(s, __uint_as_float(mbits[t]));
    const int64_t u = uidx[k];
    const uint64_t r = kk / (uint64_t)m;
    rows[u] = (int64_t)r;
    cols[u] = (int64_t)(kk - r * (uint64_t)m);
    S[u] = __fmul_rn(s, invL);
  }
}

void carve_partition(Carver& cv, int64_t nnz, uint32_t** k1, uint32_t** v1, uint32_t** k2,
                     uint32_t** v2, int64_t** hist, int64_t** stmp, int64_t** counts) {
  const int64_t e = std::max<int64_t>(nnz, 1);
  *k1 = cv.take<uint32_t>(e);
  *v1 = cv.take<uint32_t>(e);
  *k2 = cv.take<uint32_t>(e);
  *v2 = cv.take<uint32_t>(e);
  const int64_t nh = radix_hist_elems(1, e);
  *hist = cv.take<int64_t>(nh);
  *stmp = cv.take<int64_t>(scan_tmp_elems(nh));
  *counts = cv.take<int64_t>(kMaxOwnerParts);
}

void carve_coalesce(Carver& cv, int64_t nraw, uint64_t** k1, uint32_t** m1, uint64_t** k2,
                    uint32_t** m2, int64_t** hist, int64_t** stmp, int64_t** scal) {
  const int64_t e = std::max<int64_t>(nraw, 1);
  *k1 = cv.take<uint64_t>(e);
  *k2 = cv.take<uint64_t>(e);
  *m1 = cv.take<uint32_t>(e);
  *m2 = cv.take<uint32_t>(e);
  const int64_t nh = radix_hist_elems(1, e);
  *hist = cv.take<int64_t>(nh);
  *stmp = cv.take<int64_t>(scan_tmp_elems(std::max<int64_t>(nh, e)));
  *scal = cv.take<int64_t>(4);
}

}  // namespace

size_t partition_workspace_bytes(int64_t nnz) {
  Carver cv(nullptr, 0);
  uint32_t *k1, *v1, *k2, *v2;
  int64_t *hist, *stmp, *counts;
  carve_partition(cv, nnz, &k1, &v1, &k2, &v2, &hist, &stmp, &counts);
  return cv.used;
}

int partition_coo(const int64_t* seg, const int64_t* other, const float* vals, int64_t nnz,
                  const int64_t* bounds_host, int parts, void* ws, size_t ws_bytes,
                  int64_t* seg_out, int64_t* other_out, float* vals_out, int64_t* counts_host,
                  cudaStream_t st) {
  SINKSLOT_REQUIRE(parts >= 1 && parts <= kMaxOwnerParts, "partition: parts must be 1..64");
  SINKSLOT_REQUIRE(nnz >= 0 && nnz < (int64_t(1) << 32), "partition: nnz must be < 2^32");
  SINKSLOT_REQUIRE(bounds_host && counts_host, "partition: null argument");
  for (int p = 0; p < parts; ++p)
    SINKSLOT_REQUIRE(bounds_host[p] <= bounds_host[p + 1], "partition: bounds must not decrease");
  Carver cv(ws, ws_bytes);
  uint32_t *k1, *v1, *k2, *v2;
  int64_t *hist, *stmp, *counts;
  carve_partition(cv, nnz, &k1, &v1, &k2, &v2, &hist, &stmp, &counts);
  if (!cv.ok) {
    set_error("partition: workspace too small");
    return kWorkspaceTooSmall;
  }
  for (int p = 0; p < parts; ++p) counts_host[p] = 0;
  if (nnz == 0) return kOk;
  Bounds bd{};
  bd.parts = parts;
  for (int p = 0; p <= parts; ++p) bd.b[p] = bounds_host[p];
  part_kernel<<<grid_for(nnz, 256), 256, 0, st>>>(seg, nnz, bd, k1);
  SINKSLOT_CHECK_LAUNCH();
  bool alt = false;
  SINKSLOT_TRY((radix_sort_pairs<uint32_t, uint32_t>(k1, v1, k2, v2, true, 1, nnz,
                                                     std::max(1, bits_for((uint64_t)parts)), hist,
                                                     stmp, &alt, st)));
  const uint32_t* skey = alt ? k2 : k1;
  const uint32_t* perm = alt ? v2 : v1;
  gather_coo_kernel<<<grid_for(nnz, 256), 256, 0, st>>>(perm, nnz, seg, other, vals, seg_out,
                                                        other_out, vals_out);
  SINKSLOT_CHECK_LAUNCH();
  part_counts_kernel<<<1, 64, 0, st>>>(skey, nnz, parts, counts);
  SINKSLOT_CHECK_LAUNCH();
  SINKSLOT_CUDA_TRY(cudaMemcpyAsync(counts_host, counts, parts * sizeof(int64_t),
                                    cudaMemcpyDeviceToHost, st));
  SINKSLOT_CUDA_TRY(cudaStreamSynchronize(st));
  return kOk;
}

size_t coalesce_workspace_bytes(int64_t nraw) {
  Carver cv(nullptr, 0);
  uint64_t *k1, *k2;
  uint32_t *m1, *m2;
  int64_t *hist, *stmp, *scal;
  carve_coalesce(cv, nraw, &k1, &m1, &k2, &m2, &hist, &stmp, &scal);
  return cv.used;
}

int coalesce_coo(const int64_t* R, const int64_t* C, const float* mass, int64_t nraw, int64_t n,
                 int64_t m, int L, void* ws, size_t ws_bytes, int64_t* rows, int64_t* cols,
                 float* S, int64_t* nnz_host, cudaStream_t st) {
  SINKSLOT_REQUIRE(n >= 1 && m >= 1 && L >= 1 && nraw >= 0, "coalesce: bad sizes");
  SINKSLOT_REQUIRE(nnz_host != nullptr, "coalesce: null argument");
  Carver cv(ws, ws_bytes);
  uint64_t *k1, *k2;
  uint32_t *m1, *m2;
  int64_t *hist, *stmp, *scal;
  carve_coalesce(cv, nraw, &k1, &m1, &k2, &m2, &hist, &stmp, &scal);
  if (!cv.ok) {
    set_error("coalesce: workspace too small");
    return kWorkspaceTooSmall;
  }
  *nnz_host = 0;
  if (nraw == 0) return kOk;
  raw_key_kernel<<<grid_for(nraw, 256), 256, 0, st>>>(R, C, mass, nraw, m, k1, m1);
  SINKSLOT_CHECK_LAUNCH();
  bool alt = false;
  SINKSLOT_TRY((radix_sort_pairs<uint64_t, uint32_t>(k1, m1, k2, m2, false, 1, nraw,
                                                     bits_for((uint64_t)n * (uint64_t)m), hist,
                                                     stmp, &alt, st)));
  const uint64_t* skey = alt ? k2 : k1;
  const uint32_t* smass = alt ? m2 : m1;
  // the free key buffer holds the head flags, then the unique positions
  int64_t* uidx = reinterpret_cast<int64_t*>(alt ? k1 : k2);
  flag_kernel<<<grid_for(nraw, 256), 256, 0, st>>>(skey, nraw, uidx);
  SINKSLOT_CHECK_LAUNCH();
  SINKSLOT_TRY(scan_exclusive_i64(uidx, nraw, stmp, scal, st));
  sum_runs_kernel<<<grid_for(nraw, 256), 256, 0, st>>>(skey, smass, nraw, uidx,
                                                       1.0f / (float)L, m, rows, cols, S);
  SINKSLOT_CHECK_LAUNCH();
  SINKSLOT_CUDA_TRY(cudaMemcpyAsync(nnz_host, scal, sizeof(int64_t), cudaMemcpyDeviceToHost, st));
  SINKSLOT_CUDA_TRY(cudaStreamSynchronize(st));
  return kOk;
}

}  // namespace sinkslot
