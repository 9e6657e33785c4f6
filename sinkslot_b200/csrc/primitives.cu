// primitives.cu -- device-wide exclusive scan and a stable, segmented LSD radix
// sort (8-bit digits).  Both are HBM-bound integer passes: tiles of 2048 keys,
// 256-thread blocks, warp-level match/ballot ranking for stability, and each
// tile reordered by digit in shared memory before it is written out, so the
// stores of a digit's run are coalesced.
#include "common.cuh"
#include "primitives.h"

namespace sinkslot {

// --------------------------------------------------------------------------
// Exclusive scan (int64): 8192 elements per block, recursive over block sums.
// --------------------------------------------------------------------------
constexpr int kScanThreads = 1024;
constexpr int kScanItems = 8;
constexpr int kScanTile = kScanThreads * kScanItems;

__device__ __forceinline__ int64_t warp_incl_scan(int64_t v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int64_t t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

__global__ void __launch_bounds__(kScanThreads) scan_block_kernel(int64_t* data, int64_t n,
                                                                  int64_t* block_sums) {
  __shared__ int64_t warp_tot[kScanThreads / 32];
  const int64_t base = (int64_t)blockIdx.x * kScanTile + (int64_t)threadIdx.x * kScanItems;
  int64_t v[kScanItems];
  int64_t run = 0;
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) {
    const int64_t p = base + i;
    v[i] = p < n ? data[p] : 0;
    const int64_t t = v[i];
    v[i] = run;  // exclusive within the thread
    run += t;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int64_t incl = warp_incl_scan(run, lane);
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int64_t w = lane < kScanThreads / 32 ? warp_tot[lane] : 0;
    int64_t wi = warp_incl_scan(w, lane);
    if (lane < kScanThreads / 32) warp_tot[lane] = wi - w;
    if (lane == 31 && block_sums) block_sums[blockIdx.x] = wi;
  }
  __syncthreads();
  const int64_t off = warp_tot[warp] + incl - run;
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) {
    const int64_t p = base + i;
    if (p < n) data[p] = v[i] + off;
  }
}

__global__ void scan_add_kernel(int64_t* data, int64_t n, const int64_t* block_offsets) {
  const int64_t add = block_offsets[blockIdx.x];
  const int64_t base = (int64_t)blockIdx.x * kScanTile;
  for (int i = threadIdx.x; i < kScanTile; i += blockDim.x) {
    const int64_t p = base + i;
    if (p < n) data[p] += add;
  }
}

__global__ void scan_total_kernel(const int64_t* data_excl, const int64_t* last_in, int64_t n,
                                  int64_t* total) {
  total[0] = data_excl[n - 1] + last_in[0];
}

size_t scan_tmp_elems(int64_t n) {
  size_t t = 1;  // saved last element
  int64_t m = n;
  while (m > kScanTile) {
    m = ceil_div64(m, kScanTile);
    t += (size_t)m + 1;
  }
  return t + 1;
}

static int scan_rec(int64_t* data, int64_t n, int64_t* tmp, cudaStream_t stream) {
  const int64_t nb = ceil_div64(n, kScanTile);
  if (nb <= 1) {
    scan_block_kernel<<<1, kScanThreads, 0, stream>>>(data, n, nullptr);
    SINKSLOT_CHECK_LAUNCH();
    return kOk;
  }
  int64_t* sums = tmp;
  scan_block_kernel<<<(unsigned)nb, kScanThreads, 0, stream>>>(data, n, sums);
  SINKSLOT_CHECK_LAUNCH();
  SINKSLOT_TRY(scan_rec(sums, nb, tmp + nb + 1, stream));
  scan_add_kernel<<<(unsigned)nb, 256, 0, stream>>>(data, n, sums);
  SINKSLOT_CHECK_LAUNCH();
  return kOk;
}

int scan_exclusive_i64(int64_t* data, int64_t n, int64_t* tmp, int64_t* total,
                       cudaStream_t stream) {
  if (n <= 0) {
    if (total) SINKSLOT_CUDA_TRY(cudaMemsetAsync(total, 0, sizeof(int64_t), stream));
    return kOk;
  }
  int64_t* last = tmp;  // keep the last input for the total
  if (total)
    SINKSLOT_CUDA_TRY(cudaMemcpyAsync(last, data + n - 1, sizeof(int64_t),
                                      cudaMemcpyDeviceToDevice, stream));
  SINKSLOT_TRY(scan_rec(data, n, tmp + 1, stream));
  if (total) {
    scan_total_kernel<<<1, 1, 0, stream>>>(data, last, n, total);
    SINKSLOT_CHECK_LAUNCH();
  }
  return kOk;
}

// --------------------------------------------------------------------------
// Radix sort
// --------------------------------------------------------------------------
constexpr int kSortThreads = 256;
constexpr int kSortWarps = kSortThreads / 32;
#ifndef SINKSLOT_SORT_ITEMS
#define SINKSLOT_SORT_ITEMS 8
#endif
constexpr int kSortItems = SINKSLOT_SORT_ITEMS;  // keys per thread of a tile
constexpr int kSortTile = kSortThreads * kSortItems;  // keys per tile
constexpr int kRadix = 256;
static_assert(kSortThreads == kRadix, "the scatter kernel gives each thread one digit");

int64_t radix_hist_elems(int64_t nseg, int64_t seglen) {
  return nseg * kRadix * ceil_div64(seglen, kSortTile);
}

template <typename K>
__global__ void __launch_bounds__(kSortThreads) radix_hist_kernel(const K* __restrict__ keys,
                                                                  int64_t seglen, int ntiles,
                                                                  int shift,
                                                                  int64_t* __restrict__ hist) {
  __shared__ uint32_t wh[kSortWarps][kRadix];
  const int seg = blockIdx.y, tile = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < kSortWarps * kRadix; i += kSortThreads) (&wh[0][0])[i] = 0;
  __syncthreads();
  const K* segk = keys + (int64_t)seg * seglen;
  const int64_t chunk = (int64_t)tile * kSortTile + (int64_t)warp * 32 * kSortItems;
#pragma unroll 4
  for (int r = 0; r < kSortItems; ++r) {
    const int64_t idx = chunk + r * 32 + lane;
    if (idx < seglen) {
      const uint32_t dg = (uint32_t)(segk[idx] >> shift) & 0xFFu;
      atomicAdd(&wh[warp][dg], 1u);
    }
  }
  __syncthreads();
  for (int d = threadIdx.x; d < kRadix; d += kSortThreads) {
    uint32_t t = 0;
#pragma unroll
    for (int w = 0; w < kSortWarps; ++w) t += wh[w][d];
    hist[((int64_t)seg * kRadix + d) * ntiles + tile] = t;
  }
}

// Exclusive scan of one value per thread over the 256 threads of the block.
__device__ __forceinline__ uint32_t block_excl_scan256(uint32_t v, uint32_t* warp_tot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const uint32_t w = lane < kSortWarps ? warp_tot[lane] : 0u;
    uint32_t wi = w;
#pragma unroll
    for (int o = 1; o < kSortWarps; o <<= 1) {
      const uint32_t t = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += t;
    }
    if (lane < kSortWarps) warp_tot[lane] = wi - w;
  }
  __syncthreads();
  return warp_tot[warp] + incl - v;
}

// Dynamic shared memory of the scatter kernel: the tile's keys and values in
// digit order (stable), then per-(warp, digit) counts, per-digit tile starts
// and global run starts.
template <typename K, typename V>
constexpr size_t scatter_smem() {
  return (size_t)kSortTile * (sizeof(K) + sizeof(V)) + (size_t)kSortWarps * kRadix * 4 +
         kRadix * 4 + kRadix * 8 + 64;
}

// Occupancy of the scatter pass, which is latency-bound (one tile per block):
// registers bounded for 5 blocks per SM (4 with 12-byte key/value pairs, which
// would spill at 5) and the whole shared-memory carveout (measured at 2^20: the
// first set-up's 16 passes 11.6 -> 9.2 ms against the defaults; a warm set-up's
// stay at ~9.3 ms).
#ifndef SINKSLOT_SORT_MIN_BLOCKS
#define SINKSLOT_SORT_MIN_BLOCKS 5
#endif
template <typename K, typename V>
constexpr int sort_min_blocks() {
  return sizeof(K) + sizeof(V) > 8 ? (SINKSLOT_SORT_MIN_BLOCKS > 4 ? 4 : SINKSLOT_SORT_MIN_BLOCKS)
                                   : SINKSLOT_SORT_MIN_BLOCKS;
}
#ifndef SINKSLOT_SORT_CARVEOUT
#define SINKSLOT_SORT_CARVEOUT 100
#endif

// One pass: the tile's keys are ranked (stable: warp match by digit, warps in
// order), placed in shared memory in digit order, and written out run by run,
// so consecutive threads store consecutive addresses of each digit's run.
template <typename K, typename V>
__global__ void __launch_bounds__(kSortThreads, (sort_min_blocks<K, V>())) radix_scatter_kernel(
    const K* __restrict__ keys_in, const V* __restrict__ vals_in, K* __restrict__ keys_out,
    V* __restrict__ vals_out, int64_t seglen, int ntiles, int shift,
    const int64_t* __restrict__ offs) {
  extern __shared__ __align__(16) unsigned char sm[];
  K* skey = reinterpret_cast<K*>(sm);
  V* sval = reinterpret_cast<V*>(sm + (size_t)kSortTile * sizeof(K));
  uint32_t(*wcnt)[kRadix] = reinterpret_cast<uint32_t(*)[kRadix]>(
      sm + (size_t)kSortTile * (sizeof(K) + sizeof(V)));
  uint32_t* dstart = reinterpret_cast<uint32_t*>(&wcnt[kSortWarps][0]);
  int64_t* gbase = reinterpret_cast<int64_t*>(dstart + kRadix);
  uint32_t* warp_tot = reinterpret_cast<uint32_t*>(gbase + kRadix);
  const int seg = blockIdx.y, tile = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < kSortWarps * kRadix; i += kSortThreads) (&wcnt[0][0])[i] = 0;
  __syncthreads();
  const int64_t segbase = (int64_t)seg * seglen;
  const int64_t tile0 = (int64_t)tile * kSortTile;
  const int valid_n = (int)min((int64_t)kSortTile, seglen - tile0);
  const int64_t chunk = tile0 + (int64_t)warp * 32 * kSortItems;
  const uint32_t lt_mask = (1u << lane) - 1u;
  K key[kSortItems];
  V val[kSortItems];
  uint32_t loc[kSortItems];
#pragma unroll
  for (int r = 0; r < kSortItems; ++r) {
    const int64_t idx = chunk + r * 32 + lane;
    const bool valid = idx < seglen;
    key[r] = valid ? keys_in[segbase + idx] : K(0);
    val[r] = valid ? (vals_in ? vals_in[segbase + idx] : (V)idx) : V(0);
    const uint32_t dg = valid ? ((uint32_t)(key[r] >> shift) & 0xFFu) : 0x100u;
    const uint32_t peers = __match_any_sync(0xffffffffu, dg);
    const uint32_t rank = __popc(peers & lt_mask);
    uint32_t base = 0;
    if (valid) base = wcnt[warp][dg];
    __syncwarp();
    if (valid && rank == 0) wcnt[warp][dg] = base + __popc(peers);
    __syncwarp();
    loc[r] = base + rank;
  }
  __syncthreads();
  // per digit (one per thread): warp prefixes in place, the tile-local start of
  // the digit, and the global start of this tile's run of it
  {
    const int d = threadIdx.x;  // kSortThreads == kRadix
    uint32_t run = 0;
#pragma unroll
    for (int w = 0; w < kSortWarps; ++w) {
      const uint32_t c = wcnt[w][d];
      wcnt[w][d] = run;
      run += c;
    }
    const uint32_t start = block_excl_scan256(run, warp_tot);
    dstart[d] = start;
    gbase[d] = offs[((int64_t)seg * kRadix + d) * ntiles + tile];
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < kSortItems; ++r) {
    const int64_t idx = chunk + r * 32 + lane;
    if (idx < seglen) {
      const uint32_t dg = (uint32_t)(key[r] >> shift) & 0xFFu;
      const uint32_t p = dstart[dg] + wcnt[warp][dg] + loc[r];
      skey[p] = key[r];
      sval[p] = val[r];
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < valid_n; i += kSortThreads) {
    const K k = skey[i];
    const uint32_t dg = (uint32_t)(k >> shift) & 0xFFu;
    const int64_t pos = gbase[dg] + (i - (int)dstart[dg]);
    keys_out[pos] = k;
    vals_out[pos] = sval[i];
  }
}

template <typename K, typename V>
int radix_sort_pairs(K* keys, V* vals, K* keys_alt, V* vals_alt, bool identity_vals,
                     int64_t nseg, int64_t seglen, int key_bits, int64_t* hist, int64_t* scan_tmp,
                     bool* result_in_alt, cudaStream_t stream) {
  *result_in_alt = false;
  SINKSLOT_REQUIRE(keys && vals && keys_alt && vals_alt, "radix sort: null buffer");
  if (nseg <= 0 || seglen <= 0) return kOk;
  SINKSLOT_REQUIRE(nseg <= 65535, "radix sort: too many segments");
  const int64_t ntiles = ceil_div64(seglen, kSortTile);
  SINKSLOT_REQUIRE(ntiles <= 0x7fffffff, "radix sort: segment too long");
  const int64_t nh = nseg * kRadix * ntiles;
  if (key_bits < 1) key_bits = 1;
  {
    // the dynamic shared-memory limit is a per-device function attribute
    static bool configured[64] = {};
    int dev = 0;
    SINKSLOT_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64 || !configured[dev]) {
      SINKSLOT_CUDA_TRY(cudaFuncSetAttribute(radix_scatter_kernel<K, V>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)scatter_smem<K, V>()));
      SINKSLOT_CUDA_TRY(cudaFuncSetAttribute(radix_scatter_kernel<K, V>,
                                             cudaFuncAttributePreferredSharedMemoryCarveout,
                                             SINKSLOT_SORT_CARVEOUT));
      if (dev >= 0 && dev < 64) configured[dev] = true;
    }
  }
  K* kin = keys;
  V* vin = vals;
  K* kout = keys_alt;
  V* vout = vals_alt;
  bool first = true;
  bool in_alt = false;
  for (int shift = 0; shift < key_bits; shift += 8) {
    dim3 grid((unsigned)ntiles, (unsigned)nseg);
    radix_hist_kernel<K><<<grid, kSortThreads, 0, stream>>>(kin, seglen, (int)ntiles, shift, hist);
    SINKSLOT_CHECK_LAUNCH();
    SINKSLOT_TRY(scan_exclusive_i64(hist, nh, scan_tmp, nullptr, stream));
    radix_scatter_kernel<K, V><<<grid, kSortThreads, scatter_smem<K, V>(), stream>>>(
        kin, (first && identity_vals) ? nullptr : vin, kout, vout, seglen, (int)ntiles, shift, hist);
    SINKSLOT_CHECK_LAUNCH();
    first = false;
    K* tk = kin; kin = kout; kout = tk;
    V* tv = vin; vin = vout; vout = tv;
    in_alt = !in_alt;
  }
  *result_in_alt = in_alt;
  return kOk;
}

template int radix_sort_pairs<uint32_t, uint32_t>(uint32_t*, uint32_t*, uint32_t*, uint32_t*, bool,
                                                  int64_t, int64_t, int, int64_t*, int64_t*, bool*,
                                                  cudaStream_t);
template int radix_sort_pairs<uint64_t, uint32_t>(uint64_t*, uint32_t*, uint64_t*, uint32_t*, bool,
                                                  int64_t, int64_t, int, int64_t*, int64_t*, bool*,
                                                  cudaStream_t);
template int radix_sort_pairs<uint32_t, uint64_t>(uint32_t*, uint64_t*, uint32_t*, uint64_t*, bool,
                                                  int64_t, int64_t, int, int64_t*, int64_t*, bool*,
                                                  cudaStream_t);

}  // namespace sinkslot
