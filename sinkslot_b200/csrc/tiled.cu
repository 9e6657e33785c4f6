// tiled.cu -- half-step with the gathered potential staged in shared memory.
//
// Why: a half-step gathers one potential value per support entry at random
// (67M gathers of a 4 MB vector per half-step at N = M = 2^20).  From global
// memory every gather is its own 32-byte sector request through L1TEX and L2,
// which caps the plain kernel near 1/4 of the HBM roofline.  Here each CTA owns
// a panel of R rows and walks the gathered axis in blocks of W entries: the
// block is copied into shared memory (cp.async, double-buffered) once per panel
// and every gather becomes a shared-memory load.
//
// Layout (built once per solve from the CSR side): tile (p, b) = the entries of
// panel p whose column lies in block b, in CSR order; per entry one uint32
// (row within the panel << 16 | column within the block) and the fp32 lam.
//
// Arithmetic: the log-sum-exp of a row is stabilised by the row's previous
// value, sigma = base - self_old (the LSE the previous half-step produced), so
// each term exp(lam + other - sigma) is O(1) and the terms of a row can be
// added in any order: each term is rounded to fixed point in 2^-32 units,
// split into a high part (bits 20+) and a low part (bits 0-19), and the parts
// are summed with native 32-bit shared-memory integer atomics -- exact and
// order-independent, so the result is deterministic.  The high-part sum cannot
// overflow because terms are capped at 2^k with k = 20 - ceil(log2(longest
// row)); the low-part sum cannot overflow for rows of up to 4096 entries.  A
// row is handed back to the exact (max-stabilised) kernel when a term exceeds
// the cap or its sum is below 2^-8 -- the first iteration, where sigma is not
// yet an estimate, and any row whose potential moved by more than a few units.
#include <algorithm>
#include <cfloat>
#include <cmath>

#include "common.cuh"
#include "epilogue.cuh"
#include "primitives.h"
#include "sinkhorn.h"
#include "tiled.h"

namespace sinkslot {

constexpr int kTileThreads = 1024;
constexpr int kTileUnroll = 8;
constexpr size_t kSmemCap = 227 * 1024;
constexpr float kFixScale = 4294967296.0f;  // 2^32
constexpr double kFixInv = 1.0 / 4294967296.0;
constexpr unsigned long long kFixMin = 1ull << 24;  // sums below 2^-8 go to the exact pass
constexpr int kLoBits = 20;

// shared memory per panel row: sigma, high sum, low sum (4 B each) + a flag bit
static size_t rows_smem(int R) {
  return 3 * align_up((size_t)R * 4, 16) + align_up((size_t)((R + 31) / 32) * 4, 16);
}

TileGeom tile_geom(int64_t nseg, int64_t m_o, int64_t nnz, int sms) {
  TileGeom g;
  g.nseg = nseg;
  g.m_o = m_o;
  g.nnz = nnz;
  if (nseg <= 0 || m_o <= 0) return g;
  int64_t P = sms;
  if (nseg < P * 32) P = std::max<int64_t>(1, ceil_div64(nseg, 32));
  int64_t R = ceil_div64(nseg, P);
  // keep at least 2 x 4096 floats of staging room and R < 2^16
  while ((int64_t)rows_smem((int)std::min<int64_t>(R, 1 << 20)) + 2 * 4096 * 4 + 1024 >
             (int64_t)kSmemCap ||
         R > 65535) {
    P += sms;
    R = ceil_div64(nseg, P);
  }
  const size_t avail = kSmemCap - rows_smem((int)R) - 1024;
  int logW = 2;
  while (logW < 16 && ((size_t)2 * 4 * ((size_t)1 << (logW + 1))) <= avail &&
         ((int64_t)1 << logW) < m_o)
    ++logW;
  g.P = (int)P;
  g.R = (int)R;
  g.logW = logW;
  g.B = (int)ceil_div64(m_o, (int64_t)1 << logW);
  g.smem_bytes = 2 * 4 * ((size_t)1 << logW) + rows_smem((int)R);
  const int64_t ntiles = (int64_t)g.P * g.B;
  Carver cv(nullptr, 0);
  cv.take<int64_t>(8);               // header: [0] longest row
  cv.take<int64_t>(ntiles + 1);      // tile starts
  cv.take<uint32_t>(std::max<int64_t>(nnz, 1));  // meta
  cv.take<float>(std::max<int64_t>(nnz, 1));     // lam
  g.layout_bytes = cv.used;
  Carver bw(nullptr, 0);
  const int64_t e = std::max<int64_t>(nnz, 1);
  bw.take<uint32_t>(e);  // row id
  bw.take<uint32_t>(e); bw.take<uint32_t>(e); bw.take<uint32_t>(e); bw.take<uint32_t>(e);
  const int64_t nh = radix_hist_elems(1, e);
  bw.take<int64_t>(nh);
  bw.take<int64_t>(scan_tmp_elems(nh));
  g.build_bytes = bw.used;
  return g;
}

struct LayoutPtrs {
  int64_t* header;
  int64_t* tstart;
  uint32_t* meta;
  float* lam;
};

static LayoutPtrs carve_layout(void* layout, const TileGeom& g) {
  Carver cv(layout, g.layout_bytes);
  LayoutPtrs p;
  p.header = cv.take<int64_t>(8);
  p.tstart = cv.take<int64_t>((int64_t)g.P * g.B + 1);
  p.meta = cv.take<uint32_t>(std::max<int64_t>(g.nnz, 1));
  p.lam = cv.take<float>(std::max<int64_t>(g.nnz, 1));
  return p;
}

static unsigned grid_t(int64_t work, int threads) {
  int64_t g = ceil_div64(work, threads);
  const int64_t cap = (int64_t)num_sms() * 8;
  return (unsigned)std::max<int64_t>(1, std::min(g, cap));
}

// ---------------------------------------------------------------------------
// layout builder
// ---------------------------------------------------------------------------
__global__ void rowid_kernel(const int32_t* __restrict__ ptr, int64_t nseg,
                             uint32_t* __restrict__ rowid, unsigned long long* longest) {
  unsigned long long best = 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nseg;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t s = ptr[i], e = ptr[i + 1];
    for (int64_t k = s; k < e; ++k) rowid[k] = (uint32_t)i;
    if ((unsigned long long)(e - s) > best) best = (unsigned long long)(e - s);
  }
  for (int o = 16; o >= 1; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
    best = t > best ? t : best;
  }
  if ((threadIdx.x & 31) == 0) atomicMax(longest, best);
}

template <typename IT>
__global__ void tilekey_kernel(const uint32_t* __restrict__ rowid, const IT* __restrict__ idx,
                               int64_t nnz, int R, int B, int logW, uint32_t* __restrict__ key) {
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < nnz;
       k += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t r = rowid[k];
    const uint32_t c = (uint32_t)idx[k];
    key[k] = (r / (uint32_t)R) * (uint32_t)B + (c >> logW);
  }
}

__global__ void tstart_kernel(const uint32_t* __restrict__ skey, int64_t nnz, int64_t ntiles,
                              int64_t* __restrict__ tstart) {
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t <= ntiles;
       t += (int64_t)gridDim.x * blockDim.x) {
    int64_t lo = 0, hi = nnz;
    while (lo < hi) {
      const int64_t mid = (lo + hi) >> 1;
      if ((int64_t)skey[mid] < t) lo = mid + 1; else hi = mid;
    }
    tstart[t] = lo;
  }
}

template <typename IT>
__global__ void tile_scatter_kernel(const uint32_t* __restrict__ perm,
                                    const uint32_t* __restrict__ rowid, const IT* __restrict__ idx,
                                    const float* __restrict__ lam, int64_t nnz, int R, int logW,
                                    uint32_t* __restrict__ meta, float* __restrict__ tlam) {
  const uint32_t wmask = (1u << logW) - 1u;
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < nnz;
       q += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t k = perm[q];
    const uint32_t r = rowid[k];
    const uint32_t c = (uint32_t)idx[k];
    meta[q] = ((r % (uint32_t)R) << 16) | (c & wmask);
    tlam[q] = lam[k];
  }
}

int build_tiles(const int32_t* ptr, const void* idx, int idx_bytes, const float* lam,
                const TileGeom& g, void* layout, void* ws, size_t ws_bytes, cudaStream_t st) {
  SINKSLOT_REQUIRE(idx_bytes == 2 || idx_bytes == 4, "build_tiles: idx_bytes must be 2 or 4");
  SINKSLOT_REQUIRE(g.nnz < (int64_t(1) << 32), "build_tiles: nnz must be < 2^32");
  SINKSLOT_REQUIRE(g.P > 0 && g.B > 0, "build_tiles: empty geometry");
  SINKSLOT_REQUIRE((int64_t)g.P * g.B < (int64_t(1) << 31), "build_tiles: too many tiles");
  LayoutPtrs L = carve_layout(layout, g);
  Carver cv(ws, ws_bytes);
  const int64_t e = std::max<int64_t>(g.nnz, 1);
  uint32_t* rowid = cv.take<uint32_t>(e);
  uint32_t* k1 = cv.take<uint32_t>(e);
  uint32_t* v1 = cv.take<uint32_t>(e);
  uint32_t* k2 = cv.take<uint32_t>(e);
  uint32_t* v2 = cv.take<uint32_t>(e);
  const int64_t nh = radix_hist_elems(1, e);
  int64_t* hist = cv.take<int64_t>(nh);
  int64_t* stmp = cv.take<int64_t>(scan_tmp_elems(nh));
  if (!cv.ok) {
    set_error("build_tiles: workspace too small");
    return kWorkspaceTooSmall;
  }
  const int64_t ntiles = (int64_t)g.P * g.B;
  SINKSLOT_CUDA_TRY(cudaMemsetAsync(L.header, 0, 8 * sizeof(int64_t), st));
  rowid_kernel<<<grid_t(g.nseg, 256), 256, 0, st>>>(
      ptr, g.nseg, rowid, reinterpret_cast<unsigned long long*>(L.header));
  SINKSLOT_CHECK_LAUNCH();
  if (g.nnz > 0) {
    if (idx_bytes == 2)
      tilekey_kernel<int16_t><<<grid_t(g.nnz, 256), 256, 0, st>>>(
          rowid, static_cast<const int16_t*>(idx), g.nnz, g.R, g.B, g.logW, k1);
    else
      tilekey_kernel<int32_t><<<grid_t(g.nnz, 256), 256, 0, st>>>(
          rowid, static_cast<const int32_t*>(idx), g.nnz, g.R, g.B, g.logW, k1);
    SINKSLOT_CHECK_LAUNCH();
    bool alt = false;
    SINKSLOT_TRY(radix_sort_pairs<uint32_t>(k1, v1, k2, v2, true, 1, g.nnz,
                                            bits_for((uint64_t)std::max<int64_t>(ntiles, 2)), hist,
                                            stmp, &alt, st));
    const uint32_t* skey = alt ? k2 : k1;
    const uint32_t* perm = alt ? v2 : v1;
    tstart_kernel<<<grid_t(ntiles + 1, 256), 256, 0, st>>>(skey, g.nnz, ntiles, L.tstart);
    SINKSLOT_CHECK_LAUNCH();
    if (idx_bytes == 2)
      tile_scatter_kernel<int16_t><<<grid_t(g.nnz, 256), 256, 0, st>>>(
          perm, rowid, static_cast<const int16_t*>(idx), lam, g.nnz, g.R, g.logW, L.meta, L.lam);
    else
      tile_scatter_kernel<int32_t><<<grid_t(g.nnz, 256), 256, 0, st>>>(
          perm, rowid, static_cast<const int32_t*>(idx), lam, g.nnz, g.R, g.logW, L.meta, L.lam);
    SINKSLOT_CHECK_LAUNCH();
  } else {
    SINKSLOT_CUDA_TRY(cudaMemsetAsync(L.tstart, 0, (ntiles + 1) * sizeof(int64_t), st));
  }
  return kOk;
}

// ---------------------------------------------------------------------------
// tiled half-step
// ---------------------------------------------------------------------------
struct TKArgs {
  int64_t nseg, m_o;
  int P, R, B, logW;
  const int64_t* header;
  const int64_t* tstart;
  const uint32_t* meta;
  const float* lam;
  const float* other;
  const float* base;
  const float* self_old;
  float* out;
  float w_old, w_new;
  float* prev;
  uint32_t* acc;
  int* fb_count;
  int* fb_list;
  int* fb_reset;
  int aligned16;  // `other` is 16-byte aligned: stage with 16-byte copies
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// copy other[b*W, min((b+1)*W, m_o)) into buf (all threads participate)
__device__ __forceinline__ void stage_block(const TKArgs& a, int b, float* buf) {
  const int64_t W = (int64_t)1 << a.logW;
  const int64_t c0 = (int64_t)b * W;
  const int64_t cnt = std::min<int64_t>(W, a.m_o - c0);
  const float* src = a.other + c0;
  if (a.aligned16) {
    const int64_t n16 = cnt >> 2;
    for (int64_t q = threadIdx.x; q < n16; q += kTileThreads) cp_async16(buf + 4 * q, src + 4 * q);
    for (int64_t q = (n16 << 2) + threadIdx.x; q < cnt; q += kTileThreads) cp_async4(buf + q, src + q);
  } else {
    for (int64_t q = threadIdx.x; q < cnt; q += kTileThreads) cp_async4(buf + q, src + q);
  }
}

template <int OUT, int CHK>
__global__ void __launch_bounds__(kTileThreads, 1) tiled_half_step_kernel(const TKArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int W = 1 << a.logW;
  const size_t rbytes = align_up((size_t)a.R * 4, 16);
  float* pot0 = reinterpret_cast<float*>(smem);
  float* pot1 = pot0 + W;
  float* sig = reinterpret_cast<float*>(smem + (size_t)2 * 4 * W);
  uint32_t* hi = reinterpret_cast<uint32_t*>(reinterpret_cast<unsigned char*>(sig) + rbytes);
  uint32_t* lo = reinterpret_cast<uint32_t*>(reinterpret_cast<unsigned char*>(hi) + rbytes);
  uint32_t* flags = reinterpret_cast<uint32_t*>(reinterpret_cast<unsigned char*>(lo) + rbytes);
  if (a.fb_reset && blockIdx.x == 0 && threadIdx.x == 0) *a.fb_reset = 0;

  // Terms are capped at 2^k, k = 20 - ceil(log2(longest row)), so the high-part
  // sum of any row stays below 2^32; longer rows than 4096 would overflow the
  // low-part sum, and then every row goes to the exact pass.
  const long long longest = a.header[0] > 0 ? a.header[0] : 1;
  int lg = 0;
  while ((1ll << lg) < longest) ++lg;
  const int k = kLoBits - lg;
  const float capd = (longest <= 4096 && k >= 1) ? ((float)k - 0.01f) * 0.69314718f : -INFINITY;
  uint32_t chk_bits = 0;
  constexpr int64_t kRound = (int64_t)kTileThreads * kTileUnroll;

  for (int p = blockIdx.x; p < a.P; p += gridDim.x) {
    const int64_t row0 = (int64_t)p * a.R;
    const int rows = (int)std::min<int64_t>(a.R, a.nseg - row0);
    if (rows <= 0) break;
    const int64_t pb = (int64_t)p * a.B;
    for (int r = threadIdx.x; r < a.R; r += kTileThreads) {
      hi[r] = 0u;
      lo[r] = 0u;
      sig[r] = r < rows ? __fsub_rn(a.base[row0 + r], a.self_old[row0 + r]) : 0.0f;
    }
    for (int r = threadIdx.x; r < (a.R + 31) / 32; r += kTileThreads) flags[r] = 0u;
    stage_block(a, 0, pot0);
    cp_async_commit();
    // entries of the first round of tile 0, loaded while the block stages
    uint32_t mt[kTileUnroll];
    float lv[kTileUnroll];
    {
      const int64_t e0 = a.tstart[pb], e1 = a.tstart[pb + 1];
#pragma unroll
      for (int u = 0; u < kTileUnroll; ++u) {
        const int64_t e = e0 + (int64_t)u * kTileThreads + threadIdx.x;
        mt[u] = e < e1 ? ld_stream(a.meta + e) : 0xFFFFFFFFu;
        lv[u] = e < e1 ? ld_stream(a.lam + e) : 0.0f;
      }
    }
    __syncthreads();
    for (int b = 0; b < a.B; ++b) {
      const float* cur = (b & 1) ? pot1 : pot0;
      if (b + 1 < a.B) {
        stage_block(a, b + 1, (b & 1) ? pot0 : pot1);
        cp_async_commit();
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      __syncthreads();
      const int64_t e0 = a.tstart[pb + b];
      const int64_t e1 = a.tstart[pb + b + 1];
      // prefetch the next tile's first round; it lands while this tile computes
      uint32_t nmt[kTileUnroll];
      float nlv[kTileUnroll];
      {
        const int64_t f0 = e1;
        const int64_t f1 = (b + 1 < a.B) ? a.tstart[pb + b + 2] : e1;
#pragma unroll
        for (int u = 0; u < kTileUnroll; ++u) {
          const int64_t e = f0 + (int64_t)u * kTileThreads + threadIdx.x;
          nmt[u] = e < f1 ? ld_stream(a.meta + e) : 0xFFFFFFFFu;
          nlv[u] = e < f1 ? ld_stream(a.lam + e) : 0.0f;
        }
      }
      for (int64_t base_e = e0;;) {
#pragma unroll
        for (int u = 0; u < kTileUnroll; ++u) {
          if (mt[u] == 0xFFFFFFFFu) continue;
          const uint32_t r = mt[u] >> 16;
          const uint32_t c = mt[u] & 0xFFFFu;
          const float d = __fsub_rn(__fadd_rn(lv[u], cur[c]), sig[r]);
          if (!(d <= capd)) {
            atomicOr(flags + (r >> 5), 1u << (r & 31));
          } else {
            const unsigned long long q = __float2ull_rn(__expf(d) * kFixScale);
            atomicAdd(hi + r, (uint32_t)(q >> kLoBits));
            atomicAdd(lo + r, (uint32_t)(q & ((1u << kLoBits) - 1u)));
          }
        }
        base_e += kRound;
        if (base_e >= e1) break;
        // tiles longer than one round: the further rounds load in place
#pragma unroll
        for (int u = 0; u < kTileUnroll; ++u) {
          const int64_t e = base_e + (int64_t)u * kTileThreads + threadIdx.x;
          mt[u] = e < e1 ? ld_stream(a.meta + e) : 0xFFFFFFFFu;
          lv[u] = e < e1 ? ld_stream(a.lam + e) : 0.0f;
        }
      }
#pragma unroll
      for (int u = 0; u < kTileUnroll; ++u) {
        mt[u] = nmt[u];
        lv[u] = nlv[u];
      }
      __syncthreads();
    }
    for (int r = threadIdx.x; r < rows; r += kTileThreads) {
      const int64_t seg = row0 + r;
      const unsigned long long q = ((unsigned long long)hi[r] << kLoBits) + lo[r];
      const bool flagged = (flags[r >> 5] >> (r & 31)) & 1u;
      if (flagged || q < kFixMin) {
        a.fb_list[atomicAdd(a.fb_count, 1)] = (int)seg;
        continue;
      }
      const float tot = (float)((double)q * kFixInv);
      const float lse = __fadd_rn(sig[r], logf(tot));
      segment_epilogue<OUT, CHK>(seg, lse, a.base, a.self_old, a.out, a.w_old, a.w_new, a.prev,
                                 chk_bits);
    }
    __syncthreads();
  }
  check_reduce<CHK>(chk_bits, a.acc);
}

template <int OUT, int CHK>
static int launch_tiled(const TKArgs& a, size_t smem, cudaStream_t st) {
  // the dynamic shared-memory limit is a per-device function attribute
  static bool configured[64] = {};
  int dev = 0;
  SINKSLOT_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    SINKSLOT_CUDA_TRY(cudaFuncSetAttribute(tiled_half_step_kernel<OUT, CHK>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)kSmemCap));
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  const int grid = std::min(a.P, num_sms());
  tiled_half_step_kernel<OUT, CHK><<<grid, kTileThreads, smem, st>>>(a);
  SINKSLOT_CHECK_LAUNCH();
  return kOk;
}

int tiled_half_step(const TiledHalfStep& h, int out_mode, int chk, cudaStream_t st) {
  SINKSLOT_REQUIRE(h.base != nullptr, "tiled half step: base is required");
  SINKSLOT_REQUIRE(h.fb_count && h.fb_list, "tiled half step: fallback list is required");
  SINKSLOT_REQUIRE(out_mode != kOutNone || chk == kChkMarg, "half step: check-only needs a check");
  if (h.g.nseg <= 0) return kOk;
  LayoutPtrs L = carve_layout(const_cast<void*>(h.layout), h.g);
  TKArgs a;
  a.nseg = h.g.nseg;
  a.m_o = h.g.m_o;
  a.P = h.g.P;
  a.R = h.g.R;
  a.B = h.g.B;
  a.logW = h.g.logW;
  a.header = L.header;
  a.tstart = L.tstart;
  a.meta = L.meta;
  a.lam = L.lam;
  a.other = h.other;
  a.base = h.base;
  a.self_old = h.self_old;
  a.out = h.out;
  a.w_old = h.w_old;
  a.w_new = h.w_new;
  a.prev = h.prev;
  a.acc = h.acc;
  a.fb_count = h.fb_count;
  a.fb_list = h.fb_list;
  a.fb_reset = h.fb_count_reset;
  a.aligned16 = ((reinterpret_cast<uintptr_t>(h.other) & 15u) == 0) ? 1 : 0;
  const size_t smem = h.g.smem_bytes;
  if (out_mode == kOutPlain) {
    if (chk == kChkNone) SINKSLOT_TRY((launch_tiled<kOutPlain, kChkNone>(a, smem, st)));
    else if (chk == kChkMarg) SINKSLOT_TRY((launch_tiled<kOutPlain, kChkMarg>(a, smem, st)));
    else SINKSLOT_TRY((launch_tiled<kOutPlain, kChkPot>(a, smem, st)));
  } else if (out_mode == kOutBlend) {
    if (chk == kChkNone) SINKSLOT_TRY((launch_tiled<kOutBlend, kChkNone>(a, smem, st)));
    else if (chk == kChkMarg) SINKSLOT_TRY((launch_tiled<kOutBlend, kChkMarg>(a, smem, st)));
    else SINKSLOT_TRY((launch_tiled<kOutBlend, kChkPot>(a, smem, st)));
  } else {
    SINKSLOT_TRY((launch_tiled<kOutNone, kChkMarg>(a, smem, st)));
  }
  // exact pass over the rows the tiled pass handed back
  HalfStep x;
  x.ptr = h.ptr;
  x.idx = h.idx;
  x.idx_bytes = h.idx_bytes;
  x.lam = h.lam;
  x.nseg = h.g.nseg;
  x.nnz = h.g.nnz;
  x.other = h.other;
  x.base = h.base;
  x.self_old = h.self_old;
  x.out = h.out;
  x.w_old = h.w_old;
  x.w_new = h.w_new;
  x.prev = h.prev;
  x.acc = h.acc;
  x.list = h.fb_list;
  x.list_count = h.fb_count;
  return half_step(x, out_mode, chk, st);
}

}  // namespace sinkslot
