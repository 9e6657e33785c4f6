// tiled.cu -- half-step with the gathered potential staged in shared memory.
//
// Why: a half-step gathers one potential value per support entry at random
// (67M gathers of a 4 MB vector per half-step at N = M = 2^20).  From global
// memory every gather is its own 32-byte sector request through L1TEX and L2,
// which caps the exact kernel near 1/4 of the HBM roofline.  Here each CTA owns
// a panel of R rows and walks the gathered axis in blocks of W entries; each
// block is copied into shared memory once per panel and every gather becomes a
// shared-memory load.
//
// Layout (built once per solve from the CSR side): tile (p, b) = the entries of
// panel p whose column lies in block b, padded to a multiple of 32 entries (one
// warp slab) and arranged so that a slab's rows fall in different shared-memory
// banks (see tilekey_kernel); per entry one uint2 {meta, fp32 lam bits}, meta
// holding the byte offsets of the row's state (row within the panel, times 4)
// and of the column's potential (column within the block, times 4).  Padding names row R (a dummy row
// of the panel state) with lam = -inf, so it adds an exact zero and the inner
// loop needs no test for it.
//
// Pipeline (one CTA per SM, warp-specialised): one producer warp issues TMA
// bulk copies (cp.async.bulk) of potential blocks into a shared-memory ring of
// kStages stages, each guarded by a full/empty mbarrier pair, and prefetches
// each tile's entries into L2 (cp.async.bulk.prefetch) when it issues the
// tile's block.  31 consumer warps read their slabs of entries straight from
// L2 with coalesced 8-byte loads (the next tile's first slabs are in flight
// while the current tile is processed), wait on "full", gather potentials from
// shared memory, accumulate, and arrive on "empty".  Entries never pass through
// shared memory, whose bandwidth the gathers and the row-state atomics need.
// No CTA-wide barrier per tile.  Every mbarrier wait is bounded by a clock
// budget: on timeout the kernel records an error code, the producer waits
// (bounded) for the copies it issued, and all warps leave.
//
// Arithmetic: the log-sum-exp of a row is stabilised by the row's previous
// value, sigma = base - self_old (the LSE the previous half-step produced), so
// each term exp(lam + other - sigma) is O(1) and the terms of a row can be
// added in any order: each term is rounded to fixed point in 2^-32 units,
// split into a high part (bits 20+) and a low part (bits 0-19), and the parts
// are summed with native 32-bit shared-memory integer atomics -- exact and
// order-independent, so the result is deterministic.  The high-part sum cannot
// overflow because terms are capped at 2^k with k = 20 - ceil(log2(longest
// row)); the low-part sum cannot overflow for rows of up to 4096 entries, and
// longer rows are handed back to the exact (max-stabilised) kernel whole.  A
// row is also handed back when a term exceeds the cap or its sum is below 2^-8
// -- the first iteration, where sigma is not yet an estimate, and any row whose
// potential moved by more than a few units.
#include <algorithm>
#include <cfloat>
#include <cmath>

#include "common.cuh"
#include "epilogue.cuh"
#include "primitives.h"
#include "sinkhorn.h"
#include "tiled.h"

namespace sinkslot {

#ifndef SINKSLOT_TILE_WARPS
#define SINKSLOT_TILE_WARPS 31
#endif
constexpr int kConsumerWarps = SINKSLOT_TILE_WARPS;  // + 1 producer warp
constexpr int kConsumers = 32 * kConsumerWarps;
constexpr int kPipeThreads = kConsumers + 32;  // + one producer warp
constexpr size_t kSmemCap = 227 * 1024;

// Build-time tuning of the pipeline (defaults measured on B200):
//   SINKSLOT_TILE_STAGES   depth of the potential-block ring
//   SINKSLOT_TILE_MAX_LOGW widest potential block (2^x floats)
//   SINKSLOT_TILE_PF_LEAD  tiles between the one whose entries the producer
//                          prefetches into L2 and the one whose block it copies
//   SINKSLOT_TILE_PF_BYTES largest single L2 prefetch (a tile's range is split)
#ifndef SINKSLOT_TILE_STAGES
#define SINKSLOT_TILE_STAGES 2
#endif
#ifndef SINKSLOT_TILE_MAX_LOGW
#define SINKSLOT_TILE_MAX_LOGW 14
#endif
#ifndef SINKSLOT_TILE_PF_LEAD
#define SINKSLOT_TILE_PF_LEAD 0
#endif
#ifndef SINKSLOT_TILE_PF_BYTES
#define SINKSLOT_TILE_PF_BYTES (1 << 30)
#endif
#ifndef SINKSLOT_TILE_EARLY_INIT
#define SINKSLOT_TILE_EARLY_INIT 1
#endif
constexpr int kStages = SINKSLOT_TILE_STAGES;
constexpr int kPfLead = SINKSLOT_TILE_PF_LEAD;
constexpr uint32_t kPfBytes = SINKSLOT_TILE_PF_BYTES;
static_assert(kPfLead >= 0 && kPfBytes >= 256 && kPfBytes % 256 == 0, "prefetch tuning");
constexpr size_t kBarBytes = align_up(16 * kStages + 16, 128);  // 2 mbarriers per stage + abort
constexpr float kFixScale = 4294967296.0f;  // 2^32
constexpr double kFixInv = 1.0 / 4294967296.0;
constexpr unsigned long long kFixMin = 1ull << 24;  // sums below 2^-8 go to the exact pass
constexpr int kLoBits = 20;
// rows up to this length are summed by the tiled pass (their low-part sum of
// terms below 2^20 stays below 2^32); longer rows always go to the exact pass
constexpr int64_t kMaxTiledRow = 4096;
constexpr long long kWaitCycles = 8000000000ll;  // ~4 s at 2 GHz: a wait this long is a bug

constexpr int kSlab = 32;  // tiles are padded to whole warp slabs of entries
// Slabs of a tile of n entries: ceil(n / 32), made odd (0 for an empty tile).
// With N odd the lanes of a slab hold sorted positions q = lane * N + slab that
// are distinct mod 32, which the column-bank placement (tile_colbank_kernel)
// relies on.
__host__ __device__ inline int64_t tile_slabs(int64_t n) {
  const int64_t N = (n + kSlab - 1) / kSlab;
  return N + (N > 0 && (N & 1) == 0 ? 1 : 0);
}
// slabs a consumer warp loads and processes together (its next tile's first
// group is in flight while it works on the current tile)
#ifndef SINKSLOT_TILE_GROUP
#define SINKSLOT_TILE_GROUP 4
#endif
constexpr int kGroup = SINKSLOT_TILE_GROUP;

// Shared memory of the tiled kernel, at fixed offsets (every address in the
// inner loop is a register plus a constant):
//   [0, kRingBytes)          kStages potential blocks of up to 2^kMaxLogW floats
//   kSigOff + 4 r            sigma of panel row r (float)
//   kHiOff + 4 r, kLoOff + 4 r  its high and low fixed-point sums (uint32)
//   kFlagOff                 one flag bit per row, then the mbarriers
// for rows r = 0 .. kRowCap - 1: the panel's R rows and the dummy row R (the
// target of tile padding).
constexpr int kMaxLogW = SINKSLOT_TILE_MAX_LOGW;
static_assert(kMaxLogW >= 8 && kMaxLogW <= 14, "columns are stored as 16-bit byte offsets");
constexpr uint32_t kStageBytes = 4u << kMaxLogW;
constexpr uint32_t kRingBytes = (uint32_t)kStages * kStageBytes;
// rows: 12 bytes of state and one flag bit each, in what the ring leaves
constexpr uint32_t kRowCap =
    (uint32_t)((kSmemCap - kRingBytes - kBarBytes - 256) * 8 / 97) & ~31u;
static_assert(kRowCap >= 64 && kRowCap <= 16384, "row state: rows are 16-bit byte offsets");
constexpr uint32_t kSigOff = kRingBytes;
constexpr uint32_t kHiOff = kSigOff + 4 * kRowCap;
constexpr uint32_t kLoOff = kHiOff + 4 * kRowCap;
constexpr uint32_t kFlagOff = kLoOff + 4 * kRowCap;
constexpr uint32_t kBarOff = (uint32_t)align_up(kFlagOff + kRowCap / 8, 128);
constexpr size_t kTileSmem = kBarOff + kBarBytes;
static_assert(kTileSmem <= kSmemCap, "tiled kernel shared memory");

// Entry meta word: (row within the panel) * 4 << 16 | (column within the
// block) * 4 -- the byte offsets of the row's state words and of the column's
// potential in their shared-memory arrays.
__host__ __device__ inline uint32_t entry_meta(uint32_t row, uint32_t col) {
  return (row << 18) | (col << 2);
}
__host__ __device__ inline uint32_t meta_row(uint32_t x) { return x >> 18; }
__host__ __device__ inline uint32_t meta_col(uint32_t x) { return (x & 0xFFFFu) >> 2; }

// The direct builder cuts each panel into S sub-panels of Rs consecutive rows,
// one CTA each, which keeps in shared memory two counters per (bank, block),
// the sub-panel's CSR offsets and the panel's tile starts.
constexpr int kBanks = 32;
constexpr int kBuildThreads = 32 * kBanks;  // warp w walks the rows of bank w
constexpr int kBuildCtasPerSm = 8;          // sub-panels enough for this many CTAs per SM
constexpr size_t kDirectSmemCap = 96 * 1024;
static size_t direct_smem(int Rs, int B) {
  return 2 * (size_t)kBanks * B * 4 + align_up((size_t)(Rs + 2) * 4, 16) + (size_t)(B + 1) * 8 +
         64;
}

// Two-pass kind: the panel-sum pass keeps only the row state in shared memory
// (no potential ring), so a panel holds up to kRowCap2 - 1 rows (row byte
// offsets stay 16-bit); the block-gather pass stages one block per CTA.
constexpr uint32_t kRowCap2 = 16384;
constexpr uint32_t kSigOff2 = 0;
constexpr uint32_t kHiOff2 = 4 * kRowCap2;
constexpr uint32_t kLoOff2 = 8 * kRowCap2;
constexpr uint32_t kFlagOff2 = 12 * kRowCap2;
constexpr uint32_t kAbortOff2 = kFlagOff2 + kRowCap2 / 8;
constexpr size_t kSumSmem = kAbortOff2 + 16;
static_assert(kSumSmem <= kSmemCap, "panel-sum kernel shared memory");

// A side runs the staged kind when staging the gathered potential costs at most
// this many times its entry stream: each of the P panels copies all m_o
// potentials into shared memory per half-step (P * m_o * 4 bytes) while the
// entries are read once (nnz * 8 bytes).  Above it the two-pass kind (16
// bytes per entry, all streamed) is cheaper.  Measured on B200 (N = M = 2^k,
// half-step us, staged / two-pass): 2^21 (ratio 2.3) 292 / ~410, 2^22 (ratio
// 4.6) 964 / 820 -- staged ~ (98 + 76 ratio) us per GB of entries, two-pass
// ~381 us per GB: equal near a ratio of 3.7.
#ifndef SINKSLOT_STAGING_RATIO
#define SINKSLOT_STAGING_RATIO 4.0
#endif

static int g_tiles_kind = kTilesAuto;
void set_tiles_kind(int kind) { g_tiles_kind = kind; }
int tiles_kind() { return g_tiles_kind; }

static void panel_split(TileGeom& g, int64_t nseg, int sms, uint32_t row_cap) {
  int64_t P = sms;
  if (nseg < P * 32) P = std::max<int64_t>(1, ceil_div64(nseg, 32));
  int64_t R = ceil_div64(nseg, P);
  // the panel's rows and the dummy row within the row state (more panels per SM)
  while (R + 1 > (int64_t)row_cap) {
    P += sms;
    R = ceil_div64(nseg, P);
  }
  g.P = (int)P;
  g.R = (int)R;
}

TileGeom tile_geom(int64_t nseg, int64_t m_o, int64_t nnz, int sms, int kind) {
  TileGeom g;
  g.nseg = nseg;
  g.m_o = m_o;
  g.nnz = nnz;
  if (kind < 0) kind = g_tiles_kind;
  if (nseg <= 0 || m_o <= 0) return g;
  panel_split(g, nseg, sms, kRowCap);
  if (kind == kTilesAuto)
    kind = (double)g.P * (double)m_o * 4.0 <= SINKSLOT_STAGING_RATIO * (double)nnz * 8.0
               ? kTilesStaged : kTilesTwoPass;
  g.kind = kind == kTilesTwoPass ? kTilesTwoPass : kTilesStaged;
  if (g.kind == kTilesTwoPass) panel_split(g, nseg, sms, kRowCap2);
  // the widest block (fewest tiles), up to a ring stage
  int logW = 2;
  while (logW < kMaxLogW && ((int64_t)1 << logW) < m_o) ++logW;
  g.logW = logW;
  g.B = (int)ceil_div64(m_o, (int64_t)1 << logW);
  g.smem_bytes = g.kind == kTilesTwoPass ? kSumSmem : kTileSmem;
  const int64_t ntiles = (int64_t)g.P * g.B;
  g.cap = nnz + (2 * kSlab - 1) * ntiles;  // each tile: an odd number of slabs
  Carver cv(nullptr, 0);
  cv.take<int64_t>(8);            // header: longest row, kind, P, B
  cv.take<int64_t>(ntiles + 1);   // tile starts (padded)
  cv.take<uint2>(std::max<int64_t>(g.cap, 1));  // entries {meta, lam bits}
  if (g.kind == kTilesTwoPass) {
    cv.take<uint16_t>(std::max<int64_t>(g.cap, 1));  // row byte offset per slot
    cv.take<float>(std::max<int64_t>(g.cap, 1));     // exponent lam + potential per slot
    cv.take<uint16_t>(std::max<int64_t>(g.cap, 1));  // column byte offset per slot
    cv.take<float>(std::max<int64_t>(g.cap, 1));     // lam per slot
  }
  g.layout_bytes = cv.used;
  g.S = (int)std::min<int64_t>(16, std::max<int64_t>(1, ceil_div64((int64_t)kBuildCtasPerSm * sms,
                                                                     g.P)));
  g.S = (int)std::min<int64_t>(g.S, std::max<int64_t>(1, g.R / 64));  // >= 2 rows per warp
  g.direct = direct_smem((int)ceil_div64(g.R, g.S), g.B) <= kDirectSmemCap;
  Carver bw(nullptr, 0);
  if (g.direct) {
    bw.take<uint32_t>(ntiles * g.S * kBanks);      // per sub-panel, bank and block: entries
    bw.take<int64_t>(scan_tmp_elems(ntiles + 1));  // scan of the tile sizes
  } else {
    const int64_t e = std::max<int64_t>(nnz, 1);
    bw.take<uint32_t>(e);  // row id
    for (int i = 0; i < 4; ++i) bw.take<uint32_t>(e);  // keys / values of the sort
    const int64_t nh = radix_hist_elems(1, e);
    bw.take<int64_t>(std::max<int64_t>(nh, ntiles + 2));
    bw.take<int64_t>(scan_tmp_elems(std::max<int64_t>(nh, ntiles + 2)));
    bw.take<int64_t>(ntiles + 2);  // unpadded tile starts
  }
  g.build_bytes = bw.used;
  return g;
}

struct LayoutPtrs {
  int64_t* header;  // [0] longest row of <= kMaxTiledRow entries, [1] kind, [2] P, [3] B
  int64_t* tstart;
  uint2* ent;
  uint16_t* rowoff;  // two-pass kind: row byte offset per slot (ent.x >> 16)
  float* expo;       // two-pass kind: exponent lam + potential per slot
  uint16_t* coloff;  // two-pass kind: column byte offset per slot (ent.x & 0xFFFF)
  float* lamv;       // two-pass kind: lam per slot (ent.y)
};

static LayoutPtrs carve_layout(void* layout, const TileGeom& g) {
  Carver cv(layout, g.layout_bytes);
  LayoutPtrs p;
  p.header = cv.take<int64_t>(8);
  p.tstart = cv.take<int64_t>((int64_t)g.P * g.B + 1);
  p.ent = cv.take<uint2>(std::max<int64_t>(g.cap, 1));
  p.rowoff = nullptr;
  p.expo = nullptr;
  p.coloff = nullptr;
  p.lamv = nullptr;
  if (g.kind == kTilesTwoPass) {
    p.rowoff = cv.take<uint16_t>(std::max<int64_t>(g.cap, 1));
    p.expo = cv.take<float>(std::max<int64_t>(g.cap, 1));
    p.coloff = cv.take<uint16_t>(std::max<int64_t>(g.cap, 1));
    p.lamv = cv.take<float>(std::max<int64_t>(g.cap, 1));
  }
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
    // the longest row the tiled pass sums (longer ones are handed back whole)
    if (e - s <= kMaxTiledRow && (unsigned long long)(e - s) > best)
      best = (unsigned long long)(e - s);
  }
  for (int o = 16; o >= 1; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
    best = t > best ? t : best;
  }
  if ((threadIdx.x & 31) == 0) atomicMax(longest, best);
}

// Order inside a tile.  A warp slab (32 consecutive entries) reads and updates
// the state of its 32 rows in shared memory; row r's three words sit in banks
// (3r + j) mod 32, so two rows of a slab share a bank exactly when their
// panel-local indices agree mod 32.  The tile's entries are sorted by that
// residue (its "bank"), then dealt across the tile's N slabs with stride N:
// sorted position p goes to slab p mod N, lane p / N.  A bank's run of c
// consecutive sorted positions lands in min(c, N) different slabs, so a slab
// holds at most ceil(c / N) rows of any bank -- one, unless that bank has more
// than N entries in the tile -- and 32 different rows.  Row order (consecutive
// rows in neighbouring lanes) would leave two-way conflicts in most slabs, the
// warp spanning more than 32 row indices once rows skip.  The sums are exact
// fixed point, so the order does not change any result.
constexpr int kBankBits = 5;

// key[k] = tile << kBankBits | bank of entry k's row.  One stable sort by this
// key gives the tile runs, each ordered by bank.
template <typename IT>
__global__ void tilekey_kernel(const uint32_t* __restrict__ rowid, const IT* __restrict__ idx,
                               int64_t nnz, int R, int B, int logW, uint32_t* __restrict__ key) {
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < nnz;
       k += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t r = rowid[k];
    const uint32_t b = (uint32_t)idx[k] >> logW;
    const uint32_t pnl = r / (uint32_t)R;
    const uint32_t bank = (r - pnl * (uint32_t)R) & ((1u << kBankBits) - 1u);
    key[k] = ((pnl * (uint32_t)B + b) << kBankBits) | bank;
  }
}

// ustart[t] = #{sorted keys of tiles < t}; cntp[t] = entries of tile t rounded
// up to an odd number of slabs (sorted keys are tile << kBankBits | bank)
__global__ void tile_counts_kernel(const uint32_t* __restrict__ skey, int64_t nnz, int64_t ntiles,
                                   int64_t* __restrict__ ustart, int64_t* __restrict__ cntp) {
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t <= ntiles;
       t += (int64_t)gridDim.x * blockDim.x) {
    auto lb = [&](int64_t v) {
      const uint64_t kv = (uint64_t)v << kBankBits;
      int64_t lo = 0, hi = nnz;
      while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if ((uint64_t)skey[mid] < kv) lo = mid + 1; else hi = mid;
      }
      return lo;
    };
    const int64_t s = lb(t);
    ustart[t] = s;
    if (t < ntiles) cntp[t] = tile_slabs(lb(t + 1) - s) * kSlab;
  }
}

// padding entries: the dummy row R, column 0, lam = -inf (a zero term)
__global__ void fill_pad_kernel(uint2* __restrict__ ent, int64_t cap, int R) {
  const uint2 pad = make_uint2(entry_meta((uint32_t)R, 0u), __float_as_uint(-INFINITY));
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < cap;
       q += (int64_t)gridDim.x * blockDim.x)
    ent[q] = pad;
}

// sorted position q: skey[q] its key, perm[q] its CSR entry; its position p in
// its tile's sorted run goes to slab p mod N, lane p / N of the tile's N slabs
template <typename IT>
__global__ void tile_scatter_kernel(const uint32_t* __restrict__ skey,
                                    const uint32_t* __restrict__ perm,
                                    const uint32_t* __restrict__ rowid, const IT* __restrict__ idx,
                                    const float* __restrict__ lam, int64_t nnz, int R, int logW,
                                    const int64_t* __restrict__ ustart,
                                    const int64_t* __restrict__ tstart,
                                    uint2* __restrict__ ent) {
  const uint32_t wmask = (1u << logW) - 1u;
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < nnz;
       q += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t t = skey[q] >> kBankBits;
    const uint32_t k = perm[q];
    const int64_t ts = tstart[t];
    const uint32_t ns = (uint32_t)((tstart[t + 1] - ts) >> 5);  // slabs of the tile (>= 1)
    const uint32_t p = (uint32_t)(q - ustart[t]);               // nnz < 2^32
    const uint32_t lane = p / ns;
    const int64_t pos = ts + ((int64_t)(p - lane * ns) << 5) + lane;
    const uint32_t r = rowid[k];
    const uint32_t c = (uint32_t)idx[k];
    ent[pos] = make_uint2(entry_meta(r % (uint32_t)R, c & wmask), __float_as_uint(lam[k]));
  }
}

static int place_column_banks(const TileGeom& g, const LayoutPtrs& L, cudaStream_t st);

// header: [0] longest row (raised by the builder), [1] kind, [2] P, [3] B; the
// half-step kernels compare [1..3] with their own geometry
__global__ void layout_header_kernel(int64_t* __restrict__ header, int kind, int P, int B) {
  const int i = threadIdx.x;
  if (i < 8) header[i] = i == 1 ? kind : i == 2 ? P : i == 3 ? B : 0;
}

// two-pass kind: every slot's entry split into what each pass reads (padding
// included) -- the row byte offset for the panel-sum pass, the column byte
// offset and lam for the block-gather pass
__global__ void split_slots_kernel(const uint2* __restrict__ ent, int64_t cap,
                                   uint16_t* __restrict__ rowoff, uint16_t* __restrict__ coloff,
                                   float* __restrict__ lamv) {
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < cap;
       q += (int64_t)gridDim.x * blockDim.x) {
    const uint2 e = ent[q];
    rowoff[q] = (uint16_t)(e.x >> 16);
    coloff[q] = (uint16_t)(e.x & 0xFFFFu);
    lamv[q] = __uint_as_float(e.y);
  }
}

// ---------------------------------------------------------------------------
// direct builder: one CTA per sub-panel, no sort
// ---------------------------------------------------------------------------
// Warp w walks the sub-panel's rows of bank w (panel rows r = w mod 32) in
// order and each row's entries in order; sub-panels follow one another in row
// order.  So the entries of a (block, bank) bucket are met in CSR order -- the
// order of the stable sort above -- and the layout is the same entry for
// entry.  Shared memory: two uint32 counters per (bank, block) -- the running
// slot and a scratch --, the sub-panel's CSR offsets ps[0..nr] (int32), the
// panel's tile starts ts[0..B] (int64).
struct PanelSmem {
  uint32_t* cnt;
  uint32_t* tmp;
  int32_t* ps;
  int64_t* ts;
};

__device__ __forceinline__ PanelSmem panel_smem(unsigned char* sm, int Rs, int B) {
  PanelSmem d;
  d.cnt = reinterpret_cast<uint32_t*>(sm);
  d.tmp = d.cnt + kBanks * B;
  d.ps = reinterpret_cast<int32_t*>(sm + 2 * (size_t)kBanks * B * 4);
  d.ts = reinterpret_cast<int64_t*>(sm + 2 * (size_t)kBanks * B * 4 +
                                    align_up((size_t)(Rs + 2) * 4, 16));
  return d;
}

// The rows of sub-panel s of panel p: panel-local [r_lo, r_hi).
struct SubRows {
  int64_t row0;  // first row of the panel
  int r_lo, r_hi;
};

__device__ __forceinline__ SubRows sub_rows(int64_t nseg, int R, int Rs) {
  SubRows q;
  q.row0 = (int64_t)blockIdx.y * R;
  const int rows = (int)std::max<int64_t>(0, std::min<int64_t>(R, nseg - q.row0));
  q.r_lo = std::min((int)blockIdx.x * Rs, rows);
  q.r_hi = std::min(q.r_lo + Rs, rows);
  return q;
}

// A warp's walk over the 32-entry chunks of its rows r = r_first, r_first + 32,
// ... < r_hi (panel-local; offsets in ps, indexed from r_lo).  next_chunk moves
// to the next non-empty chunk; the state starts one row before r_first.
struct ChunkWalk {
  int r, k0, e;
};

__device__ __forceinline__ bool next_chunk(const int32_t* ps, int r_lo, int r_hi, ChunkWalk& w) {
  if (w.k0 + 32 < w.e) {
    w.k0 += 32;
    return true;
  }
  do {
    w.r += kBanks;
    if (w.r >= r_hi) return false;
    w.k0 = ps[w.r - r_lo];
    w.e = ps[w.r - r_lo + 1];
  } while (w.k0 >= w.e);
  return true;
}

// Per sub-panel (blockIdx.x of gridDim.x, panel blockIdx.y): entries per
// (bank, block) into cnt_out[(p * S + s) * kBanks + bank][block], and the
// longest row of at most kMaxTiledRow entries into *longest.
template <typename IT>
__global__ void __launch_bounds__(kBuildThreads, 2) panel_count_kernel(
    const int32_t* __restrict__ ptr, const IT* __restrict__ idx, int64_t nseg, int R, int Rs,
    int B, int logW, uint32_t* __restrict__ cnt_out, unsigned long long* __restrict__ longest) {
  extern __shared__ __align__(16) unsigned char sm[];
  const PanelSmem d = panel_smem(sm, Rs, B);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const SubRows q = sub_rows(nseg, R, Rs);
  const int nr = q.r_hi - q.r_lo;
  for (int i = tid; i < kBanks * B; i += kBuildThreads) d.cnt[i] = 0;
  for (int i = tid; i <= nr; i += kBuildThreads) d.ps[i] = ptr[q.row0 + q.r_lo + i];
  __syncthreads();
  unsigned long long best = 0;
  for (int i = tid; i < nr; i += kBuildThreads) {
    const unsigned long long len = (unsigned long long)(d.ps[i + 1] - d.ps[i]);
    if (len <= (unsigned long long)kMaxTiledRow && len > best) best = len;
  }
  for (int o = 16; o >= 1; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
    best = t > best ? t : best;
  }
  if (lane == 0 && best > 0) atomicMax(longest, best);
  uint32_t* cw = d.cnt + warp * B;
  const uint32_t lt = (1u << lane) - 1u;
  // chunks of the warp's rows, each one's indices loaded a chunk ahead
  ChunkWalk cur{q.r_lo + ((warp - q.r_lo) & (kBanks - 1)) - kBanks, 0, 0};
  bool have = next_chunk(d.ps, q.r_lo, q.r_hi, cur);
  uint32_t c_cur = have && cur.k0 + lane < cur.e ? (uint32_t)(int32_t)idx[cur.k0 + lane]
                                                 : 0xFFFFFFFFu;
  while (have) {
    ChunkWalk nxt = cur;
    const bool have_n = next_chunk(d.ps, q.r_lo, q.r_hi, nxt);
    const uint32_t c_n = have_n && nxt.k0 + lane < nxt.e
                             ? (uint32_t)(int32_t)idx[nxt.k0 + lane] : 0xFFFFFFFFu;
    uint32_t b = c_cur >> logW;  // past the row's end: 0xFFFFFFFF >> logW >= B
    const bool v = b < (uint32_t)B;  // an index outside [0, m_other) is left out
    if (!v) b = 0xFFFFFFFFu;
    const uint32_t peers = __match_any_sync(0xffffffffu, b);
    if (v && (peers & lt) == 0) cw[b] += __popc(peers);
    __syncwarp();
    cur = nxt;
    c_cur = c_n;
    have = have_n;
  }
  __syncthreads();
  uint32_t* co = cnt_out + ((int64_t)blockIdx.y * gridDim.x + blockIdx.x) * kBanks * B;
  for (int i = tid; i < kBanks * B; i += kBuildThreads) co[i] = d.cnt[i];
}

// tsize[t] = entries of tile t = p * B + b over its panel's S sub-panels and
// the banks, rounded up to an odd number of slabs
__global__ void tile_size_kernel(const uint32_t* __restrict__ cnt, int64_t ntiles, int B, int S,
                                 int64_t* __restrict__ tsize) {
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < ntiles;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = t / B, b = t - p * B;
    const uint32_t* c = cnt + p * S * kBanks * B + b;
    uint32_t n = 0;
    for (int i = 0; i < S * kBanks; ++i) n += c[(int64_t)i * B];
    tsize[t] = tile_slabs(n) * kSlab;
  }
}

// Per sub-panel: every entry to its slot (sorted position q of its tile goes to
// slab q mod N, lane q / N); sub-panel 0 also writes the tile's padding to the
// slots after its entries.
template <typename IT>
__global__ void __launch_bounds__(kBuildThreads, 1) panel_scatter_kernel(
    const int32_t* __restrict__ ptr, const IT* __restrict__ idx, const float* __restrict__ lam,
    int64_t nseg, int R, int Rs, int B, int logW, const uint32_t* __restrict__ cnt_in,
    const int64_t* __restrict__ tstart, uint2* __restrict__ ent) {
  extern __shared__ __align__(16) unsigned char sm[];
  const PanelSmem d = panel_smem(sm, Rs, B);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int S = gridDim.x, s = blockIdx.x;
  const int64_t p = blockIdx.y;
  const SubRows q = sub_rows(nseg, R, Rs);
  const int nr = q.r_hi - q.r_lo;
  for (int i = tid; i <= nr; i += kBuildThreads) d.ps[i] = ptr[q.row0 + q.r_lo + i];
  for (int b = tid; b <= B; b += kBuildThreads) d.ts[b] = tstart[p * B + b];
  // per (bank, block): the entries of the earlier sub-panels (cnt) and of all
  // sub-panels (tmp)
  const uint32_t* ci = cnt_in + p * S * kBanks * B;
  for (int i = tid; i < kBanks * B; i += kBuildThreads) {
    uint32_t pre = 0, all = 0;
    for (int u = 0; u < S; ++u) {
      const uint32_t c = ci[(int64_t)u * kBanks * B + i];
      pre += u < s ? c : 0u;
      all += c;
    }
    d.cnt[i] = pre;
    d.tmp[i] = all;
  }
  __syncthreads();
  const uint2 pad = make_uint2(entry_meta((uint32_t)R, 0u), __float_as_uint(-INFINITY));
  for (int b = tid; b < B; b += kBuildThreads) {
    // each bank's first sorted position in the tile; padding after the entries
    uint32_t run = 0;
    for (int w = 0; w < kBanks; ++w) {
      d.cnt[w * B + b] += run;
      run += d.tmp[w * B + b];
    }
    if (s == 0) {
      const int64_t t0 = d.ts[b];
      const uint32_t ns = (uint32_t)((d.ts[b + 1] - t0) >> 5);
      for (uint32_t qq = run; qq < ns * kSlab; ++qq) {
        const uint32_t ln = qq / ns;
        ent[t0 + ((int64_t)(qq - ln * ns) << 5) + ln] = pad;
      }
    }
  }
  __syncthreads();
  const uint32_t wmask = (1u << logW) - 1u;
  uint32_t* cw = d.cnt + warp * B;
  const uint32_t lt = (1u << lane) - 1u;
  // chunks of the warp's rows, each one's entries loaded a chunk ahead
  ChunkWalk cur{q.r_lo + ((warp - q.r_lo) & (kBanks - 1)) - kBanks, 0, 0};
  bool have = next_chunk(d.ps, q.r_lo, q.r_hi, cur);
  uint32_t c_cur = 0xFFFFFFFFu;
  float l_cur = 0.0f;
  if (have && cur.k0 + lane < cur.e) {
    c_cur = (uint32_t)(int32_t)idx[cur.k0 + lane];
    l_cur = lam[cur.k0 + lane];
  }
  while (have) {
    ChunkWalk nxt = cur;
    const bool have_n = next_chunk(d.ps, q.r_lo, q.r_hi, nxt);
    uint32_t c_n = 0xFFFFFFFFu;
    float l_n = 0.0f;
    if (have_n && nxt.k0 + lane < nxt.e) {
      c_n = (uint32_t)(int32_t)idx[nxt.k0 + lane];
      l_n = lam[nxt.k0 + lane];
    }
    const uint32_t c = c_cur;
    uint32_t b = c >> logW;
    const bool v = cur.k0 + lane < cur.e && b < (uint32_t)B;  // as in panel_count_kernel
    if (!v) b = 0xFFFFFFFFu;
    const uint32_t peers = __match_any_sync(0xffffffffu, b);
    const uint32_t base = v ? cw[b] : 0u;
    __syncwarp();
    if (v && (peers & lt) == 0) cw[b] = base + __popc(peers);
    __syncwarp();
    if (v) {
      const uint32_t qq = base + __popc(peers & lt);
      const int64_t t0 = d.ts[b];
      const uint32_t ns = (uint32_t)((d.ts[b + 1] - t0) >> 5);
      const uint32_t ln = qq / ns;
      ent[t0 + ((int64_t)(qq - ln * ns) << 5) + ln] =
          make_uint2(entry_meta((uint32_t)cur.r, c & wmask), __float_as_uint(l_cur));
    }
    cur = nxt;
    c_cur = c_n;
    l_cur = l_n;
    have = have_n;
  }
}

// padding entries after the last tile: [*end, cap)
__global__ void fill_tail_kernel(uint2* __restrict__ ent, const int64_t* __restrict__ end,
                                 int64_t cap, int R) {
  const uint2 pad = make_uint2(entry_meta((uint32_t)R, 0u), __float_as_uint(-INFINITY));
  for (int64_t q = *end + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < cap;
       q += (int64_t)gridDim.x * blockDim.x)
    ent[q] = pad;
}

template <typename IT>
static int build_tiles_direct(const int32_t* ptr, const IT* idx, const float* lam,
                              const TileGeom& g, const LayoutPtrs& L, void* ws, size_t ws_bytes,
                              cudaStream_t st) {
  const int64_t ntiles = (int64_t)g.P * g.B;
  const int Rs = (int)ceil_div64(g.R, g.S);
  Carver cv(ws, ws_bytes);
  uint32_t* cnt = cv.take<uint32_t>(ntiles * g.S * kBanks);
  int64_t* stmp = cv.take<int64_t>(scan_tmp_elems(ntiles + 1));
  if (!cv.ok) {
    set_error("build_tiles: workspace too small");
    return kWorkspaceTooSmall;
  }
  SINKSLOT_REQUIRE(g.P <= 65535, "build_tiles: too many panels");
  const size_t smem = direct_smem(Rs, g.B);
  {
    // the dynamic shared-memory limit is a per-device function attribute
    static bool configured[64] = {};
    int dev = 0;
    SINKSLOT_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64 || !configured[dev]) {
      SINKSLOT_CUDA_TRY(cudaFuncSetAttribute(panel_count_kernel<IT>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)kDirectSmemCap));
      SINKSLOT_CUDA_TRY(cudaFuncSetAttribute(panel_scatter_kernel<IT>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)kDirectSmemCap));
      if (dev >= 0 && dev < 64) configured[dev] = true;
    }
  }
  const dim3 grid((unsigned)g.S, (unsigned)g.P);
  layout_header_kernel<<<1, 32, 0, st>>>(L.header, g.kind, g.P, g.B);
  SINKSLOT_CHECK_LAUNCH();
  panel_count_kernel<IT><<<grid, kBuildThreads, smem, st>>>(
      ptr, idx, g.nseg, g.R, Rs, g.B, g.logW, cnt,
      reinterpret_cast<unsigned long long*>(L.header));
  SINKSLOT_CHECK_LAUNCH();
  tile_size_kernel<<<grid_t(ntiles, 256), 256, 0, st>>>(cnt, ntiles, g.B, g.S, L.tstart);
  SINKSLOT_CHECK_LAUNCH();
  SINKSLOT_TRY(scan_exclusive_i64(L.tstart, ntiles, stmp, L.tstart + ntiles, st));
  panel_scatter_kernel<IT><<<grid, kBuildThreads, smem, st>>>(
      ptr, idx, lam, g.nseg, g.R, Rs, g.B, g.logW, cnt, L.tstart, L.ent);
  SINKSLOT_CHECK_LAUNCH();
  fill_tail_kernel<<<grid_t(ntiles * (kSlab - 1) + 1, 256), 256, 0, st>>>(L.ent, L.tstart + ntiles,
                                                                          g.cap, g.R);
  SINKSLOT_CHECK_LAUNCH();
  return place_column_banks(g, L, st);
}

// ---------------------------------------------------------------------------
// column-bank placement inside each row-bank run
// ---------------------------------------------------------------------------
// After the row-bank deal, a slab's 32 rows are in 32 different banks, but the
// columns it gathers from the staged potential block fall in random banks
// (~3.5 shared-memory wavefronts per gather).  Inside each row-bank run of a
// tile (sorted positions [S, S + c)), the entries may be permuted freely; this
// pass puts at sorted position q an entry whose column bank (column mod 32, the
// bank of the staged potential) is q mod 32 wherever it can.  Lanes of a slab
// hold positions q = lane * N + slab, distinct mod 32 for odd N, so entries
// placed on target gather from 32 different banks.  In a run, the k-th entry of
// column class t (in row-bank order) goes to relative position
// ((t - S) mod 32) + 32 k when that is below c; the others fill the remaining
// positions in a fixed order (classes ascending, then k), so the layout is
// deterministic.  Tiles larger than kPlaceMax entries keep the row-bank order.
// 16 warps per block, each placing two runs, and a 72 KB staging buffer plus an
// 18 KB hole table: two blocks per SM.
#ifndef SINKSLOT_TILE_COLBANK
#define SINKSLOT_TILE_COLBANK 1
#endif
constexpr int kPlaceWarps = 16;
constexpr int kPlaceThreads = 32 * kPlaceWarps;
constexpr int kPlaceMax = 9216;
constexpr size_t kPlaceSmem = (size_t)kPlaceMax * (sizeof(uint2) + sizeof(uint16_t));

__global__ void __launch_bounds__(kPlaceThreads, 2) tile_colbank_kernel(
    const int64_t* __restrict__ tstart, uint2* __restrict__ ent, int64_t ntiles, int R) {
  extern __shared__ __align__(16) unsigned char place_sm[];
  uint2* tbuf = reinterpret_cast<uint2*>(place_sm);  // the tile, by sorted position
  // free relative positions of each run, run r's at [S_r, S_r + holes): a
  // leftover entry reads its position with one load
  uint16_t* hole = reinterpret_cast<uint16_t*>(place_sm + (size_t)kPlaceMax * sizeof(uint2));
  __shared__ uint32_t ecnt[kBanks][33];   // per run: entries per column class
  __shared__ uint32_t run_k[kBanks][32];  // per run: running rank per class
  __shared__ uint32_t pre_o[kBanks][32];  // per run: leftover entries before class t
  __shared__ uint32_t rstart[kBanks + 1];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t lt = (1u << lane) - 1u;
  for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
    const int64_t ts = tstart[t];
    const int64_t len = tstart[t + 1] - ts;  // 32 N
    if (len == 0 || len > kPlaceMax) continue;  // uniform over the block
    const uint32_t N = (uint32_t)(len >> 5);
    // slots in order (coalesced): slot 32 s + l holds sorted position l N + s
    for (uint32_t q = tid; q < (uint32_t)len; q += kPlaceThreads)
      tbuf[(q & 31u) * N + (q >> 5)] = ent[ts + q];
    for (int i = tid; i < kBanks * 33; i += kPlaceThreads) (&ecnt[0][0])[i] = 0;
    __syncthreads();
    // entries per (row bank, column class), padding excluded
    for (uint32_t q = tid; q < (uint32_t)len; q += kPlaceThreads) {
      const uint32_t x = tbuf[q].x;
      if (meta_row(x) < (uint32_t)R) atomicAdd(&ecnt[meta_row(x) & (kBanks - 1)][meta_col(x) & 31u], 1u);
    }
    __syncthreads();
    if (warp == 0) {
      uint32_t v = 0;
      for (int u = 0; u < 32; ++u) v += ecnt[lane][u];
      uint32_t incl = v;
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t a = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += a;
      }
      rstart[lane] = incl - v;
      if (lane == 31) rstart[kBanks] = incl;
    }
    __syncthreads();
    // warp w: the runs of row banks w and w + kPlaceWarps
    for (int rw = warp; rw < kBanks; rw += kPlaceWarps) {
      const uint32_t S = rstart[rw], c = rstart[rw + 1] - S;
      {
        // lane = class t: positions of the class, matched entries, holes, leftovers
        const uint32_t e_t = ecnt[rw][lane];
        const uint32_t off = ((uint32_t)lane - S) & 31u;
        const uint32_t p_t = c > off ? (c - 1 - off) / 32 + 1 : 0u;
        const uint32_t m_t = e_t < p_t ? e_t : p_t;
        const uint32_t h_t = p_t - m_t, o_t = e_t - m_t;
        uint32_t ih = h_t, io = o_t;
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t a = __shfl_up_sync(0xffffffffu, ih, o);
          const uint32_t b = __shfl_up_sync(0xffffffffu, io, o);
          if (lane >= o) {
            ih += a;
            io += b;
          }
        }
        // the class's free positions: ranks e_t .. p_t - 1
        for (uint32_t i = 0; i < h_t; ++i)
          hole[S + (ih - h_t) + i] = (uint16_t)(off + 32u * (e_t + i));
        pre_o[rw][lane] = io - o_t;
        run_k[rw][lane] = 0;
      }
      __syncwarp();
      for (uint32_t j0 = 0; j0 < c; j0 += 32) {
        const uint32_t j = j0 + lane;
        const bool v = j < c;
        const uint2 e = v ? tbuf[S + j] : make_uint2(0u, 0u);
        const uint32_t cls = v ? (meta_col(e.x) & 31u) : 32u;
        const uint32_t peers = __match_any_sync(0xffffffffu, cls);
        const uint32_t base = v ? run_k[rw][cls] : 0u;
        __syncwarp();
        if (v && (peers & lt) == 0) run_k[rw][cls] = base + __popc(peers);
        __syncwarp();
        if (v) {
          const uint32_t k = base + __popc(peers & lt);
          const uint32_t off = (cls - S) & 31u;
          const uint32_t p_c = c > off ? (c - 1 - off) / 32 + 1 : 0u;
          // on target, or leftover number L into free position number L
          const uint32_t jn = k < p_c ? off + 32u * k : (uint32_t)hole[S + pre_o[rw][cls] + (k - p_c)];
          const uint32_t qn = S + jn;
          const uint32_t ln = qn / N;
          ent[ts + ((int64_t)(qn - ln * N) << 5) + ln] = e;
        }
      }
    }
    __syncthreads();  // the next tile reuses the buffers
  }
}

static int place_column_banks(const TileGeom& g, const LayoutPtrs& L, cudaStream_t st) {
#if SINKSLOT_TILE_COLBANK
  const int64_t ntiles = (int64_t)g.P * g.B;
  if (ntiles == 0 || g.nnz == 0) return kOk;
  const size_t smem = kPlaceSmem;
  static bool configured[64] = {};
  int dev = 0;
  SINKSLOT_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    SINKSLOT_CUDA_TRY(cudaFuncSetAttribute(tile_colbank_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)smem));
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  const unsigned grid = (unsigned)std::min<int64_t>(ntiles, 2 * (int64_t)num_sms());
  tile_colbank_kernel<<<grid, kPlaceThreads, smem, st>>>(L.tstart, L.ent, ntiles, g.R);
  SINKSLOT_CHECK_LAUNCH();
#else
  (void)g; (void)L; (void)st;
#endif
  return kOk;
}

static int build_tiles_body(const int32_t* ptr, const void* idx, int idx_bytes,
                            const float* lam, const TileGeom& g, void* layout, void* ws,
                            size_t ws_bytes, cudaStream_t st) {
  SINKSLOT_REQUIRE(idx_bytes == 2 || idx_bytes == 4, "build_tiles: idx_bytes must be 2 or 4");
  SINKSLOT_REQUIRE(g.nnz < (int64_t(1) << 32), "build_tiles: nnz must be < 2^32");
  SINKSLOT_REQUIRE(g.P > 0 && g.B > 0, "build_tiles: empty geometry");
  SINKSLOT_REQUIRE((int64_t)g.P * g.B < (int64_t(1) << (32 - kBankBits)),
                   "build_tiles: too many tiles");
  // the two-pass exponent pass addresses slots with 32-bit indices
  SINKSLOT_REQUIRE(g.kind != kTilesTwoPass || g.cap < (int64_t(1) << 32),
                   "build_tiles: a two-pass layout must hold fewer than 2^32 slots");
  LayoutPtrs L = carve_layout(layout, g);
  if (g.direct) {
    if (idx_bytes == 2)
      return build_tiles_direct(ptr, static_cast<const int16_t*>(idx), lam, g, L, ws, ws_bytes, st);
    return build_tiles_direct(ptr, static_cast<const int32_t*>(idx), lam, g, L, ws, ws_bytes, st);
  }
  Carver cv(ws, ws_bytes);
  const int64_t e = std::max<int64_t>(g.nnz, 1);
  const int64_t ntiles = (int64_t)g.P * g.B;
  uint32_t* rowid = cv.take<uint32_t>(e);
  uint32_t* k1 = cv.take<uint32_t>(e);
  uint32_t* v1 = cv.take<uint32_t>(e);
  uint32_t* k2 = cv.take<uint32_t>(e);
  uint32_t* v2 = cv.take<uint32_t>(e);
  const int64_t nh = std::max<int64_t>(radix_hist_elems(1, e), ntiles + 2);
  int64_t* hist = cv.take<int64_t>(nh);
  int64_t* stmp = cv.take<int64_t>(scan_tmp_elems(nh));
  int64_t* ustart = cv.take<int64_t>(ntiles + 2);
  if (!cv.ok) {
    set_error("build_tiles: workspace too small");
    return kWorkspaceTooSmall;
  }
  layout_header_kernel<<<1, 32, 0, st>>>(L.header, g.kind, g.P, g.B);
  SINKSLOT_CHECK_LAUNCH();
  fill_pad_kernel<<<grid_t(g.cap, 256), 256, 0, st>>>(L.ent, g.cap, g.R);
  SINKSLOT_CHECK_LAUNCH();
  rowid_kernel<<<grid_t(g.nseg, 256), 256, 0, st>>>(
      ptr, g.nseg, rowid, reinterpret_cast<unsigned long long*>(L.header));
  SINKSLOT_CHECK_LAUNCH();
  if (g.nnz == 0) {
    SINKSLOT_CUDA_TRY(cudaMemsetAsync(L.tstart, 0, (ntiles + 1) * sizeof(int64_t), st));
    return kOk;
  }
  if (idx_bytes == 2)
    tilekey_kernel<int16_t><<<grid_t(g.nnz, 256), 256, 0, st>>>(
        rowid, static_cast<const int16_t*>(idx), g.nnz, g.R, g.B, g.logW, k1);
  else
    tilekey_kernel<int32_t><<<grid_t(g.nnz, 256), 256, 0, st>>>(
        rowid, static_cast<const int32_t*>(idx), g.nnz, g.R, g.B, g.logW, k1);
  SINKSLOT_CHECK_LAUNCH();
  bool alt = false;
  SINKSLOT_TRY(radix_sort_pairs<uint32_t>(
      k1, v1, k2, v2, true, 1, g.nnz,
      bits_for((uint64_t)std::max<int64_t>(ntiles, 2)) + kBankBits, hist, stmp, &alt, st));
  const uint32_t* skey = alt ? k2 : k1;
  const uint32_t* perm = alt ? v2 : v1;
  // padded tile starts: exclusive scan of the rounded-up counts (in L.tstart)
  tile_counts_kernel<<<grid_t(ntiles + 1, 256), 256, 0, st>>>(skey, g.nnz, ntiles, ustart,
                                                              L.tstart);
  SINKSLOT_CHECK_LAUNCH();
  SINKSLOT_TRY(scan_exclusive_i64(L.tstart, ntiles, stmp, L.tstart + ntiles, st));
  if (idx_bytes == 2)
    tile_scatter_kernel<int16_t><<<grid_t(g.nnz, 256), 256, 0, st>>>(
        skey, perm, rowid, static_cast<const int16_t*>(idx), lam, g.nnz, g.R, g.logW, ustart,
        L.tstart, L.ent);
  else
    tile_scatter_kernel<int32_t><<<grid_t(g.nnz, 256), 256, 0, st>>>(
        skey, perm, rowid, static_cast<const int32_t*>(idx), lam, g.nnz, g.R, g.logW, ustart,
        L.tstart, L.ent);
  SINKSLOT_CHECK_LAUNCH();
  return place_column_banks(g, L, st);
}

int build_tiles(const int32_t* ptr, const void* idx, int idx_bytes, const float* lam,
                const TileGeom& g, void* layout, void* ws, size_t ws_bytes, cudaStream_t st) {
  SINKSLOT_TRY(build_tiles_body(ptr, idx, idx_bytes, lam, g, layout, ws, ws_bytes, st));
  if (g.kind == kTilesTwoPass) {
    const LayoutPtrs L = carve_layout(layout, g);
    split_slots_kernel<<<grid_t(g.cap, 256), 256, 0, st>>>(L.ent, g.cap, L.rowoff, L.coloff,
                                                           L.lamv);
    SINKSLOT_CHECK_LAUNCH();
  }
  return kOk;
}

// ---------------------------------------------------------------------------
// mbarrier / bulk-copy helpers (PTX)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// The same test, but a thread whose phase is not complete is suspended (woken
// when it completes, or after at most kSuspendNs) instead of returning at once:
// waiting warps then take no issue slots from the working ones.
constexpr uint32_t kSuspendNs = 200000;
__device__ __forceinline__ bool mbar_try_suspend(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "n"(kSuspendNs)
      : "memory");
  return ok != 0;
}
// 1-D bulk copy global -> shared, completion counted on `bar` (16-B aligned, size % 16 == 0)
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::
          "r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// Bounded wait: spins on try_wait until the phase with `parity` completes, the
// shared abort word is set by another warp, or the clock budget runs out (then
// records `code` in *err and sets the abort word).  Returns true on completion.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_w,
                                          int* err, int code) {
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_suspend(bar, parity)) return true;
    if (*abort_w) return false;
    if (clock64() - t0 > kWaitCycles) {
      atomicCAS(err, 0, code);
      *abort_w = 1;
      return false;
    }
  }
}

// The same wait for a whole consumer warp, with a warp-uniform answer: every
// lane polls the barrier (each gets acquire ordering on the staged data), the
// warp proceeds when all lanes saw the phase complete, and lane 0 alone
// decides an abort, broadcast to the warp.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort_w,
                                          int* err, int code) {
  const long long t0 = clock64();
  while (true) {
    const bool done = mbar_try_suspend(bar, parity);
    if (__all_sync(0xffffffffu, done)) return true;
    int stop = 0;
    if ((threadIdx.x & 31) == 0) {
      if (*abort_w) {
        stop = 1;
      } else if (clock64() - t0 > kWaitCycles) {
        atomicCAS(err, 0, code);
        *abort_w = 1;
        stop = 1;
      }
    }
    if (__shfl_sync(0xffffffffu, stop, 0)) return false;
  }
}

// ---------------------------------------------------------------------------
// tiled half-step
// ---------------------------------------------------------------------------
struct TKArgs {
  int64_t nseg, m_o;
  int P, R, B, logW;
  const int64_t* header;
  const int64_t* tstart;
  const uint2* ent;
  const int32_t* ptr;  // the CSR offsets (row lengths)
  const float* other;
  const float* base;
  const float* self_old;
  const float* sigma;  // optional stabilisers (else base - self_old)
  float* out;
  float w_old, w_new;
  float* prev;
  uint32_t* acc;
  int* fb_count;
  int* fb_list;
  int* fb_reset;
  int* err;
  PeerOut peers;
  unsigned int* done;
  const uint16_t* rowoff;  // two-pass kind: row byte offset per slot
  const float* expo;       // two-pass kind: exponent lam + potential per slot
};

// The state words of panel row r, addressed by its byte offset 4 r (the high
// half of an entry's meta word): sigma, high sum and low sum, in three arrays
// at fixed offsets.
__device__ __forceinline__ float* row_sigma(unsigned char* smem, uint32_t roff) {
  return reinterpret_cast<float*>(smem + kSigOff + roff);
}
__device__ __forceinline__ uint32_t* row_hi(unsigned char* smem, uint32_t roff) {
  return reinterpret_cast<uint32_t*>(smem + kHiOff + roff);
}
__device__ __forceinline__ uint32_t* row_lo(unsigned char* smem, uint32_t roff) {
  return reinterpret_cast<uint32_t*>(smem + kLoOff + roff);
}

// Row state of a panel (sigma, high and low sums at byte offsets SIG, HI, LO,
// one flag bit per row), set up and finished by NT threads.  Each thread has
// the global loads of kRowBatch rows in flight before it uses any of them
// (rows one at a time would cost one memory round trip each).
#ifndef SINKSLOT_ROW_BATCH
#define SINKSLOT_ROW_BATCH 4
#endif
constexpr int kRowBatch = SINKSLOT_ROW_BATCH;

__device__ __forceinline__ float radix_to_float(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// sigma of every panel row (the stabiliser: a.sigma, else base - self_old),
// zero sums, and the flag bits of rows longer than kMaxTiledRow (handed back
// from the start); row R (the dummy row of the padding) and any row past the
// panel's end get sigma 0.  Warp w initialises rows 32 w .. 32 w + 31, then
// 32 (w + NT/32) ...
template <int OUT, uint32_t SIG, uint32_t HI, uint32_t LO, int NT>
__device__ __forceinline__ void panel_rows_init(const TKArgs& a, unsigned char* smem,
                                                uint32_t* flags, int64_t row0, int rows,
                                                int warp, int lane) {
  for (int c0 = warp * 32; c0 <= a.R; c0 += NT * kRowBatch) {
    float sg[kRowBatch];
    bool longrow[kRowBatch];
#pragma unroll
    for (int k = 0; k < kRowBatch; ++k) {
      const int r = c0 + k * NT + lane;
      sg[k] = 0.0f;
      longrow[k] = false;
      if (r < rows && OUT != kOutMax) {
        sg[k] = a.sigma ? a.sigma[row0 + r] : __fsub_rn(a.base[row0 + r], a.self_old[row0 + r]);
        longrow[k] = a.ptr[row0 + r + 1] - a.ptr[row0 + r] > kMaxTiledRow;
      }
    }
#pragma unroll
    for (int k = 0; k < kRowBatch; ++k) {
      const int r0 = c0 + k * NT;  // warp-uniform
      if (r0 > a.R) break;
      const int r = r0 + lane;
      if (r <= a.R) {
        const uint32_t roff = 4u * (uint32_t)r;
        *reinterpret_cast<float*>(smem + SIG + roff) = sg[k];
        *reinterpret_cast<uint32_t*>(smem + HI + roff) = 0u;
        *reinterpret_cast<uint32_t*>(smem + LO + roff) = 0u;
      }
      const uint32_t word = __ballot_sync(0xffffffffu, longrow[k]);
      if (lane == 0) flags[r0 >> 5] = word;
    }
  }
}

// Each panel row's result from its sums: the largest term (max pass), the
// hand-back to the exact pass (flagged, or a sum below 2^-8), or lse = sigma +
// log(sum) and the epilogue.  Thread tid takes rows tid, tid + NT, ...
template <int OUT, int CHK, uint32_t SIG, uint32_t HI, uint32_t LO, int NT>
__device__ __forceinline__ void panel_rows_finish(const TKArgs& a, unsigned char* smem,
                                                  const uint32_t* flags, int64_t row0, int rows,
                                                  int tid, uint32_t& chk_bits) {
  for (int c0 = tid; c0 < rows; c0 += NT * kRowBatch) {
    float b[kRowBatch], old[kRowBatch], prv[kRowBatch];
#pragma unroll
    for (int k = 0; k < kRowBatch; ++k) {
      const int r = c0 + k * NT;
      b[k] = old[k] = prv[k] = 0.0f;
      if (OUT != kOutMax && r < rows) {
        const int64_t seg = row0 + r;
        b[k] = a.base[seg];
        if (OUT == kOutBlend || CHK == kChkMarg) old[k] = a.self_old[seg];
        if (CHK == kChkPot) prv[k] = a.prev[seg];
      }
    }
#pragma unroll
    for (int k = 0; k < kRowBatch; ++k) {
      const int r = c0 + k * NT;
      if (r >= rows) break;
      const int64_t seg = row0 + r;
      const uint32_t roff = 4u * (uint32_t)r;
      const uint32_t hi = *reinterpret_cast<const uint32_t*>(smem + HI + roff);
      if (OUT == kOutMax) {
        a.out[seg] = hi ? radix_to_float(hi) : -INFINITY;
        continue;
      }
      const unsigned long long q =
          ((unsigned long long)hi << kLoBits) + *reinterpret_cast<const uint32_t*>(smem + LO + roff);
      const bool flagged = (flags[r >> 5] >> (r & 31)) & 1u;
      if (flagged || q < kFixMin) {
        a.fb_list[atomicAdd(a.fb_count, 1)] = (int)seg;
        continue;
      }
      const float tot = (float)((double)q * kFixInv);
      const float lse = __fadd_rn(*reinterpret_cast<const float*>(smem + SIG + roff), logf(tot));
      segment_epilogue_loaded<OUT, CHK>(seg, lse, true, b[k], old[k], prv[k], a.out, a.w_old,
                                        a.w_new, a.prev, chk_bits, a.peers);
    }
  }
}

// One entry {meta, lam bits} against ring stage S: the exponent d = lam +
// potential[column] - sigma of its term, and its row's byte offset.  Padding
// entries name the dummy row with lam = -inf, so d = -inf and the term is an
// exact zero.
template <int S>
__device__ __forceinline__ float entry_exponent(unsigned char* smem, uint2 e, uint32_t& roff) {
  roff = e.x >> 16;
  const float pot = *reinterpret_cast<const float*>(smem + S * kStageBytes + (e.x & 0xFFFFu));
  return __fsub_rn(__fadd_rn(__uint_as_float(e.y), pot), *row_sigma(smem, roff));
}

// 2^x (hardware approximation; results below 2^-126 flush to zero, far below
// the 2^-32 resolution of the sums)
__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// exp(d) in 2^-32 fixed point, added to the row's high and low partial sums.
// Called for every entry; when d exceeds the cap (or is NaN) the caller has
// flagged the row for the exact pass and its sums are unused.
__device__ __forceinline__ void accumulate(unsigned char* smem, uint32_t roff, float d) {
  const unsigned long long q = __float2ull_rn(exp2_approx(d * 1.44269504088896341f) * kFixScale);
  atomicAdd(row_hi(smem, roff), (uint32_t)(q >> kLoBits));
  atomicAdd(row_lo(smem, roff), (uint32_t)q & ((1u << kLoBits) - 1u));
}

__device__ __forceinline__ void flag_row(uint32_t* flags, uint2 e) {
  const uint32_t r = meta_row(e.x);
  atomicOr(flags + (r >> 5), 1u << (r & 31));
}

// Prefetch of a byte range into L2 (16-byte aligned start, size a multiple of 16).
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(p), "r"(bytes) : "memory");
}

// Entries [e0, e1) of the layout into L2, in prefetches of at most kPfBytes
// (tile ranges start on 256-byte boundaries and span whole 256-byte slabs).
__device__ __forceinline__ void prefetch_entries(const uint2* ent, int64_t e0, int64_t e1) {
  const char* p = reinterpret_cast<const char*>(ent + e0);
  int64_t left = (e1 - e0) * (int64_t)sizeof(uint2);
  while (left > 0) {
    const uint32_t n = left < (int64_t)kPfBytes ? (uint32_t)left : kPfBytes;
    prefetch_l2(p, n);
    p += n;
    left -= n;
  }
}

// Lane `lane` of slabs g .. g+kGroup-1 of the tile whose entries start at e0
// (only the slabs below nsl are loaded): coalesced 8-byte streaming loads, 256
// bytes per slab.
__device__ __forceinline__ void load_group(const uint2* ent, int64_t e0, int nsl, int g, int lane,
                                           uint2 (&e)[kGroup]) {
  const uint2* p = ent + e0 + (int64_t)g * kSlab + lane;
#pragma unroll
  for (int j = 0; j < kGroup; ++j)
    if (g + j < nsl) e[j] = ld_stream(p + j * kSlab);
}

// The terms of a group of `cnt` (>= 1) slabs against ring stage S; when the
// whole group exists one vote checks the cap of its terms.
template <int S>
__device__ __forceinline__ void process_group(unsigned char* smem, uint32_t* flags,
                                              const uint2 (&e)[kGroup], int cnt, float capd) {
  if (cnt >= kGroup) {
    uint32_t ro[kGroup];
    float d[kGroup];
    bool in_cap = true;
#pragma unroll
    for (int j = 0; j < kGroup; ++j) {
      d[j] = entry_exponent<S>(smem, e[j], ro[j]);
      in_cap &= d[j] <= capd;
    }
    if (!__all_sync(0xffffffffu, in_cap)) {
#pragma unroll
      for (int j = 0; j < kGroup; ++j)
        if (!(d[j] <= capd)) flag_row(flags, e[j]);
    }
#pragma unroll
    for (int j = 0; j < kGroup; ++j) accumulate(smem, ro[j], d[j]);
  } else {
#pragma unroll
    for (int j = 0; j < kGroup - 1; ++j) {
      if (j < cnt) {
        uint32_t ro;
        const float d = entry_exponent<S>(smem, e[j], ro);
        if (!(d <= capd)) flag_row(flags, e[j]);
        accumulate(smem, ro, d);
      }
    }
  }
}

// Max mode: the largest term lam + potential[column] of each row, as the
// order-preserving integer image of the float (float_to_radix) in the row's
// high-sum word, which starts at 0 (below the image of every float).  Padding
// adds -inf to the dummy row.
template <int S>
__device__ __forceinline__ void process_group_max(unsigned char* smem, const uint2 (&e)[kGroup],
                                                  int cnt) {
#pragma unroll
  for (int j = 0; j < kGroup; ++j) {
    if (j < cnt) {
      const float pot =
          *reinterpret_cast<const float*>(smem + S * kStageBytes + (e[j].x & 0xFFFFu));
      atomicMax(row_hi(smem, e[j].x >> 16), float_to_radix(__fadd_rn(__uint_as_float(e[j].y), pot)));
    }
  }
}


// A consumer warp's groups of one tile -- slabs [0, nsl) of the entries from
// e0 -- against ring stage S.  Each group is loaded one ahead (in `en`): behind
// the warp's last group of this tile its first group of the next tile (f0,
// nsl_next) goes in flight.
template <int S, int OUT>
__device__ __forceinline__ void consume_tile(unsigned char* smem, uint32_t* flags,
                                             const uint2* ent, int64_t e0, int nsl, int64_t f0,
                                             int nsl_next, int warp, int lane, float capd,
                                             uint2 (&en)[kGroup]) {
  constexpr int kStep = kGroup * kConsumerWarps;
  for (int g = kGroup * warp; g < nsl; g += kStep) {
    uint2 e[kGroup];
#pragma unroll
    for (int j = 0; j < kGroup; ++j) e[j] = en[j];
    if (g + kStep < nsl)
      load_group(ent, e0, nsl, g + kStep, lane, en);
    else
      load_group(ent, f0, nsl_next, kGroup * warp, lane, en);
    if (OUT == kOutMax)
      process_group_max<S>(smem, e, nsl - g);
    else
      process_group<S>(smem, flags, e, nsl - g, capd);
  }
}

// consume_tile with the stage index s (< kStages) as a template argument, so
// that the potential's address is the meta word's low half plus a constant
template <int OUT, int S = 0>
__device__ __forceinline__ void consume_stage(int s, unsigned char* smem, uint32_t* flags,
                                              const uint2* ent, int64_t e0, int nsl, int64_t f0,
                                              int nsl_next, int warp, int lane, float capd,
                                              uint2 (&en)[kGroup]) {
  if constexpr (S + 1 < kStages) {
    if (s != S) {
      consume_stage<OUT, S + 1>(s, smem, flags, ent, e0, nsl, f0, nsl_next, warp, lane, capd, en);
      return;
    }
  }
  consume_tile<S, OUT>(smem, flags, ent, e0, nsl, f0, nsl_next, warp, lane, capd, en);
}

template <int OUT, int CHK>
__global__ void __launch_bounds__(kPipeThreads, 1) tiled_half_step_kernel(const TKArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int W = 1 << a.logW;
  // the potential ring, the row state, the flag bits, the mbarriers and the
  // abort word at their fixed offsets
  uint32_t* flags = reinterpret_cast<uint32_t*>(smem + kFlagOff);
  unsigned long long* bars = reinterpret_cast<unsigned long long*>(smem + kBarOff);
  volatile int* abort_w = reinterpret_cast<volatile int*>(bars + 2 * kStages);
  // bars, kStages each: potential block full, potential block empty
  const uint32_t bar0 = smem_u32(bars);
  auto pot_full = [&](int s) { return bar0 + 8u * (uint32_t)s; };
  auto pot_empty = [&](int s) { return bar0 + 8u * (uint32_t)(kStages + s); };

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  // a layout built for another kind or geometry: fail (the host reports it)
  if (a.header[1] != kTilesStaged || a.header[2] != a.P || a.header[3] != a.B) {
    chain_enter();
    if (tid == 0) atomicCAS(a.err, 0, 4);
    return;
  }
  // The kernel may start while the previous launch of the loop is finishing
  // (programmatic dependent launch).  Before chain_enter it touches only what
  // no running launch writes: its shared memory, the layout, and (consumers,
  // first panel) the row state's inputs base / self_old / the CSR offsets --
  // self_old is this side's own output, written at least three launches back.
  // The gathered potential, the stabilisers of a max pass, the error word and
  // the other side's handed-back counter are read or written after it.
#if !SINKSLOT_TILE_EARLY_INIT
  chain_enter();
  // a pipeline wait of an earlier launch timed out: do nothing (the host reports it)
  if (*(volatile int*)a.err != 0) return;
#endif
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(pot_full(s), 1);
      mbar_init(pot_empty(s), kConsumerWarps);
    }
    *abort_w = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
#if !SINKSLOT_TILE_EARLY_INIT
  if (a.fb_reset && blockIdx.x == 0 && tid == 0) *a.fb_reset = 0;
#endif
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ---------------- producer warp: lane 0 issues every copy ----------------
    if (lane != 0) return;
#if SINKSLOT_TILE_EARLY_INIT
    chain_enter();
    if (*(volatile int*)a.err != 0) return;
#endif
    long long nb = 0;  // blocks issued so far: stage nb % kStages, use nb / kStages
    int sb = 0;
    uint32_t ub = 0;   // parity of the current use of stage sb
    bool ok = true;
    for (int p = blockIdx.x; ok && p < a.P; p += gridDim.x) {
      if ((int64_t)p * a.R >= a.nseg) break;
      const int64_t pb = (int64_t)p * a.B;
      // entries of tiles [0, kPfLead) into L2 now; then, with block b, those of
      // tile b + kPfLead (pf0 .. pf1; the end after it is loaded a tile early)
      int64_t pf0 = a.tstart[pb + (kPfLead < a.B ? kPfLead : a.B)];
      if (kPfLead > 0) prefetch_entries(a.ent, a.tstart[pb], pf0);
      int64_t pf1 = kPfLead < a.B ? a.tstart[pb + kPfLead + 1] : pf0;
      for (int b = 0; ok && b < a.B; ++b) {
        if (b + kPfLead < a.B) {
          const int64_t s0 = pf0, s1 = pf1;
          pf0 = pf1;
          if (b + kPfLead + 2 <= a.B) pf1 = a.tstart[pb + b + kPfLead + 2];
          // tile b + kPfLead's entries into L2 ahead of the consumers' loads
          prefetch_entries(a.ent, s0, s1);
        }
        if (nb >= kStages && !(ok = mbar_wait(pot_empty(sb), ub ^ 1u, abort_w, a.err, 1))) break;
        const int64_t c0 = (int64_t)b * W;
        const int64_t cnt = std::min<int64_t>(W, a.m_o - c0);
        const int64_t body = cnt & ~int64_t(3);
        float* dst = reinterpret_cast<float*>(smem + (size_t)sb * kStageBytes);
        // the last few floats when the block is not a multiple of 16 bytes
        for (int64_t q = body; q < cnt; ++q) dst[q] = a.other[c0 + q];
        mbar_arrive_tx(pot_full(sb), (uint32_t)(body * 4));
        if (body > 0) bulk_g2s(smem_u32(dst), a.other + c0, (uint32_t)(body * 4), pot_full(sb));
        ++nb;
        if (++sb == kStages) { sb = 0; ub ^= 1u; }
      }
    }
    if (!ok) {
      // wait (bounded) for the copies in flight so none lands after the CTA leaves
      for (long long k = std::max(0ll, nb - kStages); k < nb; ++k) {
        const long long t0 = clock64();
        while (!mbar_try(pot_full((int)(k % kStages)), (uint32_t)((k / kStages) & 1)) &&
               clock64() - t0 < kWaitCycles) {
        }
      }
    }
    return;
  }

  // ---------------- consumer warps ----------------
  const long long longest = a.header[0] > 0 ? a.header[0] : 1;
  int lg = 0;
  while ((1ll << lg) < longest) ++lg;
  const int k = kLoBits - lg;
  // terms above 2^k would overflow the high-part sum of the longest row
  const float capd = (longest <= kMaxTiledRow && k >= 1) ? ((float)k - 0.01f) * 0.69314718f
                                                         : -INFINITY;
  uint32_t chk_bits = 0;
  int sb = 0;
  uint32_t ub = 0;
  bool ok = true;
  bool entered = !SINKSLOT_TILE_EARLY_INIT;
  if (!entered && a.sigma != nullptr) {
    chain_enter();  // the stabilisers are the previous launch's output
    entered = true;
    if (*(volatile int*)a.err != 0) ok = false;
    if (a.fb_reset && blockIdx.x == 0 && tid == 0) *a.fb_reset = 0;
  }
  // Control flow that crosses a consumer barrier follows the shared abort word
  // (identical for all consumers after bar.sync), never a thread-local flag --
  // except the error word read right after chain_enter, which every thread
  // reads after the previous launch has completed (the same value for all).
  for (int p = blockIdx.x; ok && !*abort_w && p < a.P; p += gridDim.x) {
    const int64_t row0 = (int64_t)p * a.R;
    const int rows = (int)std::min<int64_t>(a.R, a.nseg - row0);
    if (rows <= 0) break;
    const int64_t pb = (int64_t)p * a.B;
    // row state (warp w initialises rows 32w .. 32w+31, then 32(w+31) ...) and
    // flag words: rows longer than kMaxTiledRow are handed back from the start
    panel_rows_init<OUT, kSigOff, kHiOff, kLoOff, kConsumers>(a, smem, flags, row0, rows, warp,
                                                              lane);
    // Tile b holds slabs [e0, e1) / 32 of the layout.  Warp w takes groups of
    // kGroup consecutive slabs starting at kGroup*w, kGroup*(w + warps), ...
    // Its groups, taken in order across the panel's tiles, are loaded one
    // ahead: while a group is processed the next one (in this tile, or the
    // warp's first of the next tile) is in flight.  tile starts: e0, e1 bound
    // tile b, f1n the end of tile b + 1 (loaded a tile ahead of its use, so no
    // tile waits on a global load of its bounds)
    int64_t e0 = a.tstart[pb], e1 = a.tstart[pb + 1];
    int64_t f1n = a.B > 1 ? a.tstart[pb + 2] : e1;
    uint2 en[kGroup];
    load_group(a.ent, e0, (int)((e1 - e0) / kSlab), kGroup * warp, lane, en);
    if (!entered) {
      chain_enter();
      entered = true;
      if (*(volatile int*)a.err != 0) break;
      if (a.fb_reset && blockIdx.x == 0 && tid == 0) *a.fb_reset = 0;
    }
    asm volatile("bar.sync 1, %0;\n" ::"n"(kConsumers) : "memory");
    for (int b = 0; ok && b < a.B; ++b) {
      const int nsl = (int)((e1 - e0) / kSlab);
      const int64_t f0 = e1;
      const int64_t f1 = b + 1 < a.B ? f1n : e1;
      const int nsl_next = (int)((f1 - f0) / kSlab);
      if (b + 2 < a.B) f1n = a.tstart[pb + b + 3];
      // no group of this warp in tile b: its first of tile b + 1 goes in flight now
      if (kGroup * warp >= nsl) load_group(a.ent, f0, nsl_next, kGroup * warp, lane, en);
      const int s = sb;
      if (!(ok = warp_wait(pot_full(s), ub, abort_w, a.err, 3))) break;
      if (++sb == kStages) { sb = 0; ub ^= 1u; }
      consume_stage<OUT>(s, smem, flags, a.ent, e0, nsl, f0, nsl_next, warp, lane, capd, en);
      __syncwarp();
      if (lane == 0) mbar_arrive(pot_empty(s));
      e0 = f0;
      e1 = f1;
    }
    asm volatile("bar.sync 1, %0;\n" ::"n"(kConsumers) : "memory");
    if (*abort_w) break;
    panel_rows_finish<OUT, CHK, kSigOff, kHiOff, kLoOff, kConsumers>(a, smem, flags, row0, rows,
                                                                      tid, chk_bits);
    asm volatile("bar.sync 1, %0;\n" ::"n"(kConsumers) : "memory");
  }
  chain_release();
  check_reduce<CHK>(chk_bits, a.acc);
  if (a.peers.n > 0) {
    // consumers only: the producer warp stored no potential
    asm volatile("bar.sync 1, %0;\n" ::"n"(kConsumers) : "memory");
    peer_cta_done(a.peers, a.done);
  }
}


// ---------------------------------------------------------------------------
// two-pass kind
// ---------------------------------------------------------------------------
// When the gathered axis is too long to stage once per panel (P * m_o * 4
// bytes per half-step), the half-step runs in two streaming passes over the
// same layout:
//   block_gather_kernel: CTA (b, q) copies block b of the gathered potential
//     into shared memory once and walks the tiles (p, b) of the panels p of
//     chunk q in work items of at most 32 slabs; each slot's exponent lam +
//     potential[column] is stored at the slot's own index of the exponent
//     array (coalesced 2- and 4-byte loads and 4-byte stores; padding slots
//     give -inf);
//   panel_sum_kernel: one CTA per panel streams the panel's slots (tiles
//     (p, 0 .. B-1) are contiguous) -- the row byte offset and the exponent --
//     and sums exp(exponent - sigma) into the row state exactly as the staged
//     kernel does (same fixed point, cap, hand-back rule and epilogue), so the
//     two kinds give the same bits.  No gather and no potential ring: the whole
//     shared memory holds row state (up to kRowCap2 - 1 rows per panel).
// Bytes per slot and half-step: 2 + 4 read and 4 written, then 2 + 4 read (the
// layout keeps each slot split into a row offset, a column offset and lam).
constexpr int kGatherWarps = 16;
constexpr int kGatherThreads = 32 * kGatherWarps;
constexpr int kGatherCtasPerSm = 3;  // 64 KB blocks: three per SM
#ifndef SINKSLOT_GATHER_UNROLL
#define SINKSLOT_GATHER_UNROLL 8
#endif
constexpr int kGatherUnroll = SINKSLOT_GATHER_UNROLL;  // slabs a lane has in flight
constexpr int kSumWarps = 32;
constexpr int kSumThreads = 32 * kSumWarps;
constexpr int kSumGroup = 8;         // slabs a warp loads together, one group ahead
#ifndef SINKSLOT_SUM_PREFETCH
#define SINKSLOT_SUM_PREFETCH 1
#endif
// the group after the one in flight prefetched into L2 by the warp's lane 0
constexpr bool kSumPrefetch = SINKSLOT_SUM_PREFETCH;

struct BGArgs {
  int64_t m_o;
  int P, B, logW, pchunk;
  const int64_t* header;
  const int64_t* tstart;
  const uint16_t* coloff;
  const float* lamv;
  const float* other;
  float* expo;
  int* err;
};

__device__ __forceinline__ bool layout_matches(const int64_t* header, int kind, int P, int B) {
  return header[1] == kind && header[2] == P && header[3] == B;
}

// The block-gather CTA's tiles (p, b), p in its chunk, cut into work items of at
// most kItemSlabs slabs (a tile of the 2^24 problem is one item of ~24 slabs,
// one of 2^20 ~7 items of 32): a table in shared memory after the potential
// block holds each tile's first slot, its slabs and the items before it
// (exclusive prefix).  Warp w takes items w, w + kGatherWarps, ...; while it
// works on one, the slots of its next are prefetched into L2.  (One warp per
// whole tile left most warps idle where a CTA's chunk has few, large tiles.)
constexpr int kGatherMaxChunk = 768;  // tiles per CTA (table: 9 KB)
constexpr int kItemSlabs = 32;

__host__ __device__ __forceinline__ size_t gather_table_off(int logW) {
  return (size_t)4 << logW;
}
// the potential block, then the table: first slots, slab counts and item
// prefixes of kGatherMaxChunk tiles (+ the total)
__host__ __device__ __forceinline__ size_t gather_smem(int logW) {
  return gather_table_off(logW) + (size_t)kGatherMaxChunk * 8 + (size_t)(kGatherMaxChunk + 1) * 4;
}

// slots of slabs [0, ns) from slot s0 of the split arrays into L2 (tile ranges
// start on 32-slot boundaries: 64- and 128-byte aligned, whole slabs)
__device__ __forceinline__ void prefetch_item(const uint16_t* coloff, const float* lamv,
                                              uint32_t s0, int ns) {
  if (ns <= 0) return;
  prefetch_l2(coloff + s0, (uint32_t)ns * kSlab * 2u);
  prefetch_l2(lamv + s0, (uint32_t)ns * kSlab * 4u);
}

__global__ void __launch_bounds__(kGatherThreads, kGatherCtasPerSm)
    block_gather_kernel(const BGArgs a) {
  extern __shared__ __align__(16) unsigned char potb[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (!layout_matches(a.header, kTilesTwoPass, a.P, a.B)) {
    chain_enter();
    if (tid == 0) atomicCAS(a.err, 0, 4);
    return;
  }
  const int b = blockIdx.x;
  const int p0 = blockIdx.y * a.pchunk;
  const int nt = max(0, min(a.P, p0 + a.pchunk) - p0);  // <= kGatherMaxChunk
  uint32_t* te0 = reinterpret_cast<uint32_t*>(potb + gather_table_off(a.logW));
  int32_t* tsl = reinterpret_cast<int32_t*>(te0 + kGatherMaxChunk);
  int32_t* ipre = tsl + kGatherMaxChunk;
  // the tile table (the layout is static: built while the previous launch
  // finishes); slots < 2^32 because nnz < 2^32
  for (int i = tid; i < nt; i += kGatherThreads) {
    const int64_t t = (int64_t)(p0 + i) * a.B + b;
    const int64_t s0 = a.tstart[t];
    const int ns = (int)((a.tstart[t + 1] - s0) >> 5);
    te0[i] = (uint32_t)s0;
    tsl[i] = ns;
    ipre[i] = (ns + kItemSlabs - 1) / kItemSlabs;  // items of tile i, for now
  }
  __syncthreads();
  if (warp == 0) {
    // exclusive prefix of the item counts, in place: each lane sums its own run
    // [i0, i1), a warp scan gives the runs' offsets, each lane rewrites its run
    const int per = (nt + 31) / 32;
    const int i0 = min(nt, lane * per), i1 = min(nt, i0 + per);
    int run = 0;
    for (int i = i0; i < i1; ++i) run += ipre[i];
    int incl = run;
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int acc = incl - run;
    for (int i = i0; i < i1; ++i) {
      const int c = ipre[i];
      ipre[i] = acc;
      acc += c;
    }
    if (lane == 31) ipre[nt] = incl;
  }
  __syncthreads();
  const int items = ipre[nt];
  int cur = 0;  // the tile of the warp's latest located item (items only grow)
  // item j: its first slot and slabs
  auto locate = [&](int j, uint32_t& s0, int& ns) {
    while (ipre[cur + 1] <= j) ++cur;
    const int sub = j - ipre[cur];
    s0 = te0[cur] + (uint32_t)(sub * kItemSlabs * kSlab);
    ns = min(kItemSlabs, tsl[cur] - sub * kItemSlabs);
  };
  uint32_t s0 = 0;
  int ns = 0;
  if (warp < items) {
    locate(warp, s0, ns);
    if (lane == 0) prefetch_item(a.coloff, a.lamv, s0, ns);
  }
  chain_enter();
  if (*(volatile int*)a.err != 0) return;  // an earlier launch failed: do nothing
  const int64_t c0 = (int64_t)b << a.logW;
  const int cnt = (int)std::min<int64_t>((int64_t)1 << a.logW, a.m_o - c0);
  float* pot = reinterpret_cast<float*>(potb);
  for (int i = tid; i < cnt; i += kGatherThreads) pot[i] = a.other[c0 + i];
  __syncthreads();
  for (int j = warp; j < items; j += kGatherWarps) {
    // the warp's next item: located and prefetched while this one is processed
    uint32_t n0 = 0;
    int nns = 0;
    if (j + kGatherWarps < items) {
      locate(j + kGatherWarps, n0, nns);
      if (lane == 0) prefetch_item(a.coloff, a.lamv, n0, nns);
    }
    const uint16_t* cs = a.coloff + s0 + lane;
    const float* ls = a.lamv + s0 + lane;
    float* dst = a.expo + s0 + lane;
    int s = 0;
    for (; s + kGatherUnroll <= ns; s += kGatherUnroll) {
      uint32_t c[kGatherUnroll];
      float l[kGatherUnroll];
#pragma unroll
      for (int u = 0; u < kGatherUnroll; ++u) {
        c[u] = ld_stream(cs + (s + u) * kSlab);
        l[u] = ld_stream(ls + (s + u) * kSlab);
      }
#pragma unroll
      for (int u = 0; u < kGatherUnroll; ++u)
        __stcs(dst + (s + u) * kSlab,
               __fadd_rn(l[u], *reinterpret_cast<const float*>(potb + c[u])));
    }
    for (; s < ns; ++s) {
      const uint32_t c = ld_stream(cs + s * kSlab);
      __stcs(dst + s * kSlab,
             __fadd_rn(ld_stream(ls + s * kSlab), *reinterpret_cast<const float*>(potb + c)));
    }
    s0 = n0;
    ns = nns;
  }
  chain_release();
}

__device__ __forceinline__ float* row_sigma2(unsigned char* smem, uint32_t roff) {
  return reinterpret_cast<float*>(smem + kSigOff2 + roff);
}
__device__ __forceinline__ uint32_t* row_hi2(unsigned char* smem, uint32_t roff) {
  return reinterpret_cast<uint32_t*>(smem + kHiOff2 + roff);
}
__device__ __forceinline__ uint32_t* row_lo2(unsigned char* smem, uint32_t roff) {
  return reinterpret_cast<uint32_t*>(smem + kLoOff2 + roff);
}

// slabs g .. g + kSumGroup - 1 (those below nsl) of the panel whose slots start
// at e0: lane `lane`'s row offsets and exponents
__device__ __forceinline__ void load_sum_group(const uint16_t* rowoff, const float* expo,
                                               int64_t e0, int nsl, int g, int lane,
                                               uint32_t (&ro)[kSumGroup],
                                               float (&x)[kSumGroup]) {
  const int64_t q = e0 + (int64_t)g * kSlab + lane;
#pragma unroll
  for (int j = 0; j < kSumGroup; ++j)
    if (g + j < nsl) {
      ro[j] = ld_stream(rowoff + q + j * kSlab);
      x[j] = ld_stream(expo + q + j * kSlab);
    }
}

// the slots of slabs g .. g + kSumGroup - 1 (below nsl) into L2
__device__ __forceinline__ void prefetch_sum_group(const uint16_t* rowoff, const float* expo,
                                                   int64_t e0, int nsl, int g) {
  if (g >= nsl) return;
  const int64_t q = e0 + (int64_t)g * kSlab;
  const uint32_t n = (uint32_t)min(kSumGroup, nsl - g) * kSlab;
  prefetch_l2(rowoff + q, n * 2u);
  prefetch_l2(expo + q, n * 4u);
}

template <int OUT, int CHK>
__global__ void __launch_bounds__(kSumThreads, 1) panel_sum_kernel(const TKArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint32_t* flags = reinterpret_cast<uint32_t*>(smem + kFlagOff2);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (!layout_matches(a.header, kTilesTwoPass, a.P, a.B)) {
    chain_enter();
    if (tid == 0) atomicCAS(a.err, 0, 4);
    return;
  }
  const long long longest = a.header[0] > 0 ? a.header[0] : 1;
  int lg = 0;
  while ((1ll << lg) < longest) ++lg;
  const int k = kLoBits - lg;
  // terms above 2^k would overflow the high-part sum of the longest row
  const float capd = (longest <= kMaxTiledRow && k >= 1) ? ((float)k - 0.01f) * 0.69314718f
                                                         : -INFINITY;
  uint32_t chk_bits = 0;
  // Before chain_enter the kernel reads only what no running launch writes:
  // the layout, base, self_old (this side's own output, written at least four
  // launches back) and the CSR offsets.  The exponents (the previous launch's
  // output), the stabilisers of a max pass and the error word come after it.
  bool entered = false;
  if (a.sigma != nullptr) {
    chain_enter();
    entered = true;
    if (a.fb_reset && blockIdx.x == 0 && tid == 0) *a.fb_reset = 0;
  }
  constexpr int kStep = kSumGroup * kSumWarps;
  for (int p = blockIdx.x; p < a.P; p += gridDim.x) {
    const int64_t row0 = (int64_t)p * a.R;
    const int rows = (int)std::min<int64_t>(a.R, a.nseg - row0);
    if (rows <= 0) break;
    // row state and flag words (rows longer than kMaxTiledRow are handed back
    // from the start)
    panel_rows_init<OUT, kSigOff2, kHiOff2, kLoOff2, kSumThreads>(a, smem, flags, row0, rows,
                                                                  warp, lane);
    const int64_t e0 = a.tstart[(int64_t)p * a.B];
    const int nsl = (int)((a.tstart[(int64_t)(p + 1) * a.B] - e0) >> 5);
    if (!entered) {
      chain_enter();
      entered = true;
      if (a.fb_reset && blockIdx.x == 0 && tid == 0) *a.fb_reset = 0;
    }
    // every thread reads the word after the previous launches completed: the
    // same value in all threads
    if (*(volatile int*)a.err != 0) break;
    __syncthreads();
    uint32_t ron[kSumGroup];
    float xn[kSumGroup];
    if (kSumPrefetch && lane == 0)
      prefetch_sum_group(a.rowoff, a.expo, e0, nsl, kSumGroup * warp + kStep);
    load_sum_group(a.rowoff, a.expo, e0, nsl, kSumGroup * warp, lane, ron, xn);
    for (int g = kSumGroup * warp; g < nsl; g += kStep) {
      uint32_t ro[kSumGroup];
      float x[kSumGroup];
#pragma unroll
      for (int j = 0; j < kSumGroup; ++j) {
        ro[j] = ron[j];
        x[j] = xn[j];
      }
      if (kSumPrefetch && lane == 0) prefetch_sum_group(a.rowoff, a.expo, e0, nsl, g + 2 * kStep);
      load_sum_group(a.rowoff, a.expo, e0, nsl, g + kStep, lane, ron, xn);
      const int cnt = nsl - g;
      if (OUT == kOutMax) {
#pragma unroll
        for (int j = 0; j < kSumGroup; ++j)
          if (j < cnt) atomicMax(row_hi2(smem, ro[j]), float_to_radix(x[j]));
      } else if (cnt >= kSumGroup) {
        float d[kSumGroup];
        bool in_cap = true;
#pragma unroll
        for (int j = 0; j < kSumGroup; ++j) {
          d[j] = __fsub_rn(x[j], *row_sigma2(smem, ro[j]));
          in_cap &= d[j] <= capd;
        }
        if (!__all_sync(0xffffffffu, in_cap)) {
#pragma unroll
          for (int j = 0; j < kSumGroup; ++j)
            if (!(d[j] <= capd)) {
              const uint32_t r = ro[j] >> 2;
              atomicOr(flags + (r >> 5), 1u << (r & 31));
            }
        }
#pragma unroll
        for (int j = 0; j < kSumGroup; ++j) {
          const unsigned long long q =
              __float2ull_rn(exp2_approx(d[j] * 1.44269504088896341f) * kFixScale);
          atomicAdd(row_hi2(smem, ro[j]), (uint32_t)(q >> kLoBits));
          atomicAdd(row_lo2(smem, ro[j]), (uint32_t)q & ((1u << kLoBits) - 1u));
        }
      } else {
#pragma unroll
        for (int j = 0; j < kSumGroup - 1; ++j) {
          if (j < cnt) {
            const float d = __fsub_rn(x[j], *row_sigma2(smem, ro[j]));
            if (!(d <= capd)) {
              const uint32_t r = ro[j] >> 2;
              atomicOr(flags + (r >> 5), 1u << (r & 31));
            }
            const unsigned long long q =
                __float2ull_rn(exp2_approx(d * 1.44269504088896341f) * kFixScale);
            atomicAdd(row_hi2(smem, ro[j]), (uint32_t)(q >> kLoBits));
            atomicAdd(row_lo2(smem, ro[j]), (uint32_t)q & ((1u << kLoBits) - 1u));
          }
        }
      }
    }
    __syncthreads();
    panel_rows_finish<OUT, CHK, kSigOff2, kHiOff2, kLoOff2, kSumThreads>(a, smem, flags, row0,
                                                                         rows, tid, chk_bits);
    __syncthreads();
  }
  if (!entered) chain_enter();
  chain_release();
  check_reduce<CHK>(chk_bits, a.acc);
  if (a.peers.n > 0) {
    __syncthreads();
    peer_cta_done(a.peers, a.done);
  }
}

static int launch_block_gather(const TiledHalfStep& h, cudaStream_t st) {
  const TileGeom& g = h.g;
  const LayoutPtrs L = carve_layout(const_cast<void*>(h.layout), g);
  BGArgs a;
  a.m_o = g.m_o;
  a.P = g.P;
  a.B = g.B;
  a.logW = g.logW;
  a.header = L.header;
  a.tstart = L.tstart;
  a.coloff = L.coloff;
  a.lamv = L.lamv;
  a.other = h.other;
  a.expo = L.expo;
  a.err = h.err;
  // panel chunks: about four waves of CTAs in all (each restages its block),
  // at most kGatherMaxChunk tiles each
  const int64_t waves = 4 * (int64_t)kGatherCtasPerSm * num_sms();
  int64_t Q = std::min<int64_t>(g.P, std::max<int64_t>(1, ceil_div64(waves, g.B)));
  Q = std::max<int64_t>(Q, ceil_div64(g.P, kGatherMaxChunk));
  a.pchunk = (int)ceil_div64(g.P, Q);
  Q = ceil_div64(g.P, a.pchunk);
  SINKSLOT_REQUIRE(Q <= 65535 && a.pchunk <= kGatherMaxChunk,
                   "two-pass half step: too many panel chunks");
  const size_t smem = gather_smem(g.logW);
  static bool configured[64] = {};
  int dev = 0;
  SINKSLOT_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    SINKSLOT_CUDA_TRY(cudaFuncSetAttribute(block_gather_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)gather_smem(kMaxLogW)));
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  SINKSLOT_CUDA_TRY(launch_chained(block_gather_kernel, dim3((unsigned)g.B, (unsigned)Q),
                                   dim3(kGatherThreads), smem, st, a));
  return kOk;
}

template <int OUT, int CHK>
static int launch_panel_sum(const TKArgs& a, cudaStream_t st) {
  static bool configured[64] = {};
  int dev = 0;
  SINKSLOT_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    SINKSLOT_CUDA_TRY(cudaFuncSetAttribute(panel_sum_kernel<OUT, CHK>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)kSumSmem));
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  const int grid = std::min(a.P, num_sms());
  SINKSLOT_CUDA_TRY(launch_chained(panel_sum_kernel<OUT, CHK>, dim3(grid), dim3(kSumThreads),
                                   kSumSmem, st, a));
  return kOk;
}

template <int OUT, int CHK>
static int launch_tiled_kind(const TKArgs& a, const TileGeom& g, cudaStream_t st);

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
  SINKSLOT_CUDA_TRY(launch_chained(tiled_half_step_kernel<OUT, CHK>, dim3(grid),
                                   dim3(kPipeThreads), smem, st, a));
  return kOk;
}

static TKArgs tk_args(const TiledHalfStep& h) {
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
  a.ent = L.ent;
  a.ptr = h.ptr;
  a.other = h.other;
  a.base = h.base;
  a.self_old = h.self_old;
  a.sigma = h.sigma;
  a.out = h.out;
  a.w_old = h.w_old;
  a.w_new = h.w_new;
  a.prev = h.prev;
  a.acc = h.acc;
  a.fb_count = h.fb_count;
  a.fb_list = h.fb_list;
  a.fb_reset = h.fb_count_reset;
  a.err = h.err;
  a.peers = h.peers;
  a.done = h.done;
  a.rowoff = L.rowoff;
  a.expo = L.expo;
  return a;
}

static int exact_handed_back(const TiledHalfStep& h, int out_mode, int chk, cudaStream_t st,
                             unsigned int* ctas) {
  // exact pass over the rows the tiled pass handed back (stabilised by their
  // own running maximum: the exact kernel needs no sigma)
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
  x.peers = h.peers;
  x.done = h.done;
  if (ctas) *ctas += (unsigned)std::min(h.g.P, num_sms());
  return half_step(x, out_mode, chk, st, ctas);
}

int tiled_half_step(const TiledHalfStep& h, int out_mode, int chk, cudaStream_t st,
                    unsigned int* ctas) {
  SINKSLOT_REQUIRE(h.base != nullptr, "tiled half step: base is required");
  SINKSLOT_REQUIRE(h.fb_count && h.fb_list && h.err, "tiled half step: fallback list is required");
  SINKSLOT_REQUIRE(out_mode != kOutNone || chk == kChkMarg, "half step: check-only needs a check");
  SINKSLOT_REQUIRE((reinterpret_cast<uintptr_t>(h.other) & 15u) == 0,
                   "tiled half step: the gathered potential must be 16-byte aligned");
  if (h.g.nseg <= 0) return kOk;
  const TKArgs a = tk_args(h);
  // two-pass kind: the exponents first -- except after a max pass over the same
  // potential (sigma given), which left them in place
  if (h.g.kind == kTilesTwoPass && h.sigma == nullptr) SINKSLOT_TRY(launch_block_gather(h, st));
  if (out_mode == kOutPlain) {
    if (chk == kChkNone) SINKSLOT_TRY((launch_tiled_kind<kOutPlain, kChkNone>(a, h.g, st)));
    else if (chk == kChkMarg) SINKSLOT_TRY((launch_tiled_kind<kOutPlain, kChkMarg>(a, h.g, st)));
    else SINKSLOT_TRY((launch_tiled_kind<kOutPlain, kChkPot>(a, h.g, st)));
  } else if (out_mode == kOutBlend) {
    if (chk == kChkNone) SINKSLOT_TRY((launch_tiled_kind<kOutBlend, kChkNone>(a, h.g, st)));
    else if (chk == kChkMarg) SINKSLOT_TRY((launch_tiled_kind<kOutBlend, kChkMarg>(a, h.g, st)));
    else SINKSLOT_TRY((launch_tiled_kind<kOutBlend, kChkPot>(a, h.g, st)));
  } else {
    SINKSLOT_TRY((launch_tiled_kind<kOutNone, kChkMarg>(a, h.g, st)));
  }
  return exact_handed_back(h, out_mode, chk, st, ctas);
}

int tiled_max_pass(const TiledHalfStep& h, float* sigma_out, cudaStream_t st, unsigned int* ctas) {
  SINKSLOT_REQUIRE(sigma_out != nullptr && h.err, "tiled max pass: bad arguments");
  SINKSLOT_REQUIRE((reinterpret_cast<uintptr_t>(h.other) & 15u) == 0,
                   "tiled half step: the gathered potential must be 16-byte aligned");
  if (h.g.nseg <= 0) return kOk;
  TKArgs a = tk_args(h);
  a.out = sigma_out;
  a.peers.n = 0;
  a.fb_reset = nullptr;
  if (h.g.kind == kTilesTwoPass) SINKSLOT_TRY(launch_block_gather(h, st));
  SINKSLOT_TRY((launch_tiled_kind<kOutMax, kChkNone>(a, h.g, st)));
  if (ctas) *ctas += (unsigned)std::min(h.g.P, num_sms());
  return kOk;
}

template <int OUT, int CHK>
static int launch_tiled_kind(const TKArgs& a, const TileGeom& g, cudaStream_t st) {
  if (g.kind == kTilesTwoPass) return launch_panel_sum<OUT, CHK>(a, st);
  return launch_tiled<OUT, CHK>(a, g.smem_bytes, st);
}

}  // namespace sinkslot
