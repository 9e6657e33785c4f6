// tiled.h -- column-blocked ("tiled") layout of a CSR side and the half-step
// that stages the gathered potential in shared memory.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "epilogue.cuh"

namespace sinkslot {

// How a tiled layout is used by the half-step:
//   kTilesStaged   one pass per half-step: each panel's CTA stages every block
//                  of the gathered potential in shared memory (P * m_o * 4
//                  bytes copied per half-step);
//   kTilesTwoPass  two passes: one CTA per block stages it once and writes each
//                  entry's exponent lam + potential in layout order, then one
//                  CTA per panel sums its entries without a gather -- for
//                  gathered axes too long to stage once per panel.
// kTilesAuto picks by the cost of staging (tile_geom).
enum TilesKind { kTilesAuto = 0, kTilesStaged = 1, kTilesTwoPass = 2 };

// Process-wide kind used when a layout's geometry is computed (auto unless set):
// a layout must be built and used under the same setting (the kernels check
// the kind and geometry recorded in the layout's header and fail otherwise).
void set_tiles_kind(int kind);
int tiles_kind();

// Geometry of a tiled layout: P panels of R rows; the gathered axis (length
// m_o) cut into B blocks of W = 2^logW entries.  Tile (p, b) holds the entries
// of panel p whose column falls in block b, padded to a multiple of 32 entries
// (warp slabs) and dealt so that a slab's rows lie in different shared-memory
// banks.
struct TileGeom {
  int64_t nseg = 0, m_o = 0, nnz = 0;
  int P = 0, R = 0, B = 0, logW = 0;
  int64_t cap = 0;          // entries in the layout (nnz plus tile padding)
  size_t smem_bytes = 0;    // dynamic shared memory of the tiled kernel
  size_t layout_bytes = 0;  // header + tile_start + meta + lam
  size_t build_bytes = 0;   // scratch of the builder
  bool direct = false;      // built by the per-panel counting kernels (else by a sort)
  int S = 1;                // sub-panels (CTAs) per panel of the direct builder
  int kind = kTilesStaged;  // kTilesStaged or kTilesTwoPass (never auto)
};

// kind: kTilesAuto / kTilesStaged / kTilesTwoPass, or -1 for tiles_kind()
TileGeom tile_geom(int64_t nseg, int64_t m_o, int64_t nnz, int sms, int kind = -1);

// Builds the layout (into `layout`, layout_bytes) from a CSR side.
int build_tiles(const int32_t* ptr, const void* idx, int idx_bytes, const float* lam,
                const TileGeom& g, void* layout, void* ws, size_t ws_bytes, cudaStream_t st);

struct TiledHalfStep {
  TileGeom g;
  const void* layout = nullptr;
  // exact CSR for rows the tiled pass hands back (see tiled.cu)
  const int32_t* ptr = nullptr;
  const void* idx = nullptr;
  int idx_bytes = 4;
  const float* lam = nullptr;
  // per launch
  const float* other = nullptr;
  const float* base = nullptr;
  const float* self_old = nullptr;
  // optional per-segment stabilisers; without them a segment's stabiliser is
  // base - self_old, the log-sum-exp of its previous half-step
  const float* sigma = nullptr;
  float* out = nullptr;
  float w_old = 0.5f, w_new = 0.5f;
  float* prev = nullptr;
  uint32_t* acc = nullptr;
  int* fb_count = nullptr;        // rows handed to the exact pass (reset by the caller)
  int* fb_list = nullptr;         // nseg entries
  int* fb_count_reset = nullptr;  // optional counter this launch zeroes (the other side's)
  int* err = nullptr;             // set nonzero when a pipeline wait times out
  PeerOut peers = {{}, 0};        // optional peer copies of `out`
  unsigned int* done = nullptr;   // CTA counter for the peer publish step
};

// tiled pass + exact pass over the rows it handed back; *ctas (optional) is
// increased by the number of CTAs launched
int tiled_half_step(const TiledHalfStep& h, int out_mode, int chk, cudaStream_t st,
                    unsigned int* ctas = nullptr);

// One tiled pass that writes, for every segment s, max_k (lam_k + other[idx_k])
// into sigma_out[s] (-inf for an empty segment; NaN when a term is NaN).  Used
// as the stabilisers of a tiled half-step that has no previous log-sum-exp (the
// first column half-step of a solve): every term of that pass is then at most
// 1 and every sum at least 1, so no segment is handed back for its range.
int tiled_max_pass(const TiledHalfStep& h, float* sigma_out, cudaStream_t st,
                   unsigned int* ctas = nullptr);

}  // namespace sinkslot
