// sinkhorn.h -- half-step launcher and solve loops.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "epilogue.cuh"
#include "tiled.h"

namespace sinkslot {

// One CSR (or CSC) side plus the per-launch operands of a half-step.
struct HalfStep {
  const int32_t* ptr = nullptr;  // nseg + 1 segment offsets
  const void* idx = nullptr;     // gathered-axis index per entry (int16 or int32)
  int idx_bytes = 4;
  const float* lam = nullptr;    // log S - C / eps per entry
  int64_t nseg = 0;
  int64_t nnz = 0;
  int group = 0;                 // lanes per segment (0: from the mean length)
  // per launch
  const float* other = nullptr;  // gathered potential
  const float* selfpot = nullptr;  // optional per-segment potential added to every term
  const float* base = nullptr;   // log marginal
  const float* self_old = nullptr;
  float* out = nullptr;
  float w_old = 0.5f, w_new = 0.5f;
  float* prev = nullptr;
  uint32_t* acc = nullptr;
  const int* list = nullptr;        // optional: compute only these segments
  const int* list_count = nullptr;  // device count of `list`
  PeerOut peers = {{}, 0};          // optional peer copies of `out`
  unsigned int* done = nullptr;     // CTA counter for the peer publish step
};

// out_mode: 0 store, 1 alpha-blend store, 2 no store; chk: 0 none, 1 marginal, 2 potential.
// *ctas (optional) is increased by the number of CTAs launched.
int half_step(const HalfStep& h, int out_mode, int chk, cudaStream_t st,
              unsigned int* ctas = nullptr);

struct SolveSpec {
  HalfStep row, col;
  // optional column-blocked layouts of both sides (tiled.h); null: exact kernel
  const void* row_tiles = nullptr;
  const void* col_tiles = nullptr;
  TileGeom row_geom, col_geom;
  const float* log_a = nullptr;
  const float* log_b = nullptr;
  int variant = 0;  // 0 alternating, 1 symmetric
  int mode = 0;     // 0 fixed, 1 potential, 2 marginal
  int64_t n_iters = 0, max_iter = 0, check_every = 1;
  double tol = 0, eps = 0, alpha = 0.5;
};

size_t solve_work_floats(int64_t n, int64_t m);
int solve_loop(const SolveSpec& sp, float* phi, float* psi, float* work, int64_t work_floats,
               int64_t* iters_run, int* converged, double* final_viol, cudaStream_t st);

}  // namespace sinkslot
