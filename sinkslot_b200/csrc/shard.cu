// shard.cu -- the Sinkhorn loop over a row/column partition of the support
// across the GPUs of one node, one process per GPU.
//
// Rank g owns rows [r0, r0 + nr) of the CSR side and columns [c0, c0 + nc) of
// the CSC side.  Every rank holds the full potentials phi (n) and psi (m) in a
// buffer that its peers can write (a CUDA IPC mapping).  A half-step computes
// the rank's own slice, and its epilogue stores every value both locally and
// into the same place of every peer's buffer (peer stores over NVLink, spread
// over the whole kernel, so the transfer overlaps the computation).  Each CTA
// then fences its stores at system scope and counts itself; a one-thread
// publish kernel acquires the count and writes the barrier epoch into a flag
// word of every peer (release, system scope).  Before the next half-step reads
// the other side's potential, a one-warp kernel waits until every peer's flag
// for that epoch has arrived (acquire, system scope).  Every wait is bounded:
// after about four seconds it records an error code and the loop's remaining
// kernels run without waiting; the host reports the error.  The exchange is
// plain peer stores and flag words; no library collective is involved.
//
// The symmetric variant reads the previous (phi, psi) in both half-steps and
// writes the next pair, so each rank keeps two buffers per potential (current,
// next), both peer-writable.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>

#include <cuda.h>

#include "../../include/sinkslot_b200.h"
#include "common.cuh"
#include "epilogue.cuh"
#include "sinkhorn.h"
#include "tiled.h"

namespace sinkslot {

constexpr int kMaxRanks = 8;
constexpr long long kFlagWaitCycles = 8000000000ll;  // ~4 s at 2 GHz

struct PeerFlags {
  uint32_t* p[kMaxRanks];
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int ld_acquire_gpu(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// After the half-step's kernels, whose CTAs stored their outputs into the peers'
// buffers and counted themselves in *done: acquires the count (all `expected`
// CTAs), makes the stores visible system-wide and raises flag `rank` of every
// peer to `epoch`.  One thread; bounded like every wait here.
__global__ void publish_kernel(unsigned int* done, unsigned int expected, PeerFlags flags,
                               int rank, int world, uint32_t epoch, int* err) {
  if (threadIdx.x != 0) return;
  const long long t0 = clock64();
  while (ld_acquire_gpu(done) < expected) {
    if (*(volatile int*)err != 0) break;
    if (clock64() - t0 > kFlagWaitCycles) {
      atomicCAS(err, 0, 6);
      break;
    }
  }
  *done = 0u;  // for the next half-step (its kernels are ordered after this one)
  __threadfence_system();
  for (int g = 0; g < world; ++g)
    if (g != rank) st_release_sys(flags.p[g] + rank, epoch);
}

// Waits until every peer has published `epoch` in this rank's flag words.
// Bounded: on timeout records code 5 in *err; once *err is set it waits no more.
__global__ void wait_epoch_kernel(const uint32_t* flags, int rank, int world, uint32_t epoch,
                                  int* err) {
  const int t = threadIdx.x;
  if (t >= world || t == rank) return;
  if (*(volatile int*)err != 0) return;
  const long long t0 = clock64();
  while (ld_acquire_sys(flags + t) < epoch) {
    if (clock64() - t0 > kFlagWaitCycles) {
      atomicCAS(err, 0, 5);
      return;
    }
    __nanosleep(200);
  }
}

struct ShardSpec {
  HalfStep row, col;  // local slices (nseg = nr / nc), indices into the full other side
  int64_t r0 = 0, c0 = 0;
  const void* row_tiles = nullptr;
  const void* col_tiles = nullptr;
  TileGeom row_geom, col_geom;
  const float* log_a = nullptr;  // full n
  const float* log_b = nullptr;  // full m
  int64_t n = 0, m = 0;
  int variant = 0;
  double alpha = 0.5;
  int rank = 0, world = 1;
  float* phi[kMaxRanks][2] = {};  // every rank's phi buffers (this rank's are local)
  float* psi[kMaxRanks][2] = {};
  uint32_t* flags[kMaxRanks] = {};
};

static int64_t pad4s(int64_t v) { return (v + 3) & ~int64_t(3); }

size_t shard_work_floats(int64_t nr, int64_t nc) {
  return (size_t)(2 * (pad4s(nr) + pad4s(nc)) + 64 + pad4s(nc));
}

static int read_words(const void* d, void* h, size_t bytes, cudaStream_t st) {
  SINKSLOT_CUDA_TRY(cudaMemcpyAsync(h, d, bytes, cudaMemcpyDeviceToHost, st));
  SINKSLOT_CUDA_TRY(cudaStreamSynchronize(st));
  return kOk;
}

// Runs iterations it0 .. it0 + n_iters - 1; the last one carries the check
// `check` (0 none, 1 potential, 2 marginal) whose local maxima come back in
// *c0, *c1.  *cur holds the index (0/1) of the buffers with the current
// potentials on entry and on return; *epoch the last barrier epoch used.
int shard_loop(const ShardSpec& sp, int64_t it0, int64_t n_iters, int check, int* cur,
               uint32_t* epoch, float* work, int64_t work_floats, double* c0, double* c1,
               cudaStream_t st) {
  const int64_t nr = sp.row.nseg, nc = sp.col.nseg;
  SINKSLOT_REQUIRE(sp.world >= 1 && sp.world <= kMaxRanks, "solve_shard: world must be 1..8");
  SINKSLOT_REQUIRE(sp.rank >= 0 && sp.rank < sp.world, "solve_shard: bad rank");
  SINKSLOT_REQUIRE(sp.variant == 0 || sp.variant == 1, "solve_shard: variant must be 0 or 1");
  SINKSLOT_REQUIRE(check >= 0 && check <= 2, "solve_shard: check must be 0, 1 or 2");
  SINKSLOT_REQUIRE(*cur == 0 || *cur == 1, "solve_shard: cur must be 0 or 1");
  SINKSLOT_REQUIRE(work_floats >= (int64_t)shard_work_floats(nr, nc),
                   "solve_shard: work buffer too small");
  SINKSLOT_REQUIRE(sp.r0 % 4 == 0 && sp.c0 % 4 == 0,
                   "solve_shard: slice starts must be multiples of 4");
  for (int g = 0; g < sp.world; ++g)
    SINKSLOT_REQUIRE(sp.phi[g][0] && sp.psi[g][0] && sp.flags[g] &&
                         (sp.variant == 0 || (sp.phi[g][1] && sp.psi[g][1])),
                     "solve_shard: missing peer buffer");
  // work: prev_phi (nr) | prev_psi (nc) | 64 words: [0,1] check maxima, [2,3]
  //       handed-back counts, [4] error, [8] publish counter | lists (nr, nc) |
  //       stabilisers of the first column half-step (nc)
  const int64_t nr4 = pad4s(nr), nc4 = pad4s(nc);
  float* prev_phi = work;
  float* prev_psi = work + nr4;
  uint32_t* acc = reinterpret_cast<uint32_t*>(work + nr4 + nc4);
  int* fb_count = reinterpret_cast<int*>(acc + 2);
  int* perr = reinterpret_cast<int*>(acc + 4);
  unsigned int* done = acc + 8;
  int* fb_rows = reinterpret_cast<int*>(work + nr4 + nc4 + 64);
  int* fb_cols = fb_rows + nr4;
  float* sigma0 = work + 2 * (nr4 + nc4) + 64;
  if (it0 == 0) {
    SINKSLOT_CUDA_TRY(cudaMemsetAsync(acc, 0, 64 * sizeof(uint32_t), st));
    SINKSLOT_CUDA_TRY(cudaMemsetAsync(prev_phi, 0, (nr4 + nc4) * sizeof(float), st));
  }
  if (check) SINKSLOT_CUDA_TRY(cudaMemsetAsync(acc, 0, 2 * sizeof(uint32_t), st));
  const float w_old = (float)(1.0 - sp.alpha), w_new = (float)sp.alpha;
  const int me = sp.rank;
  int c = *cur;
  uint32_t ep = *epoch;

  // after a half-step that stored into the peers (its kernels launched `ctas`
  // CTAs): publish the next epoch, then wait for every peer's
  auto publish = [&](unsigned int ctas) -> int {
    ++ep;
    if (sp.world > 1) {
      PeerFlags fl{};
      for (int g = 0; g < sp.world; ++g) fl.p[g] = sp.flags[g];
      publish_kernel<<<1, 32, 0, st>>>(done, ctas, fl, me, sp.world, ep, perr);
      SINKSLOT_CHECK_LAUNCH();
      wait_epoch_kernel<<<1, 32, 0, st>>>(sp.flags[me], me, sp.world, ep, perr);
      SINKSLOT_CHECK_LAUNCH();
    }
    return kOk;
  };

  auto side_step = [&](bool row, int64_t it, int out_mode, int chk) -> int {
    const HalfStep& side = row ? sp.row : sp.col;
    const int64_t off = row ? sp.r0 : sp.c0;
    const int nb = sp.variant == 0 ? c : 1 - c;  // buffer written
    float* self_cur = (row ? sp.phi[me][c] : sp.psi[me][c]) + off;
    float* out = (row ? sp.phi[me][nb] : sp.psi[me][nb]) + off;
    // alternating writes in place, so the column half-step reads the phi just
    // written; symmetric reads the previous pair in both half-steps
    const float* other = row ? sp.psi[me][c] : sp.phi[me][c];
    const float* base = (row ? sp.log_a : sp.log_b) + off;
    float* prev = row ? prev_phi : prev_psi;
    uint32_t* acc_side = acc + (row ? 0 : 1);
    const void* tiles = row ? sp.row_tiles : sp.col_tiles;
    // the peers' copies of `out` (same offset in their buffer `nb`)
    PeerOut po{};
    po.n = 0;
    if (out_mode != kOutNone)
      for (int g = 0; g < sp.world; ++g)
        if (g != me) po.p[po.n++] = (row ? sp.phi[g][nb] : sp.psi[g][nb]) + off;
    unsigned int ctas = 0;
    // The first iteration (as in the single-GPU loop): a half-step that gathers
    // the zero start potential runs the exact kernel without the gather; the
    // alternating first column half-step with a tiled layout takes its
    // stabilisers from a tiled max pass.
    const bool first = it == 0 && out_mode != kOutNone;
    const bool zero_other = first && (row || sp.variant == 1);
    if (side.nseg > 0) {
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
        t.peers = po;
        t.done = done;
        if (it == 0) {
          t.sigma = sigma0;
          SINKSLOT_TRY(tiled_max_pass(t, sigma0, st));
        }
        SINKSLOT_TRY(tiled_half_step(t, out_mode, chk, st, &ctas));
      } else {
        HalfStep h = side;
        h.other = zero_other ? nullptr : other;
        h.base = base;
        h.prev = prev;
        h.acc = acc_side;
        h.w_old = w_old;
        h.w_new = w_new;
        h.self_old = self_cur;
        h.out = out;
        h.peers = po;
        h.done = done;
        SINKSLOT_TRY(half_step(h, out_mode, chk, st, &ctas));
      }
    }
    if (out_mode == kOutNone) return kOk;
    return publish(ctas);
  };

  const int step_out = sp.variant == 0 ? kOutPlain : kOutBlend;
  for (int64_t k = 0; k < n_iters; ++k) {
    const int64_t it = it0 + k;
    const bool last = k + 1 == n_iters;
    const int chk = !last || check == 0 ? kChkNone : (check == 1 ? kChkPot : kChkMarg);
    if (sp.variant == 0) {
      SINKSLOT_TRY(side_step(true, it, step_out, chk));
      SINKSLOT_TRY(side_step(false, it, step_out, chk));
    } else {
      SINKSLOT_TRY(side_step(true, it, step_out, chk == kChkPot ? kChkPot : kChkNone));
      SINKSLOT_TRY(side_step(false, it, step_out, chk == kChkPot ? kChkPot : kChkNone));
      c = 1 - c;
      if (chk == kChkMarg) {
        SINKSLOT_TRY(side_step(true, it, kOutNone, kChkMarg));
        SINKSLOT_TRY(side_step(false, it, kOutNone, kChkMarg));
      }
    }
  }
  *cur = c;
  *epoch = ep;
  uint32_t h[8];
  SINKSLOT_TRY(read_words(acc, h, sizeof(h), st));
  if (h[4] != 0) {
    set_error(h[4] == 5   ? "solve_shard: a peer did not publish its potentials in time (code 5)"
              : h[4] == 4 ? "solve_shard: a tiled layout was built for another kind or geometry "
                            "(code 4); build and solve under the same tiles kind"
                          : "solve_shard: a shared-memory pipeline wait timed out (code " +
                                std::to_string(h[4]) + ")");
    return kCudaError;
  }
  float f0, f1;
  memcpy(&f0, &h[0], 4);
  memcpy(&f1, &h[1], 4);
  *c0 = f0;
  *c1 = f1;
  return kOk;
}

// base address of the allocation holding p (driver entry point, no link-time
// dependency on libcuda)
static int alloc_base(const void* p, uintptr_t* base) {
  using Fn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static Fn fn = nullptr;
  if (fn == nullptr) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    SINKSLOT_CUDA_TRY(cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q));
    SINKSLOT_REQUIRE(f != nullptr && q == cudaDriverEntryPointSuccess,
                     "ipc: cuMemGetAddressRange is not available");
    fn = reinterpret_cast<Fn>(f);
  }
  CUdeviceptr b = 0;
  size_t sz = 0;
  if (fn(&b, &sz, (CUdeviceptr)(uintptr_t)p) != CUDA_SUCCESS) {
    set_error("ipc: pointer is not in a device allocation");
    return kInvalidArgument;
  }
  *base = (uintptr_t)b;
  return kOk;
}

}  // namespace sinkslot

using namespace sinkslot;

extern "C" int sinkslot_ipc_export(const void* ptr, void* handle_host, int64_t* offset_host) {
  set_error("");
  SINKSLOT_REQUIRE(ptr && handle_host && offset_host, "ipc_export: null argument");
  uintptr_t base = 0;
  SINKSLOT_TRY(alloc_base(ptr, &base));
  cudaIpcMemHandle_t h;
  SINKSLOT_CUDA_TRY(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
  static_assert(sizeof(h) == SINKSLOT_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle_host, &h, sizeof(h));
  *offset_host = (int64_t)((uintptr_t)ptr - base);
  return kOk;
}

extern "C" int sinkslot_ipc_import(const void* handle_host, int64_t offset, void** ptr_host) {
  set_error("");
  SINKSLOT_REQUIRE(handle_host && ptr_host && offset >= 0, "ipc_import: bad argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle_host, sizeof(h));
  void* base = nullptr;
  SINKSLOT_CUDA_TRY(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
  *ptr_host = static_cast<char*>(base) + offset;
  return kOk;
}

extern "C" int sinkslot_ipc_close(void* ptr, int64_t offset) {
  set_error("");
  SINKSLOT_REQUIRE(ptr && offset >= 0, "ipc_close: bad argument");
  SINKSLOT_CUDA_TRY(cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset));
  return kOk;
}

extern "C" int sinkslot_shard_work_floats(int64_t nr, int64_t nc, int64_t* floats_host) {
  set_error("");
  SINKSLOT_REQUIRE(floats_host && nr >= 0 && nc >= 0, "shard_work_floats: bad args");
  *floats_host = (int64_t)shard_work_floats(nr, nc);
  return kOk;
}

extern "C" int sinkslot_solve_shard(
    const int32_t* r_ptr, const void* r_idx, int r_idx_bytes, const float* r_lam, int64_t r_nnz,
    int64_t r0, int64_t nr, const void* r_tiles, int64_t r_tiles_bytes, const int32_t* c_ptr,
    const void* c_idx, int c_idx_bytes, const float* c_lam, int64_t c_nnz, int64_t c0,
    int64_t nc, const void* c_tiles, int64_t c_tiles_bytes, const float* log_a,
    const float* log_b, int64_t n, int64_t m, int variant, double alpha, int rank, int world,
    float* const* phi_bufs_host, float* const* psi_bufs_host, uint32_t* const* flags_host,
    int64_t it0, int64_t n_iters, int check, int* cur_host, uint32_t* epoch_host, float* work,
    int64_t work_floats, double* check0_host, double* check1_host, void* stream) {
  set_error("");
  SINKSLOT_REQUIRE(r_ptr && c_ptr && log_a && log_b && phi_bufs_host && psi_bufs_host &&
                       flags_host && cur_host && epoch_host && work && check0_host && check1_host,
                   "solve_shard: null argument");
  SINKSLOT_REQUIRE(world >= 1 && world <= kMaxRanks && rank >= 0 && rank < world,
                   "solve_shard: bad rank/world");
  SINKSLOT_REQUIRE(r0 >= 0 && nr >= 0 && r0 + nr <= n && c0 >= 0 && nc >= 0 && c0 + nc <= m,
                   "solve_shard: slice out of range");
  SINKSLOT_REQUIRE(r_nnz == 0 || (r_idx && r_lam), "solve_shard: null row entries");
  SINKSLOT_REQUIRE(c_nnz == 0 || (c_idx && c_lam), "solve_shard: null column entries");
  ShardSpec sp;
  sp.row.ptr = r_ptr;
  sp.row.idx = r_idx;
  sp.row.idx_bytes = r_idx_bytes;
  sp.row.lam = r_lam;
  sp.row.nseg = nr;
  sp.row.nnz = r_nnz;
  sp.col.ptr = c_ptr;
  sp.col.idx = c_idx;
  sp.col.idx_bytes = c_idx_bytes;
  sp.col.lam = c_lam;
  sp.col.nseg = nc;
  sp.col.nnz = c_nnz;
  sp.r0 = r0;
  sp.c0 = c0;
  // either side may run tiled or exact (a null layout)
  if (r_tiles) {
    SINKSLOT_REQUIRE(nr > 0, "solve_shard: a tiled layout needs a non-empty row slice");
    sp.row_geom = tile_geom(nr, m, r_nnz, num_sms());
    SINKSLOT_REQUIRE(r_tiles_bytes >= (int64_t)sp.row_geom.layout_bytes,
                     "solve_shard: tiled layout buffer too small");
    sp.row_tiles = r_tiles;
  }
  if (c_tiles) {
    SINKSLOT_REQUIRE(nc > 0, "solve_shard: a tiled layout needs a non-empty column slice");
    sp.col_geom = tile_geom(nc, n, c_nnz, num_sms());
    SINKSLOT_REQUIRE(c_tiles_bytes >= (int64_t)sp.col_geom.layout_bytes,
                     "solve_shard: tiled layout buffer too small");
    sp.col_tiles = c_tiles;
  }
  sp.log_a = log_a;
  sp.log_b = log_b;
  sp.n = n;
  sp.m = m;
  sp.variant = variant;
  sp.alpha = alpha;
  sp.rank = rank;
  sp.world = world;
  for (int g = 0; g < world; ++g) {
    sp.phi[g][0] = phi_bufs_host[2 * g];
    sp.phi[g][1] = phi_bufs_host[2 * g + 1];
    sp.psi[g][0] = psi_bufs_host[2 * g];
    sp.psi[g][1] = psi_bufs_host[2 * g + 1];
    sp.flags[g] = flags_host[g];
  }
  return shard_loop(sp, it0, n_iters, check, cur_host, epoch_host, work, work_floats, check0_host,
                    check1_host, static_cast<cudaStream_t>(stream));
}
