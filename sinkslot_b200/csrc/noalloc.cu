// noalloc.cu -- sinkslot_solve_csr_static: the Sinkhorn solve loop with its
// scratch in a fixed device array of the library instead of a caller buffer.
//
// Some callers have no way to hand in device scratch: a thin FFI binding
// (ctypes, cgo, JNI) that holds only the tensors its host framework gave it and
// owns no device allocator to size and free a work buffer with, or code that
// runs under a memory pool it may not grow.  For small problems this entry
// point needs no scratch from them: the loop runs in `g_solve_scratch`, a
// file-scope __device__ array of SINKSLOT_STATIC_SOLVE_FLOATS floats (4 MiB)
// that every GPU which loads the library holds until the process exits.
//
// Rules of use:
//   - The first call on a device looks up the array's device address
//     (cudaGetSymbolAddress, with that device current) and keeps it; make that
//     first call before any stream capture on the device.  The kept address
//     belongs to the device's primary context: after cudaDeviceReset (or any
//     teardown of that context) it is stale, so a host that resets a device
//     must not call this entry point on it again in the same process.
//   - There is one array per device: calls that overlap on the same device
//     (two host threads, or two streams whose work interleaves) share it and
//     race.  Serialise them.
//   - Problems whose scratch (sinkslot_solve_work_floats: 3 * (pad4(n) +
//     pad4(m)) + 64 floats, pad4 rounding up to a multiple of 4) exceeds the
//     array are rejected with status 1; use sinkslot_solve_csr with a caller
//     buffer.
//   - Each call zeroes the part of the array it uses, on its stream, before
//     the solve reads it.
#include <mutex>
#include <string>

#include "../../include/sinkslot_b200.h"
#include "common.cuh"
#include "sinkhorn.h"

namespace {

static __device__ __align__(256) float g_solve_scratch[SINKSLOT_STATIC_SOLVE_FLOATS];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
float* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_solve_scratch on the current device, looked up once.
int scratch_for_current_device(float** out) {
  int dev = -1;
  SINKSLOT_CUDA_TRY(cudaGetDevice(&dev));
  SINKSLOT_REQUIRE(dev >= 0 && dev < kMaxDevices, "solve_csr_static: device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    SINKSLOT_CUDA_TRY(cudaGetSymbolAddress(&p, g_solve_scratch));
    SINKSLOT_REQUIRE(p != nullptr, "solve_csr_static: scratch symbol has no device address");
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return sinkslot::kOk;
}

}  // namespace

extern "C" int sinkslot_solve_csr_static(
    const int32_t* r_ptr, const void* r_idx, int r_idx_bytes, const float* r_lam,
    const int32_t* c_ptr, const void* c_idx, int c_idx_bytes, const float* c_lam, int64_t nnz,
    const float* log_a, const float* log_b, int64_t n, int64_t m, int variant, int stop_mode,
    int64_t n_iters, int64_t max_iter, int64_t check_every, double tol, double eps, double alpha,
    const void* r_tiles, int64_t r_tiles_bytes, const void* c_tiles, int64_t c_tiles_bytes,
    float* phi, float* psi, int64_t* iters_host, int* converged_host, double* final_viol_host,
    void* stream) {
  sinkslot::set_error("");
  SINKSLOT_REQUIRE(n >= 1 && m >= 1, "solve_csr_static: n and m must be >= 1");
  const int64_t need = (int64_t)sinkslot::solve_work_floats(n, m);
  if (need > (int64_t)SINKSLOT_STATIC_SOLVE_FLOATS) {
    sinkslot::set_error("solve_csr_static: an (n, m) = (" + std::to_string(n) + ", " +
                        std::to_string(m) + ") solve needs " + std::to_string(need) +
                        " scratch floats; the static scratch holds at most " +
                        std::to_string((int64_t)SINKSLOT_STATIC_SOLVE_FLOATS) +
                        " (use sinkslot_solve_csr with a work buffer)");
    return sinkslot::kInvalidArgument;
  }
  float* work = nullptr;
  SINKSLOT_TRY(scratch_for_current_device(&work));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  SINKSLOT_CUDA_TRY(cudaMemsetAsync(work, 0, (size_t)need * sizeof(float), st));
  return sinkslot_solve_csr(r_ptr, r_idx, r_idx_bytes, r_lam, c_ptr, c_idx, c_idx_bytes, c_lam,
                            nnz, log_a, log_b, n, m, variant, stop_mode, n_iters, max_iter,
                            check_every, tol, eps, alpha, r_tiles, r_tiles_bytes, c_tiles,
                            c_tiles_bytes, phi, psi, work, need, iters_host, converged_host,
                            final_viol_host, stream);
}
