// common.cuh -- shared helpers for the sm_100a SinkSLOT kernels.
#pragma once

#include <cuda_runtime.h>
#include <utility>
#include <stdint.h>

#include <string>

namespace sinkslot {

// Status codes returned by every extern "C" entry point (0 = success).
enum Status : int {
  kOk = 0,
  kInvalidArgument = 1,
  kCudaError = 2,
  kWorkspaceTooSmall = 3,
  kUnsupported = 4,
};

// Per-thread last error message (read through sinkslot_last_error()).
void set_error(const std::string& msg);
const char* last_error();

#define SINKSLOT_CUDA_TRY(expr)                                                 \
  do {                                                                          \
    cudaError_t err__ = (expr);                                                 \
    if (err__ != cudaSuccess) {                                                 \
      ::sinkslot::set_error(std::string(#expr) + ": " + cudaGetErrorString(err__)); \
      return ::sinkslot::kCudaError;                                            \
    }                                                                           \
  } while (0)

#define SINKSLOT_CHECK_LAUNCH()                                                 \
  do {                                                                          \
    cudaError_t err__ = cudaGetLastError();                                     \
    if (err__ != cudaSuccess) {                                                 \
      ::sinkslot::set_error(std::string("kernel launch: ") + cudaGetErrorString(err__)); \
      return ::sinkslot::kCudaError;                                            \
    }                                                                           \
  } while (0)

#define SINKSLOT_REQUIRE(cond, msg)                                             \
  do {                                                                          \
    if (!(cond)) {                                                              \
      ::sinkslot::set_error(msg);                                               \
      return ::sinkslot::kInvalidArgument;                                      \
    }                                                                           \
  } while (0)

#define SINKSLOT_TRY(expr)                                                      \
  do {                                                                          \
    int st__ = (expr);                                                          \
    if (st__ != ::sinkslot::kOk) return st__;                                   \
  } while (0)

constexpr int kNumSMs = 148;  // B200: 2 dies x 74 SMs

inline int num_sms() {
  static int cached = -1;
  if (cached < 0) {
    int dev = 0, v = 0;
    if (cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0)
      cached = v;
    else
      cached = kNumSMs;
  }
  return cached;
}

__host__ __device__ inline int64_t ceil_div64(int64_t a, int64_t b) { return (a + b - 1) / b; }

__host__ __device__ constexpr inline size_t align_up(size_t x, size_t a = 256) {
  return (x + a - 1) / a * a;
}

// Bump allocator over a caller-provided workspace.  Every carve is 256-byte
// aligned; `ok` turns false when the workspace is too small.
struct Carver {
  char* base;
  size_t cap;
  size_t used = 0;
  bool ok = true;
  Carver(void* p, size_t c) : base(static_cast<char*>(p)), cap(c) {}
  template <typename T>
  T* take(size_t count) {
    size_t bytes = align_up(count > 0 ? count * sizeof(T) : 1);
    if (used + bytes > cap) {
      ok = false;
      used += bytes;
      return nullptr;
    }
    T* r = reinterpret_cast<T*>(base + used);
    used += bytes;
    return r;
  }
};

// Order-preserving map of a float to uint32 (radix order), with -0.0 mapped to
// +0.0 first so the two compare equal (CUB's DeviceRadixSort does the same).
__device__ __forceinline__ uint32_t float_to_radix(float f) {
  uint32_t u = __float_as_uint(f);
  if (u == 0x80000000u) u = 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Non-negative float (or +NaN) as an order-preserving uint32 for atomicMax.
__device__ __forceinline__ uint32_t nonneg_float_bits(float f) { return __float_as_uint(fabsf(f)); }

template <typename T>
__device__ __forceinline__ T ld_stream(const T* p) {
  return __ldcs(p);
}

// Programmatic dependent launch.  The solve loop's half-step kernels are
// launched so that each may be scheduled before the one ahead of it has
// finished (launch_chained below).  Every such kernel waits, before it reads or
// writes anything, until the kernel before it has completed and its writes are
// visible (chain_enter); as each waits for the one before, the completion of any
// of them implies the completion of all earlier ones.  A block lets the next
// kernel start launching once its main work is done (chain_release): released
// at entry instead, the next grid's launch competed with the running one
// (measured 4% slower per half-step; released late, 1.8% faster than no chaining).
#ifndef SINKSLOT_PDL
#define SINKSLOT_PDL 1
#endif
__device__ __forceinline__ void chain_enter() {
#if SINKSLOT_PDL
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
#endif
}
__device__ __forceinline__ void chain_release() {
#if SINKSLOT_PDL
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
#endif
}

template <typename... Params, typename... Args>
static inline cudaError_t launch_chained(void (*kernel)(Params...), dim3 grid, dim3 block,
                                         size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = SINKSLOT_PDL;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace sinkslot
