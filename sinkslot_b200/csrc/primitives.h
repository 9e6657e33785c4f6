// primitives.h -- device-wide scan and stable LSD radix sort used by the support
// builder and the CSR/CSC transposition.  All launches go to the caller's stream;
// temporaries come from caller-provided memory.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace sinkslot {

// Exclusive scan of n int64 values in place.  `tmp` needs scan_tmp_elems(n)
// int64 elements.  If `total` is non-null, the sum of all inputs is written to
// total[0] (device memory).
size_t scan_tmp_elems(int64_t n);
int scan_exclusive_i64(int64_t* data, int64_t n, int64_t* tmp, int64_t* total,
                       cudaStream_t stream);

// Stable LSD radix sort of (key, value) pairs, ascending by key bits
// [0, key_bits), applied independently to `nseg` back-to-back segments of
// `seglen` elements.  Key/value types: (uint32_t, uint32_t), (uint64_t,
// uint32_t) or (uint32_t, uint64_t); with `identity_vals` the first pass ignores
// the contents of `vals` and uses each element's index within its segment (all
// four buffers must still be given).
// Ping-pongs between (keys, vals) and (keys_alt, vals_alt); on return
// `*result_in_alt` tells which pair holds the sorted data.
// Workspace: radix_hist_elems(nseg, seglen) int64 for the digit histogram plus
// scan_tmp_elems of that count for the scan.
int64_t radix_hist_elems(int64_t nseg, int64_t seglen);
template <typename K, typename V = uint32_t>
int radix_sort_pairs(K* keys, V* vals, K* keys_alt, V* vals_alt, bool identity_vals,
                     int64_t nseg, int64_t seglen, int key_bits, int64_t* hist, int64_t* scan_tmp,
                     bool* result_in_alt, cudaStream_t stream);

// Number of bits needed to hold values in [0, v).
inline int bits_for(uint64_t v) {
  int b = 0;
  while (b < 64 && (v > (uint64_t(1) << b))) ++b;
  return b;
}

}  // namespace sinkslot
