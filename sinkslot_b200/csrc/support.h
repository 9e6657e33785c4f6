// support.h -- host launchers for support construction and COO -> CSR.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace sinkslot {

int project(const float* X, int64_t n, int d, const float* theta, int C, float* out,
            cudaStream_t stream);
uint32_t torch_inner_scan_log_tx(uint32_t num_rows, uint32_t row_size);

size_t ot1d_workspace_bytes(int64_t n, int64_t m, int C);
int ot1d_batched(const float* PXt, const float* PYt, const float* a, const float* b, int64_t n,
                 int64_t m, int C, int scan_rows, void* ws, size_t ws_bytes, int64_t* R,
                 int64_t* Cc, float* M, uint32_t* ix, uint32_t* iy, float* ca, float* cb,
                 int64_t* count_out, cudaStream_t stream);

size_t support_workspace_bytes(int64_t n, int64_t m, int d, int L, int chunk);
int build_support(const float* X, const float* Y, const float* a, const float* b, int64_t n,
                  int64_t m, int d, const float* theta, const float* PX, const float* PY, int L,
                  int chunk, void* ws, size_t ws_bytes, int64_t* nnz_out, cudaStream_t stream);
int support_export(const void* ws, size_t ws_bytes, int64_t n, int64_t m, int d, int L, int chunk,
                   int64_t nnz, int64_t* rows, int64_t* cols, float* S, cudaStream_t stream);

size_t csr_workspace_bytes(int64_t nnz, int64_t nseg);
int coo_to_csr(const int64_t* seg, const int64_t* idx, const float* vals, int64_t nnz, int64_t nseg,
               int idx_bytes, void* ws, size_t ws_bytes, int32_t* out_ptr, void* out_idx,
               float* out_vals, int64_t* out_perm, int* was_sorted, cudaStream_t stream);

// A support built across the GPUs of a node (partition.cu): stable partition
// of COO entries by the part owning their segment (bounds[0..parts], at most
// kMaxOwnerParts parts), and the coalesce of raw entries received in slice order.
constexpr int kMaxOwnerParts = 64;
size_t partition_workspace_bytes(int64_t nnz);
int partition_coo(const int64_t* seg, const int64_t* other, const float* vals, int64_t nnz,
                  const int64_t* bounds_host, int parts, void* ws, size_t ws_bytes,
                  int64_t* seg_out, int64_t* other_out, float* vals_out, int64_t* counts_host,
                  cudaStream_t st);
size_t coalesce_workspace_bytes(int64_t nraw);
int coalesce_coo(const int64_t* R, const int64_t* C, const float* mass, int64_t nraw, int64_t n,
                 int64_t m, int L, void* ws, size_t ws_bytes, int64_t* rows, int64_t* cols,
                 float* S, int64_t* nnz_host, cudaStream_t st);

}  // namespace sinkslot
