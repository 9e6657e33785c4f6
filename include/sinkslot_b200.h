/*
 * sinkslot_b200.h -- C ABI of the sm_100a SinkSLOT sparse-Sinkhorn backend
 * (libsinkslot_b200.so).
 *
 * Conventions
 *   - Every pointer argument is DEVICE memory unless its name ends in `_host`.
 *   - `stream` is a cudaStream_t passed as void*; all work is enqueued on it.
 *     Calls that return a count to the host (nnz, iterations, ...) synchronise
 *     that stream, exactly where the reference reads a value back with
 *     .item()/int()/bool().
 *   - No call allocates device memory.  Scratch comes from a caller-provided
 *     workspace whose size the matching *_workspace_bytes call reports
 *     (sinkslot_solve_csr_static alone uses the library's static array).
 *   - Return value: 0 on success, otherwise a status code (1 invalid argument,
 *     2 CUDA error, 3 workspace too small, 4 unsupported); the message is in
 *     sinkslot_last_error() (per calling thread).
 *   - Reference paths are relative to cai4cai/SinkSLOT's torch-ext/ tree.
 */
#ifndef SINKSLOT_B200_H_
#define SINKSLOT_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Last error message of the calling thread ("" if none). */
const char* sinkslot_last_error(void);

/* ABI version (major * 100 + minor). */
int sinkslot_abi_version(void);

/* ---------------------------------------------------------------------------
 * Support construction
 * ------------------------------------------------------------------------- */

/* Projections out[c, i] = <X[i, :], theta[c, :]> as the sequential fp32 FMA
 * chain over d, slice-major (L, n).  Replaces `X @ th.T` in
 * sinkslot/solver.py:221 (transposed to the (C, len) layout of
 * `_ot_1d_coo_batched_cuda`, solver.py:117). */
int sinkslot_project(const float* X, int64_t n, int d, const float* theta, int L, float* out,
                     void* stream);

int sinkslot_ot1d_workspace_bytes(int64_t n, int64_t m, int C, int64_t* bytes_host);

/* One call of the batched 1-D north-west-corner builder over C slices:
 * replaces `_ot_1d_coo_batched_cuda(PX, PY, a, b)`, sinkslot/solver.py:107-150.
 * PXt (C, n) and PYt (C, m) are slice-major projections.  Writes the kept
 * (R, Cc, mass) triples in the reference's emission order (slice-major, merged
 * position ascending); capacity C * (n + m).  Optional (nullable) outputs: the
 * per-slice argsort permutations ix (C, n) / iy (C, m) as uint32 and the
 * cumsums ca (C, n) / cb (C, m).  *count_host receives the number of triples.
 * scan_rows: the cumsums follow the association torch's CUDA scan uses for a
 * (scan_rows, len) tensor -- 0 means C, the reference's own call; a caller
 * building some of the slices of a larger batch (one rank of a partitioned
 * build) passes that batch's slice count, so the bits equal the batch's. */
int sinkslot_ot1d_batched(const float* PXt, const float* PYt, const float* a, const float* b,
                          int64_t n, int64_t m, int C, int scan_rows, void* workspace,
                          int64_t workspace_bytes, int64_t* R, int64_t* Cc, float* mass,
                          uint32_t* ix, uint32_t* iy, float* ca, float* cb, int64_t* count_host,
                          void* stream);

int sinkslot_support_workspace_bytes(int64_t n, int64_t m, int d, int L, int chunk,
                                     int64_t* bytes_host);

/* Sliced-lifted support: replaces `sot_plan_coo(X, Y, a, b, L, seed, chunk,
 * ot1d=_ot_1d_coo_batched_cuda)`, sinkslot/solver.py:153-232.  The
 * projections come either from PX (n, L) / PY (m, L), row-major -- the
 * reference's `X @ th.T` per chunk (solver.py:221), computed by the caller's
 * GEMM so their bits are the reference's -- or, when PX and PY are NULL, from
 * theta (L, d) fp32 (get_random_projections(d, L, seed) cast to fp32,
 * solver.py:193) as the sequential FMA chain over d.  chunk <= 0 means all L
 * slices in one batch.  The coalesced support stays in the workspace;
 * *nnz_host receives its size.  Call sinkslot_support_export with the same
 * sizes to read it out. */
int sinkslot_build_support(const float* X, const float* Y, const float* a, const float* b,
                           int64_t n, int64_t m, int d, const float* theta, const float* PX,
                           const float* PY, int L, int chunk, void* workspace,
                           int64_t workspace_bytes, int64_t* nnz_host, void* stream);

/* rows, cols (int64) and S (fp32) of the support built by
 * sinkslot_build_support, sorted by rows * m + cols: the return value of
 * sot_plan_coo (solver.py:232). */
int sinkslot_support_export(const void* workspace, int64_t workspace_bytes, int64_t n, int64_t m,
                            int d, int L, int chunk, int64_t nnz, int64_t* rows, int64_t* cols,
                            float* S, void* stream);

/* Support built across the GPUs of a node (one process each, each rank
 * building a contiguous range of the slices with sinkslot_ot1d_batched).  No
 * counterpart in the reference, whose support is built on one device
 * (sot_plan_coo, sinkslot/solver.py:153-232); together they give each rank the
 * rows of that support it owns, bit-identical to the single-device build. */

int sinkslot_partition_workspace_bytes(int64_t nnz, int64_t* bytes_host);

/* Stable partition of COO entries (seg, other, vals; other / vals nullable) by
 * the part owning seg: part p holds bounds_host[p] <= seg < bounds_host[p+1]
 * (host array of parts + 1 non-decreasing values, 1 <= parts <= 64; segments
 * outside the range go to the nearest end part).  Writes the entries part by
 * part, each part in input order, and counts_host[p] (host). */
int sinkslot_partition_coo(const int64_t* seg, const int64_t* other, const float* vals,
                           int64_t nnz, const int64_t* bounds_host, int parts, void* workspace,
                           int64_t workspace_bytes, int64_t* seg_out, int64_t* other_out,
                           float* vals_out, int64_t* counts_host, void* stream);

int sinkslot_coalesce_workspace_bytes(int64_t nraw, int64_t* bytes_host);

/* The coalesce of sot_plan_coo (sinkslot/solver.py:194-232) over raw entries
 * (R, C, mass) of an n x m problem with L slices: unique keys R * m + C in
 * ascending order, each key's masses summed in input order, times 1/L.
 * rows / cols / S need room for nraw entries; *nnz_host receives the count. */
int sinkslot_coalesce_coo(const int64_t* R, const int64_t* C, const float* mass, int64_t nraw,
                          int64_t n, int64_t m, int L, void* workspace, int64_t workspace_bytes,
                          int64_t* rows, int64_t* cols, float* S, int64_t* nnz_host,
                          void* stream);

int sinkslot_csr_workspace_bytes(int64_t nnz, int64_t nseg, int64_t* bytes_host);

/* COO -> CSR: replaces `to_csr(rows, cols, vals, n, narrow_key)`,
 * sinkslot/solver.py:235-276.  Stable by `seg`; identity permutation when
 * `seg` is already non-decreasing (*was_sorted_host = 1).  Writes indptr
 * (nseg + 1, int32), idx = other[perm] as int16 (idx_bytes 2) or int32
 * (idx_bytes 4), vals[perm] (vals/out_vals nullable) and perm (int64,
 * nullable).  With out_perm NULL (and vals given) the sort carries each
 * entry's index and value instead of its position: no gather afterwards. */
int sinkslot_coo_to_csr(const int64_t* seg, const int64_t* other, const float* vals, int64_t nnz,
                        int64_t nseg, int idx_bytes, void* workspace, int64_t workspace_bytes,
                        int32_t* indptr, void* idx, float* out_vals, int64_t* perm,
                        int* was_sorted_host, void* stream);

/* max(v) over n int64 (0 if n == 0): the `int(idx.max())` of solver.py:275.
 * workspace: 8 bytes. */
int sinkslot_max_index(const int64_t* v, int64_t n, void* workspace, int64_t* max_host,
                       void* stream);

/* ---------------------------------------------------------------------------
 * Cost and the Sinkhorn iteration
 * ------------------------------------------------------------------------- */

/* cost[k] = ||x[rows[k]] - y[cols[k]]||^2 and lam[k] = log(max(S[k], tiny)) -
 * cost[k] / eps.  Replaces `sparse_sqeuclidean_cost` (sinkslot/solver.py:303-360)
 * and the `lam` line of sinkslot_solve (sinkslot/sinkhorn_solvers.py:700).
 * lam / cost / S are nullable (lam needs S). */
int sinkslot_cost_lam(const float* x, const float* y, int d, const int64_t* rows,
                      const int64_t* cols, const float* S, int64_t nnz, double eps, float* lam,
                      float* cost, void* stream);

/* Segmented log-sum-exp half-step: out[s] = base[s] - LSE_{k in s}((lam[k] +
 * selfpot[s]) + other[idx[k]]) (out[s] = LSE when base is NULL; selfpot is
 * nullable and then zero).  Replaces `seg_lse_online(indptr, colidx, lam, phi,
 * psi, n, ..., base, out)`, sinkslot/sinkhorn_solvers.py:121-146, whose `phi`
 * is selfpot here (all-zero in the reference loops, :229). */
int sinkslot_seg_lse(const int32_t* indptr, const void* idx, int idx_bytes, const float* lam,
                     int64_t nnz, const float* selfpot, const float* other, const float* base,
                     int64_t nseg, float* out, void* stream);

/* Scratch floats sinkslot_solve_csr needs for an (n, m) problem. */
int sinkslot_solve_work_floats(int64_t n, int64_t m, int64_t* floats_host);

/* Bytes of the column-blocked layout of one CSR side (nseg segments gathering
 * from a potential of length m_other) and of the scratch its builder needs.
 * The geometry follows the current device's SM count: build and solve on the
 * same device model. */
int sinkslot_tiles_bytes(int64_t nseg, int64_t m_other, int64_t nnz, int64_t* layout_bytes_host,
                         int64_t* build_bytes_host);

/* The tiled layout's geometry: geom_host[0..4] = panels P, rows per panel R,
 * column blocks B, log2 of the block width W, dynamic shared memory bytes.
 * Layout bytes: int64 header[8] | int64 tile_start[P*B + 1] | uint32
 * entries[cap][2] = {row within panel << 16 | column within block, lam bits},
 * each part 256-byte aligned; tile t = p*B + b holds entries [tile_start[t],
 * tile_start[t+1]), padded with entries {R << 16, -inf} to 32 N entries, N
 * odd: with the tile's entries stably sorted by (row within panel) mod 32 (the
 * row bank), sorted position p is stored at slot 32*(p mod N) + p / N.  Inside
 * each row-bank run [S, S + c) of a tile of at most 9216 entries the entries
 * are then re-placed by column bank: the k-th entry (in run order) whose
 * column mod 32 is t goes to position S + ((t - S) mod 32) + 32 k when that is
 * below S + c, the others fill the remaining positions by class, then rank.
 * cap = nnz + 63*P*B. */
int sinkslot_tiles_geometry(int64_t nseg, int64_t m_other, int64_t nnz, int* geom_host);

/* How the half-step uses a tiled layout (no counterpart in the reference):
 * 1 staged -- one pass; each panel's CTA copies every block of the gathered
 * potential into shared memory (P * m_other * 4 bytes per half-step); 2
 * two-pass -- one CTA per block stages it once and stores each entry's
 * exponent lam + potential in layout order, then one CTA per panel sums its
 * entries with no gather (16 bytes per entry, all streamed; for gathered axes
 * too long to stage once per panel); 0 auto (the default) -- staged while
 * P * m_other * 4 <= 4 * nnz * 8, else two-pass.  The setting is process-wide
 * and read whenever a layout's geometry is computed (sinkslot_tiles_bytes,
 * sinkslot_tiles_geometry, sinkslot_build_tiles, the solve entry points): a
 * layout must be built and used under the same setting.  A two-pass layout is
 * the staged one followed by uint16 row byte offsets[cap], float
 * exponents[cap], uint16 column byte offsets[cap] and float lam[cap] (each
 * slot's entry split by what each pass reads; each part 256-byte aligned);
 * header[1..3] of every layout
 * hold its kind, P and B, and a half-step given a layout of another kind or
 * geometry fails with an error status instead of reading it. */
int sinkslot_set_tiles_kind(int kind);
int sinkslot_get_tiles_kind(int* kind_host);
/* The kind (1 or 2) a layout of these sizes gets under the current setting. */
int sinkslot_tiles_kind_of(int64_t nseg, int64_t m_other, int64_t nnz, int* kind_host);

/* Column-blocked layout of a CSR side for the shared-memory-staged half-step
 * (no counterpart in the reference: a layout of its CSR, `to_csr`,
 * sinkslot/solver.py:235-276, built once per solve). */
int sinkslot_build_tiles(const int32_t* indptr, const void* idx, int idx_bytes, const float* lam,
                         int64_t nseg, int64_t m_other, int64_t nnz, void* layout,
                         int64_t layout_bytes, void* workspace, int64_t workspace_bytes,
                         void* stream);

/* Full Sinkhorn loop over prebuilt CSR (rows) / CSC (cols): replaces
 * `sinkslot_alternating_triton` (variant 0) and `sinkslot_symmetric_triton`
 * (variant 1), sinkslot/sinkhorn_solvers.py:195-419, with the semantics of
 * their torch twins (:443-588).  stop_mode: 0 fixed (n_iters), 1 potential,
 * 2 marginal (up to max_iter, checked every check_every).  r_tiles / c_tiles
 * (each nullable) are layouts from sinkslot_build_tiles of the two sides; a
 * side with one runs the shared-memory-staged half-step (in the first
 * iteration only the alternating variant's column half-step does, after a
 * tiled max pass that gives its stabilisers), a side without the exact
 * kernel.  phi (n), psi (m) receive the absorbed potentials.
 * *converged_host: -1 (fixed mode), 0 or 1; *final_viol_host: NaN in fixed
 * mode. */
int sinkslot_solve_csr(const int32_t* r_ptr, const void* r_idx, int r_idx_bytes,
                       const float* r_lam, const int32_t* c_ptr, const void* c_idx,
                       int c_idx_bytes, const float* c_lam, int64_t nnz, const float* log_a,
                       const float* log_b, int64_t n, int64_t m, int variant, int stop_mode,
                       int64_t n_iters, int64_t max_iter, int64_t check_every, double tol,
                       double eps, double alpha, const void* r_tiles, int64_t r_tiles_bytes,
                       const void* c_tiles, int64_t c_tiles_bytes, float* phi, float* psi,
                       float* work, int64_t work_floats, int64_t* iters_host, int* converged_host,
                       double* final_viol_host, void* stream);

/* Capacity, in floats, of the library's static solve scratch (4 MiB held on
 * every device that loads the library, until the process exits). */
#define SINKSLOT_STATIC_SOLVE_FLOATS (1 << 20)

/* sinkslot_solve_csr without the work buffer: the loop's scratch is the
 * library's static device array (no counterpart in the reference; for callers
 * that cannot allocate device scratch).  Allocates nothing.  Status 1 when
 * sinkslot_solve_work_floats(n, m) > SINKSLOT_STATIC_SOLVE_FLOATS, i.e. when
 * 3 * (pad4(n) + pad4(m)) + 64 > 2^20 with pad4(v) = v rounded up to a multiple
 * of 4.  The first call on a device resolves the array's address and should
 * come before any stream capture there; the address is kept for the life of
 * the device's primary context (a host that resets the device with
 * cudaDeviceReset must not call this entry point on it again in the same
 * process).  Calls that overlap on one device share the array and race. */
int sinkslot_solve_csr_static(const int32_t* r_ptr, const void* r_idx, int r_idx_bytes,
                              const float* r_lam, const int32_t* c_ptr, const void* c_idx,
                              int c_idx_bytes, const float* c_lam, int64_t nnz,
                              const float* log_a, const float* log_b, int64_t n, int64_t m,
                              int variant, int stop_mode, int64_t n_iters, int64_t max_iter,
                              int64_t check_every, double tol, double eps, double alpha,
                              const void* r_tiles, int64_t r_tiles_bytes, const void* c_tiles,
                              int64_t c_tiles_bytes, float* phi, float* psi, int64_t* iters_host,
                              int* converged_host, double* final_viol_host, void* stream);

/* ---------------------------------------------------------------------------
 * Row/column-partitioned solve over the GPUs of one node (one process each)
 * ------------------------------------------------------------------------- */

#define SINKSLOT_IPC_HANDLE_BYTES 64

/* CUDA IPC handle of the allocation holding `ptr` (64 bytes into handle_host)
 * and ptr's byte offset inside it, for a peer process to map with
 * sinkslot_ipc_import (no counterpart in the reference). */
int sinkslot_ipc_export(const void* ptr, void* handle_host, int64_t* offset_host);
/* Maps a peer's allocation (peer access enabled); *ptr_host = base + offset. */
int sinkslot_ipc_import(const void* handle_host, int64_t offset, void** ptr_host);
/* Unmaps a pointer returned by sinkslot_ipc_import (same offset). */
int sinkslot_ipc_close(void* ptr, int64_t offset);

/* Scratch floats sinkslot_solve_shard needs for nr local rows and nc local
 * columns. */
int sinkslot_shard_work_floats(int64_t nr, int64_t nc, int64_t* floats_host);

/* The Sinkhorn loop of sinkslot_solve_csr (variant 0 alternating, 1
 * symmetric) for rank `rank` of `world` (<= 8) processes, one GPU each, that
 * partition the rows and columns (no counterpart in the reference, whose loop
 * runs on one device; sinkslot/sinkhorn_solvers.py:195-419).  This rank owns
 * CSR rows [r0, r0+nr) (r_ptr rebased to 0, r_idx global column ids) and CSC
 * columns [c0, c0+nc); r0 and c0 are multiples of 4.  phi_bufs_host[2g+k] /
 * psi_bufs_host[2g+k] are rank g's potential buffers k = 0, 1 (n / m floats;
 * k = 1 only for the symmetric variant) and flags_host[g] its `world` flag
 * words (zeroed before the first call), as mapped in this process: local for
 * g == rank, sinkslot_ipc_import'ed otherwise.  After each half-step the rank
 * stores its slice into every peer's buffer and publishes a barrier epoch; the
 * next half-step waits for all peers' epochs (bounded: a peer missing for ~4 s
 * fails the call with status 2).  Runs iterations it0 .. it0+n_iters-1; the
 * last carries check 0 none / 1 potential / 2 marginal and returns this rank's
 * two check maxima (row, column side) in *check0_host, *check1_host.
 * *cur_host: buffer index holding the current potentials (in/out);
 * *epoch_host: last epoch used (in/out, 0 before the first call). */
int sinkslot_solve_shard(const int32_t* r_ptr, const void* r_idx, int r_idx_bytes,
                         const float* r_lam, int64_t r_nnz, int64_t r0, int64_t nr,
                         const void* r_tiles, int64_t r_tiles_bytes, const int32_t* c_ptr,
                         const void* c_idx, int c_idx_bytes, const float* c_lam, int64_t c_nnz,
                         int64_t c0, int64_t nc, const void* c_tiles, int64_t c_tiles_bytes,
                         const float* log_a, const float* log_b, int64_t n, int64_t m,
                         int variant, double alpha, int rank, int world,
                         float* const* phi_bufs_host, float* const* psi_bufs_host,
                         uint32_t* const* flags_host, int64_t it0, int64_t n_iters, int check,
                         int* cur_host, uint32_t* epoch_host, float* work, int64_t work_floats,
                         double* check0_host, double* check1_host, void* stream);

/* ---------------------------------------------------------------------------
 * Plan export and gradient
 * ------------------------------------------------------------------------- */

/* Plan values exp(phi[r] + psi[c] + log S - cost / eps), cost recomputed from
 * x, y.  grad_form 0: `((phi[r] + psi[c]) + log_S) - cost/eps` as in
 * sparse_transport_plan (sinkslot/sinkhorn_solvers.py:757-758); grad_form 1:
 * `(phi[r] + psi[c]) + (log_S - cost/eps)` as in slot_grad / _SLOTCostFn
 * (sinkslot/gradient.py:94-97, sinkslot/samples_loss.py:69-73). */
int sinkslot_plan_values(const float* phi, const float* psi, const int64_t* rows,
                         const int64_t* cols, const float* S, const float* x, const float* y,
                         int d, int64_t nnz, double eps, int grad_form, float* out, void* stream);

int sinkslot_barycentric_workspace_bytes(int64_t nnz, int64_t n, int64_t m, int d,
                                         int64_t* bytes_host);

/* Barycentric projections of a sparse plan and the envelope gradient:
 * replaces `sparse_barycentric_map(T_vals, rows, cols, x, y)` (sinkslot/gradient.py:25-61)
 * and `2 * a[:, None] * (X - Tx)` (gradient.py:99, samples_loss.py:82).
 * Tx (n, d), Ty (m, d), grad (n, d) are nullable; grad needs a.  d <= 16. */
int sinkslot_barycentric(const float* T, const int64_t* rows, const int64_t* cols, int64_t nnz,
                         const float* x, const float* y, int64_t n, int64_t m, int d,
                         const float* a, float* Tx, float* Ty, float* grad, void* workspace,
                         int64_t workspace_bytes, void* stream);

int sinkslot_hvp_workspace_bytes(int64_t n, int64_t m, int64_t* bytes_host);

/* Hessian-vector product out = H(X) v of grad_X SLOT_eps on a frozen support:
 * replaces `hvp_x_sqeuclid_from_potentials` (sinkslot/hvp.py:34-113), whose
 * linear solve goes through torchsparsegradutils' MINRES.  The plan T is given
 * by rows (r_ptr, r_idx, r_T: CSR, n rows) and by columns (c_ptr, c_idx, c_T:
 * CSC, m columns); idx_bytes 2 or 4.  Solves [[diag(a + tau2), P], [P^T,
 * diag(b + tau2)]] [u; w] = rhs by MINRES on the device until the residual is
 * at most tol * ||rhs|| or max_iter iterations (the reference passes a for b:
 * one marginal for both clouds).  x (n, d), y (m, d), v (n, d) fp32, d <= 16.
 * sol_out (nullable, n + m) receives (u, w); *iters_host the iterations run,
 * *resid_host the final relative residual. */
int sinkslot_hvp(const float* x, const float* y, int d, const float* v, const float* a,
                 const float* b, const int32_t* r_ptr, const void* r_idx, const float* r_T,
                 const int32_t* c_ptr, const void* c_idx, const float* c_T, int idx_bytes,
                 int64_t n, int64_t m, double eps, double tau2, double tol, int64_t max_iter,
                 void* workspace, int64_t workspace_bytes, float* out, float* sol_out,
                 int64_t* iters_host, double* resid_host, void* stream);

/* dual value <phi, a> + <psi, b> accumulated in fp64 into out[0] (device);
 * the caller multiplies by eps (sinkslot/samples_loss.py:74). */
int sinkslot_dual_value(const float* phi, const float* a, int64_t n, const float* psi,
                        const float* b, int64_t m, double* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SINKSLOT_B200_H_ */
