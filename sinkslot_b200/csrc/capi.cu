// capi.cu -- extern "C" entry points of libsinkslot_b200.so (declared in
// include/sinkslot_b200.h).  Thin argument checks + dispatch to the launchers.
#include <string>

#include "../../include/sinkslot_b200.h"
#include "common.cuh"
#include "export.h"
#include "hvp.h"
#include "primitives.h"
#include "sinkhorn.h"
#include "support.h"

namespace sinkslot {

static thread_local std::string g_last_error;
void set_error(const std::string& msg) { g_last_error = msg; }
const char* last_error() { return g_last_error.c_str(); }

}  // namespace sinkslot

using namespace sinkslot;

#define ST(s) static_cast<cudaStream_t>(s)

// Clear the previous message, run, and keep the message only on failure.
#define CAPI_BODY(expr)        \
  do {                         \
    g_last_error_clear();      \
    return (expr);             \
  } while (0)

static void g_last_error_clear() { set_error(""); }

extern "C" {

const char* sinkslot_last_error(void) { return last_error(); }

int sinkslot_abi_version(void) { return 101; }

int sinkslot_project(const float* X, int64_t n, int d, const float* theta, int L, float* out,
                     void* stream) {
  CAPI_BODY(project(X, n, d, theta, L, out, ST(stream)));
}

int sinkslot_ot1d_workspace_bytes(int64_t n, int64_t m, int C, int64_t* bytes_host) {
  g_last_error_clear();
  SINKSLOT_REQUIRE(bytes_host && n >= 1 && m >= 1 && C >= 1, "ot1d_workspace_bytes: bad args");
  *bytes_host = (int64_t)ot1d_workspace_bytes(n, m, C);
  return kOk;
}

int sinkslot_ot1d_batched(const float* PXt, const float* PYt, const float* a, const float* b,
                          int64_t n, int64_t m, int C, int scan_rows, void* workspace,
                          int64_t workspace_bytes, int64_t* R, int64_t* Cc, float* mass,
                          uint32_t* ix, uint32_t* iy, float* ca, float* cb, int64_t* count_host,
                          void* stream) {
  g_last_error_clear();
  SINKSLOT_REQUIRE(PXt && PYt && a && b && R && Cc && mass && count_host && workspace,
                   "ot1d_batched: null argument");
  return ot1d_batched(PXt, PYt, a, b, n, m, C, scan_rows, workspace, (size_t)workspace_bytes, R,
                      Cc, mass, ix, iy, ca, cb, count_host, ST(stream));
}

int sinkslot_support_workspace_bytes(int64_t n, int64_t m, int d, int L, int chunk,
                                     int64_t* bytes_host) {
  g_last_error_clear();
  SINKSLOT_REQUIRE(bytes_host && n >= 1 && m >= 1 && d >= 1 && L >= 1,
                   "support_workspace_bytes: bad args");
  *bytes_host = (int64_t)support_workspace_bytes(n, m, d, L, chunk);
  return kOk;
}

int sinkslot_build_support(const float* X, const float* Y, const float* a, const float* b,
                           int64_t n, int64_t m, int d, const float* theta, const float* PX,
                           const float* PY, int L, int chunk, void* workspace,
                           int64_t workspace_bytes, int64_t* nnz_host, void* stream) {
  g_last_error_clear();
  SINKSLOT_REQUIRE(a && b && workspace && nnz_host && ((X && Y && theta) || (PX && PY)),
                   "build_support: null argument");
  return build_support(X, Y, a, b, n, m, d, theta, PX, PY, L, chunk, workspace,
                       (size_t)workspace_bytes, nnz_host, ST(stream));
}

int sinkslot_support_export(const void* workspace, int64_t workspace_bytes, int64_t n, int64_t m,
                            int d, int L, int chunk, int64_t nnz, int64_t* rows, int64_t* cols,
                            float* S, void* stream) {
  g_last_error_clear();
  SINKSLOT_REQUIRE(workspace && (nnz == 0 || (rows && cols && S)), "support_export: null argument");
  return support_export(workspace, (size_t)workspace_bytes, n, m, d, L, chunk, nnz, rows, cols, S,
                        ST(stream));
}

int sinkslot_partition_workspace_bytes(int64_t nnz, int64_t* bytes_host) {
  g_last_error_clear();
  SINKSLOT_REQUIRE(bytes_host && nnz >= 0, "partition_workspace_bytes: bad args");
  *bytes_host = (int64_t)partition_workspace_bytes(nnz);
  return kOk;
}

int sinkslot_partition_coo(const int64_t* seg, const int64_t* other, const float* vals,
                           int64_t nnz, const int64_t* bounds_host, int parts, void* workspace,
                           int64_t workspace_bytes, int64_t* seg_out, int64_t* other_out,
                           float* vals_out, int64_t* counts_host, void* stream) {
  g_last_error_clear();
  SINKSLOT_REQUIRE(workspace && (nnz == 0 || (seg && seg_out)) && (!other || other_out) &&
                       (!vals || vals_out),
                   "partition_coo: null argument");
  return partition_coo(seg, other, vals, nnz, bounds_host, parts, workspace,
                       (size_t)workspace_bytes, seg_out, other_out, vals_out, counts_host,
                       ST(stream));
}

int sinkslot_coalesce_workspace_bytes(int64_t nraw, int64_t* bytes_host) {
  g_last_error_clear();
  SINKSLOT_REQUIRE(bytes_host && nraw >= 0, "coalesce_workspace_bytes: bad args");
  *bytes_host = (int64_t)coalesce_workspace_bytes(nraw);
  return kOk;
}

int sinkslot_coalesce_coo(const int64_t* R, const int64_t* C, const float* mass, int64_t nraw,
                          int64_t n, int64_t m, int L, void* workspace, int64_t workspace_bytes,
                          int64_t* rows, int64_t* cols, float* S, int64_t* nnz_host,
                          void* stream) {
  g_last_error_clear();
  SINKSLOT_REQUIRE(workspace && (nraw == 0 || (R && C && mass && rows && cols && S)),
                   "coalesce_coo: null argument");
  return coalesce_coo(R, C, mass, nraw, n, m, L, workspace, (size_t)workspace_bytes, rows, cols,
                      S, nnz_host, ST(stream));
}

int sinkslot_hvp_workspace_bytes(int64_t n, int64_t m, int64_t* bytes_host) {
  g_last_error_clear();
  SINKSLOT_REQUIRE(bytes_host && n >= 0 && m >= 0, "hvp_workspace_bytes: bad args");
  *bytes_host = (int64_t)hvp_workspace_bytes(n, m);
  return kOk;
}

int sinkslot_hvp(const float* x, const float* y, int d, const float* v, const float* a,
                 const float* b, const int32_t* r_ptr, const void* r_idx, const float* r_T,
                 const int32_t* c_ptr, const void* c_idx, const float* c_T, int idx_bytes,
                 int64_t n, int64_t m, double eps, double tau2, double tol, int64_t max_iter,
                 void* workspace, int64_t workspace_bytes, float* out, float* sol_out,
                 int64_t* iters_host, double* resid_host, void* stream) {
  g_last_error_clear();
  SINKSLOT_REQUIRE(x && y && v && a && b && r_ptr && c_ptr && workspace && out,
                   "hvp: null argument");
  HvpArgs h;
  h.x = x; h.y = y; h.v = v; h.a = a; h.b = b; h.d = d;
  h.r_ptr = r_ptr; h.r_idx = r_idx; h.r_T = r_T;
  h.c_ptr = c_ptr; h.c_idx = c_idx; h.c_T = c_T; h.idx_bytes = idx_bytes;
  h.n = n; h.m = m; h.eps = eps; h.tau2 = tau2; h.tol = tol; h.max_iter = max_iter;
  h.ws = workspace; h.ws_bytes = (size_t)workspace_bytes;
  h.out = out; h.sol_out = sol_out; h.iters_host = iters_host; h.resid_host = resid_host;
  return hvp(h, ST(stream));
}

int sinkslot_csr_workspace_bytes(int64_t nnz, int64_t nseg, int64_t* bytes_host) {
  g_last_error_clear();
  SINKSLOT_REQUIRE(bytes_host && nnz >= 0 && nseg >= 0, "csr_workspace_bytes: bad args");
  *bytes_host = (int64_t)csr_workspace_bytes(nnz, nseg);
  return kOk;
}

int sinkslot_coo_to_csr(const int64_t* seg, const int64_t* other, const float* vals, int64_t nnz,
                        int64_t nseg, int idx_bytes, void* workspace, int64_t workspace_bytes,
                        int32_t* indptr, void* idx, float* out_vals, int64_t* perm,
                        int* was_sorted_host, void* stream) {
  g_last_error_clear();
  SINKSLOT_REQUIRE(indptr && was_sorted_host && workspace && (nnz == 0 || (seg && other && idx)),
                   "to_csr: null argument");
  SINKSLOT_REQUIRE(vals == nullptr || out_vals != nullptr, "to_csr: vals given without out_vals");
  return coo_to_csr(seg, other, vals, nnz, nseg, idx_bytes, workspace, (size_t)workspace_bytes,
                    indptr, idx, vals ? out_vals : nullptr, perm, was_sorted_host, ST(stream));
}

int sinkslot_max_index(const int64_t* v, int64_t n, void* workspace, int64_t* max_host,
                       void* stream) {
  g_last_error_clear();
  SINKSLOT_REQUIRE(workspace && max_host && (n == 0 || v), "max_index: null argument");
  return max_index(v, n, workspace, max_host, ST(stream));
}

int sinkslot_cost_lam(const float* x, const float* y, int d, const int64_t* rows,
                      const int64_t* cols, const float* S, int64_t nnz, double eps, float* lam,
                      float* cost, void* stream) {
  g_last_error_clear();
  SINKSLOT_REQUIRE(nnz == 0 || (x && y && rows && cols), "cost_lam: null argument");
  SINKSLOT_REQUIRE(lam == nullptr || eps != 0.0, "cost_lam: eps must be nonzero");
  return cost_lam(x, y, d, rows, cols, S, nnz, eps, lam, cost, ST(stream));
}

int sinkslot_seg_lse(const int32_t* indptr, const void* idx, int idx_bytes, const float* lam,
                     int64_t nnz, const float* selfpot, const float* other, const float* base,
                     int64_t nseg, float* out, void* stream) {
  g_last_error_clear();
  SINKSLOT_REQUIRE(indptr && out && (nnz == 0 || (idx && lam && other)), "seg_lse: null argument");
  HalfStep h;
  h.ptr = indptr;
  h.idx = idx;
  h.idx_bytes = idx_bytes;
  h.lam = lam;
  h.nseg = nseg;
  h.nnz = nnz;
  h.other = other;
  h.selfpot = selfpot;
  h.base = base;
  h.out = out;
  h.self_old = out;
  return half_step(h, 0, 0, ST(stream));
}

int sinkslot_solve_work_floats(int64_t n, int64_t m, int64_t* floats_host) {
  g_last_error_clear();
  SINKSLOT_REQUIRE(floats_host && n >= 0 && m >= 0, "solve_work_floats: bad args");
  *floats_host = (int64_t)solve_work_floats(n, m);
  return kOk;
}

int sinkslot_solve_csr(const int32_t* r_ptr, const void* r_idx, int r_idx_bytes,
                       const float* r_lam, const int32_t* c_ptr, const void* c_idx,
                       int c_idx_bytes, const float* c_lam, int64_t nnz, const float* log_a,
                       const float* log_b, int64_t n, int64_t m, int variant, int stop_mode,
                       int64_t n_iters, int64_t max_iter, int64_t check_every, double tol,
                       double eps, double alpha, const void* r_tiles, int64_t r_tiles_bytes,
                       const void* c_tiles, int64_t c_tiles_bytes, float* phi, float* psi,
                       float* work, int64_t work_floats, int64_t* iters_host, int* converged_host,
                       double* final_viol_host, void* stream) {
  g_last_error_clear();
  SINKSLOT_REQUIRE(r_ptr && c_ptr && log_a && log_b && phi && psi && work && iters_host &&
                       converged_host && final_viol_host,
                   "solve_csr: null argument");
  SINKSLOT_REQUIRE(nnz == 0 || (r_idx && r_lam && c_idx && c_lam), "solve_csr: null argument");
  SolveSpec sp;
  // either side may run tiled or exact (a null layout)
  if (r_tiles) {
    sp.row_geom = tile_geom(n, m, nnz, num_sms());
    SINKSLOT_REQUIRE(r_tiles_bytes >= (int64_t)sp.row_geom.layout_bytes,
                     "solve_csr: tiled layout buffer too small");
    sp.row_tiles = r_tiles;
  }
  if (c_tiles) {
    sp.col_geom = tile_geom(m, n, nnz, num_sms());
    SINKSLOT_REQUIRE(c_tiles_bytes >= (int64_t)sp.col_geom.layout_bytes,
                     "solve_csr: tiled layout buffer too small");
    sp.col_tiles = c_tiles;
  }
  sp.row.ptr = r_ptr;
  sp.row.idx = r_idx;
  sp.row.idx_bytes = r_idx_bytes;
  sp.row.lam = r_lam;
  sp.row.nseg = n;
  sp.row.nnz = nnz;
  sp.col.ptr = c_ptr;
  sp.col.idx = c_idx;
  sp.col.idx_bytes = c_idx_bytes;
  sp.col.lam = c_lam;
  sp.col.nseg = m;
  sp.col.nnz = nnz;
  sp.log_a = log_a;
  sp.log_b = log_b;
  sp.variant = variant;
  sp.mode = stop_mode;
  sp.n_iters = n_iters;
  sp.max_iter = max_iter;
  sp.check_every = check_every;
  sp.tol = tol;
  sp.eps = eps;
  sp.alpha = alpha;
  return solve_loop(sp, phi, psi, work, work_floats, iters_host, converged_host, final_viol_host,
                    ST(stream));
}

int sinkslot_tiles_bytes(int64_t nseg, int64_t m_other, int64_t nnz, int64_t* layout_bytes_host,
                         int64_t* build_bytes_host) {
  g_last_error_clear();
  SINKSLOT_REQUIRE(layout_bytes_host && build_bytes_host && nseg >= 1 && m_other >= 1 && nnz >= 0,
                   "tiles_bytes: bad args");
  const TileGeom g = tile_geom(nseg, m_other, nnz, num_sms());
  *layout_bytes_host = (int64_t)g.layout_bytes;
  *build_bytes_host = (int64_t)g.build_bytes;
  return kOk;
}

int sinkslot_tiles_geometry(int64_t nseg, int64_t m_other, int64_t nnz, int* geom_host) {
  g_last_error_clear();
  SINKSLOT_REQUIRE(geom_host && nseg >= 1 && m_other >= 1 && nnz >= 0, "tiles_geometry: bad args");
  const TileGeom g = tile_geom(nseg, m_other, nnz, num_sms());
  geom_host[0] = g.P;
  geom_host[1] = g.R;
  geom_host[2] = g.B;
  geom_host[3] = g.logW;
  geom_host[4] = (int)g.smem_bytes;
  return kOk;
}

int sinkslot_set_tiles_kind(int kind) {
  g_last_error_clear();
  SINKSLOT_REQUIRE(kind == kTilesAuto || kind == kTilesStaged || kind == kTilesTwoPass,
                   "set_tiles_kind: kind must be 0 (auto), 1 (staged) or 2 (two-pass)");
  set_tiles_kind(kind);
  return kOk;
}

int sinkslot_get_tiles_kind(int* kind_host) {
  g_last_error_clear();
  SINKSLOT_REQUIRE(kind_host != nullptr, "get_tiles_kind: null argument");
  *kind_host = tiles_kind();
  return kOk;
}

int sinkslot_tiles_kind_of(int64_t nseg, int64_t m_other, int64_t nnz, int* kind_host) {
  g_last_error_clear();
  SINKSLOT_REQUIRE(kind_host && nseg >= 1 && m_other >= 1 && nnz >= 0, "tiles_kind_of: bad args");
  *kind_host = tile_geom(nseg, m_other, nnz, num_sms()).kind;
  return kOk;
}

int sinkslot_build_tiles(const int32_t* indptr, const void* idx, int idx_bytes, const float* lam,
                         int64_t nseg, int64_t m_other, int64_t nnz, void* layout,
                         int64_t layout_bytes, void* workspace, int64_t workspace_bytes,
                         void* stream) {
  g_last_error_clear();
  SINKSLOT_REQUIRE(indptr && layout && workspace && (nnz == 0 || (idx && lam)),
                   "build_tiles: null argument");
  SINKSLOT_REQUIRE(nseg >= 1 && m_other >= 1 && nnz >= 0, "build_tiles: bad sizes");
  const TileGeom g = tile_geom(nseg, m_other, nnz, num_sms());
  SINKSLOT_REQUIRE(layout_bytes >= (int64_t)g.layout_bytes, "build_tiles: layout buffer too small");
  SINKSLOT_REQUIRE(workspace_bytes >= (int64_t)g.build_bytes, "build_tiles: workspace too small");
  return build_tiles(indptr, idx, idx_bytes, lam, g, layout, workspace, (size_t)workspace_bytes,
                     ST(stream));
}

int sinkslot_plan_values(const float* phi, const float* psi, const int64_t* rows,
                         const int64_t* cols, const float* S, const float* x, const float* y,
                         int d, int64_t nnz, double eps, int grad_form, float* out, void* stream) {
  g_last_error_clear();
  SINKSLOT_REQUIRE(nnz == 0 || (phi && psi && rows && cols && S && x && y && out),
                   "plan_values: null argument");
  SINKSLOT_REQUIRE(eps != 0.0, "plan_values: eps must be nonzero");
  return plan_values(phi, psi, rows, cols, S, x, y, d, nnz, eps, grad_form, out, ST(stream));
}

int sinkslot_barycentric_workspace_bytes(int64_t nnz, int64_t n, int64_t m, int d,
                                         int64_t* bytes_host) {
  g_last_error_clear();
  SINKSLOT_REQUIRE(bytes_host && nnz >= 0 && n >= 0 && m >= 0 && d >= 1,
                   "barycentric_workspace_bytes: bad args");
  *bytes_host = (int64_t)bary_workspace_bytes(nnz, n, m, d);
  return kOk;
}

int sinkslot_barycentric(const float* T, const int64_t* rows, const int64_t* cols, int64_t nnz,
                         const float* x, const float* y, int64_t n, int64_t m, int d,
                         const float* a, float* Tx, float* Ty, float* grad, void* workspace,
                         int64_t workspace_bytes, void* stream) {
  g_last_error_clear();
  SINKSLOT_REQUIRE(workspace && x && y && (nnz == 0 || (T && rows && cols)),
                   "barycentric: null argument");
  return barycentric(T, rows, cols, nnz, x, y, n, m, d, a, Tx, Ty, grad, workspace,
                     (size_t)workspace_bytes, ST(stream));
}

int sinkslot_dual_value(const float* phi, const float* a, int64_t n, const float* psi,
                        const float* b, int64_t m, double* out, void* stream) {
  g_last_error_clear();
  SINKSLOT_REQUIRE(out && (n == 0 || (phi && a)) && (m == 0 || (psi && b)),
                   "dual_value: null argument");
  return dual_value(phi, a, n, psi, b, m, out, ST(stream));
}

}  // extern "C"
