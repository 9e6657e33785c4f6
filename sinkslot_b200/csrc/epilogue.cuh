// epilogue.cuh -- what a half-step does with one segment's log-sum-exp:
// res = base - lse (lse itself without base), then the write mode and the
// stop-criterion contribution.  Shared by the exact and the tiled half-steps so
// both produce the same bits for the same lse.
#pragma once

#include <cfloat>

#include "common.cuh"

namespace sinkslot {

// kOutMax: the tiled pass writes each segment's largest term lam + other instead
// of a potential (the stabilisers of a following pass; tiled.cu only).
enum OutMode { kOutPlain = 0, kOutBlend = 1, kOutNone = 2, kOutMax = 3 };
enum CheckMode { kChkNone = 0, kChkMarg = 1, kChkPot = 2 };

// Copies of a half-step's output in other GPUs' potential buffers (mapped into
// this process), indexed like `out`: the epilogue stores each value there too.
constexpr int kMaxPeers = 7;
struct PeerOut {
  float* p[kMaxPeers];
  int n;
};

// The end of a CTA of a half-step whose epilogue stored into peers: after all
// of the CTA's threads (those in `bar`) are done, one thread makes their stores
// visible system-wide and counts the CTA in *done (the publish step acquires
// the count before it raises the peers' flags).
__device__ __forceinline__ void peer_cta_done(const PeerOut& po, unsigned int* done) {
  if (po.n > 0 && done != nullptr && threadIdx.x == 0) {
    __threadfence_system();
    atomicAdd(done, 1u);
  }
}

// sinkhorn_solvers.py: the reference's `base - LSE` (:91-93), the symmetric
// blend `(1 - alpha) * x + alpha * cand` (:361-363), the marginal proxy
// `|a * exp(old - new) - a|` (:280-283, :405-412) and the potential change
// `|new - prev|` (:250-254).
// The same with the segment's inputs already loaded: b = base[seg] (has_base),
// old = self_old[seg] (read when OUT == kOutBlend or CHK == kChkMarg), prv =
// prev[seg] (read when CHK == kChkPot) -- so that a caller can have several
// segments' loads in flight before it finishes any of them.
template <int OUT, int CHK>
__device__ __forceinline__ void segment_epilogue_loaded(int64_t seg, float lse, bool has_base,
                                                        float b, float old, float prv, float* out,
                                                        float w_old, float w_new, float* prev,
                                                        uint32_t& chk_bits, const PeerOut& po) {
  const float res = has_base ? __fsub_rn(b, lse) : lse;
  float nv = res;
  if (OUT == kOutBlend) nv = __fadd_rn(__fmul_rn(w_old, old), __fmul_rn(w_new, res));
  if (OUT != kOutNone) {
    out[seg] = nv;
#pragma unroll
    for (int g = 0; g < kMaxPeers; ++g)  // constant indices: po stays in parameter space
      if (g < po.n) po.p[g][seg] = nv;
  }
  if (CHK == kChkMarg) {
    const float ea = expf(b);
    const float t = __fmul_rn(ea, expf(__fsub_rn(old, res)));
    chk_bits = max(chk_bits, nonneg_float_bits(__fsub_rn(t, ea)));
  } else if (CHK == kChkPot) {
    chk_bits = max(chk_bits, nonneg_float_bits(__fsub_rn(nv, prv)));
    prev[seg] = nv;
  }
}

template <int OUT, int CHK>
__device__ __forceinline__ void segment_epilogue(int64_t seg, float lse, const float* base,
                                                 const float* self_old, float* out, float w_old,
                                                 float w_new, float* prev, uint32_t& chk_bits,
                                                 const PeerOut& po) {
  const float b = base ? base[seg] : 0.0f;
  const float old = (OUT == kOutBlend || CHK == kChkMarg) ? self_old[seg] : 0.0f;
  const float prv = CHK == kChkPot ? prev[seg] : 0.0f;
  segment_epilogue_loaded<OUT, CHK>(seg, lse, base != nullptr, b, old, prv, out, w_old, w_new,
                                    prev, chk_bits, po);
}

template <int CHK>
__device__ __forceinline__ void check_reduce(uint32_t chk_bits, uint32_t* acc) {
  if (CHK != kChkNone) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1)
      chk_bits = max(chk_bits, __shfl_xor_sync(0xffffffffu, chk_bits, o));
    if ((threadIdx.x & 31) == 0 && chk_bits) atomicMax(acc, chk_bits);
  }
}

}  // namespace sinkslot
