// attention.cuh - declarations shared by the two decode-attention kernels
// (CUDA-core kernel in attention_decode.cu, tcgen05 kernel in
// attention_decode_tc.cu): launch arguments and the split-K epilogue.
#pragma once

#include "common.cuh"
#include "context.h"

namespace hcu {

constexpr int kMaxSplits = 64;      // key splits per (sequence, KV head, query block)
constexpr int kMaxUnits = 1 << 16;  // ticket slots at the head of the workspace

struct AttnArgs {
  const float* q;
  float* out;
  const int32_t* pos_base;
  const int64_t* row_off;
  unsigned long long seq_row_stride;
  int S, H, KV, G, QB, nqb, window, pos_base_default;
  int chunk;       // keys per split (multiple of the kernel's tile)
  int max_splits;  // gridDim.x
  float qscale;    // log2(e) / sqrt(Dh)
  float* part;     // [units, max_splits, R, DH + 2]: acc[DH], m (log2), l
  int* counters;   // [kMaxUnits] split-merge tickets, 0 between calls
  uint32_t* status;
};

// Per-CTA geometry shared by both kernels.
struct AttnUnit {
  int b, g, qb, pb, q0, qn, kstart, kend, nsplit, k_lo, k_hi, unit, rows_valid;
  long long roff;
};

__device__ __forceinline__ AttnUnit attn_unit(const AttnArgs& a, int split) {
  AttnUnit u;
  u.g = blockIdx.y;
  u.b = blockIdx.z / a.nqb;
  u.qb = blockIdx.z % a.nqb;
  u.pb = a.pos_base ? a.pos_base[u.b] : a.pos_base_default;
  u.roff = a.row_off ? a.row_off[u.b] : (long long)u.b * (long long)a.seq_row_stride;
  u.q0 = u.qb * a.QB;
  u.qn = min(a.QB, a.S - u.q0);
  const int pos_first = u.pb + u.q0, pos_last = u.pb + u.q0 + u.qn - 1;
  u.kstart = (a.window > 0 && pos_first + 1 > a.window) ? pos_first + 1 - a.window : 0;
  u.kend = pos_last + 1;
  u.nsplit = (u.kend - u.kstart + a.chunk - 1) / a.chunk;
  u.k_lo = u.kstart + split * a.chunk;
  u.k_hi = min(u.kend, u.k_lo + a.chunk);
  u.unit = (u.b * a.KV + u.g) * a.nqb + u.qb;
  u.rows_valid = min(a.QB * a.G, u.qn * a.G);
  return u;
}

__device__ __forceinline__ size_t out_index(const AttnArgs& a, const AttnUnit& u, int r, int d, int DH) {
  const int qi = u.q0 + r / a.G, h = u.g * a.G + r % a.G;
  return (((size_t)u.b * a.S + qi) * a.H + h) * DH + d;
}

// After every thread of the CTA has written its split's partial
// (acc, m, l) for unit u: take a ticket; the CTA drawing the last one merges
// all splits of the unit and re-arms the ticket.  `nthr` threads with ids
// 0..nthr-1 take part, synchronising on named barrier `barid`.  `scratch`
// holds >= 3 * kMaxSplits * R floats of shared memory.
template <int R, int DH>
__device__ void ticket_merge(const AttnArgs& a, const AttnUnit& u, int tid, int nthr, int barid, float* scratch,
                             int* s_last) {
  __threadfence();
  named_bar(barid, nthr);
  if (tid == 0) *s_last = (atomicAdd(&a.counters[u.unit], 1) == u.nsplit - 1);
  named_bar(barid, nthr);
  if (!*s_last) return;
  __threadfence();
  const float* up = a.part + (size_t)u.unit * a.max_splits * R * (DH + 2);
  float* Ms = scratch;                     // [nsplit][R]
  float* Ls = scratch + kMaxSplits * R;    // [nsplit][R]
  float* Ws = scratch + 2 * kMaxSplits * R;
  for (int i = tid; i < u.nsplit * R; i += nthr) {
    const float* pp = up + (size_t)i * (DH + 2);
    Ms[i] = __ldcg(pp + DH);
    Ls[i] = __ldcg(pp + DH + 1);
  }
  named_bar(barid, nthr);
  for (int r = tid; r < R; r += nthr) {
    float M = -1e30f;
    for (int sp = 0; sp < u.nsplit; sp++) M = fmaxf(M, Ms[sp * R + r]);
    float L = 0.f;
    for (int sp = 0; sp < u.nsplit; sp++) L += Ls[sp * R + r] * exp2f(Ms[sp * R + r] - M);
    const float inv = 1.f / L;
    for (int sp = 0; sp < u.nsplit; sp++) Ws[sp * R + r] = exp2f(Ms[sp * R + r] - M) * inv;
  }
  named_bar(barid, nthr);
  for (int e = tid; e < u.rows_valid * DH; e += nthr) {
    const int r = e / DH, d = e % DH;
    float A = 0.f;
    for (int sp = 0; sp < u.nsplit; sp++) A = fmaf(__ldcg(up + ((size_t)sp * R + r) * (DH + 2) + d), Ws[sp * R + r], A);
    a.out[out_index(a, u, r, d, DH)] = A;
  }
  if (tid == 0) a.counters[u.unit] = 0;  // re-arm for the next call
}

// Host launcher of the tcgen05 kernel (attention_decode_tc.cu).  Returns
// HCU_EUNSUPPORTED when the shape has no tensor-core variant.
int launch_attn_tc(hcu_context* h, int fmt, int R, const AttnArgs& args, dim3 grid, const CUtensorMap& tk,
                   const CUtensorMap& tv);
bool attn_tc_supported(int fmt, int Dh, int R);
constexpr int kTcTile = 128;  // tokens per tcgen05 tile

}  // namespace hcu
