// attention.cuh - declarations shared by the two decode-attention kernels
// (CUDA-core kernel in attention_decode.cu, tcgen05 kernel in
// attention_decode_tc.cu): launch arguments and the split-K epilogue.
#pragma once

#include "common.cuh"
#include "context.h"

namespace hcu {

constexpr int kMaxSplits = 64;      // key splits per (sequence, KV head, query block)

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
  int cluster;     // 1: the split CTAs of a unit are one thread-block cluster and merge through DSMEM
  uint32_t* status;
  const float* gate;  // null, or [B, S, H, Dh]: out *= sigmoid(gate) (qwen35 sigmoid_gate)
  float q8_smul;      // Q8_0: element = q * scale * q8_smul (1, or 1/127 for the WGSL convention)
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

// Writes one output element, times sigmoid(gate) when the call carries the
// qwen35 output gate (sigmoid_gate, src/kernels.ts:1249-1262: att * (1 / (1 +
// exp(-gate)))).
__device__ __forceinline__ void store_out(const AttnArgs& a, size_t idx, float v) {
  if (a.gate) v *= 1.f / (1.f + expf(-a.gate[idx]));
  a.out[idx] = v;
}

// After every thread of the CTA has written its split's partial
// (acc, m, l) for unit u: take a ticket; the CTA drawing the last one merges
// all splits of the unit and re-arms the ticket.  NT threads with ids
// 0..NT-1 take part, synchronising on named barrier `barid`.  `scratch`
// holds >= kMaxSplits * R floats of shared memory.
//
// The merge is latency-bound (a few KB to a few hundred KB read from L2 by
// one CTA), so every phase keeps many independent loads in flight: one warp
// per row gathers that row's (m, l) of all splits at once, and each thread
// accumulates its R*DH/NT output elements over batches of splits whose loads
// are issued together (about 32 in flight per thread).
template <int R, int DH, int NT>
__device__ void ticket_merge(const AttnArgs& a, const AttnUnit& u, int tid, int barid, float* scratch,
                             int* s_last) {
  static_assert(NT % 32 == 0 && kMaxSplits % 32 == 0, "merge geometry");
  __threadfence();
  named_bar(barid, NT);
  if (tid == 0) *s_last = (atomicAdd(&a.counters[u.unit], 1) == u.nsplit - 1);
  named_bar(barid, NT);
  if (!*s_last) return;
  __threadfence();
  const int n = u.nsplit;
  constexpr size_t RS = DH + 2;  // floats per (split, row) record
  const float* up = a.part + (size_t)u.unit * a.max_splits * R * RS;
  float* Ws = scratch;  // [kMaxSplits][R]: weight of split sp in row r
  const int warp = tid >> 5, lane = tid & 31;
  constexpr int SPL = kMaxSplits / 32;  // splits per lane
  for (int r = warp; r < R; r += NT / 32) {
    float mv[SPL], lv[SPL];
#pragma unroll
    for (int i = 0; i < SPL; i++) {
      const int sp = lane + 32 * i;
      const float* pp = up + ((size_t)min(sp, n - 1) * R + r) * RS;
      mv[i] = __ldcg(pp + DH);
      lv[i] = __ldcg(pp + DH + 1);
    }
#pragma unroll
    for (int i = 0; i < SPL; i++) {
      if (lane + 32 * i >= n) {
        mv[i] = -1e30f;
        lv[i] = 0.f;
      }
    }
    float M = mv[0];
#pragma unroll
    for (int i = 1; i < SPL; i++) M = fmaxf(M, mv[i]);
    M = warp_max(M);
    float L = 0.f;
#pragma unroll
    for (int i = 0; i < SPL; i++) L += lv[i] * exp2f(mv[i] - M);
    const float inv = 1.f / warp_sum(L);
#pragma unroll
    for (int i = 0; i < SPL; i++) {
      const int sp = lane + 32 * i;
      if (sp < n) Ws[sp * R + r] = exp2f(mv[i] - M) * inv;
    }
  }
  named_bar(barid, NT);

  constexpr int E = R * DH;                   // output elements of the unit
  constexpr int EPT = (E + NT - 1) / NT;      // elements per thread
  constexpr int SB = EPT >= 32 ? 1 : 32 / EPT;  // splits per load batch
  float acc[EPT];
#pragma unroll
  for (int k = 0; k < EPT; k++) acc[k] = 0.f;
  // Loads use clamped (always valid) indices and are unconditional, so the
  // compiler issues a whole batch before the first use; splits past the end
  // get weight 0.
  for (int sp0 = 0; sp0 < n; sp0 += SB) {
    float x[SB][EPT];
#pragma unroll
    for (int j = 0; j < SB; j++)
#pragma unroll
      for (int k = 0; k < EPT; k++) {
        const int sp = min(sp0 + j, n - 1), e = min(tid + k * NT, E - 1), r = e / DH, d = e % DH;
        x[j][k] = __ldcg(up + ((size_t)sp * R + r) * RS + d);
      }
#pragma unroll
    for (int j = 0; j < SB; j++)
#pragma unroll
      for (int k = 0; k < EPT; k++) {
        const int sp = min(sp0 + j, n - 1), r = min(tid + k * NT, E - 1) / DH;
        const float wgt = sp0 + j < n ? Ws[sp * R + r] : 0.f;
        acc[k] = fmaf(x[j][k], wgt, acc[k]);
      }
  }
#pragma unroll
  for (int k = 0; k < EPT; k++) {
    const int e = tid + k * NT, r = e / DH, d = e % DH;
    if (e < E && r < u.rows_valid) store_out(a, out_index(a, u, r, d, DH), acc[k]);
  }
  if (tid == 0) a.counters[u.unit] = 0;  // re-arm for the next call
}

// Thread-block cluster barrier over every thread of every CTA in the cluster
// (release / acquire: shared-memory writes before it are visible to the
// cluster's reads after it).  All threads of each warp execute it together.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The float at `local` (this CTA's shared memory) in the shared memory of
// cluster CTA `rank`.
__device__ __forceinline__ float ld_cluster_f32(const float* local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

constexpr int kMaxClusterSplits = 16;  // the largest (non-portable) cluster the split CTAs of a unit may form

// The cluster form of the split merge: CTA `split` of a unit's cluster left its
// partial (acc[R][DH], m, l per row, layout [R][DH + 2]) at `cp` in its own
// shared memory, and every CTA of the cluster has passed a cluster barrier.
// Each CTA merges its slice of the unit's R * DH outputs, reading the partials
// of all n splits through distributed shared memory.  Every thread of the CTA
// (NT) takes part; the caller ends with a second cluster barrier, so no CTA
// leaves while another still reads its partial.
template <int R, int DH, int NT>
__device__ __forceinline__ void cluster_merge(const AttnArgs& a, const AttnUnit& u, int n, const float* cp, int tid,
                                              bool write) {
  constexpr int E = R * DH;
  constexpr size_t RS = DH + 2;
  const int ncta = (int)gridDim.x, per = (E + ncta - 1) / ncta, e0 = (int)blockIdx.x * per;
  for (int e = e0 + tid; e < min(E, e0 + per); e += NT) {
    const int r = e / DH, d = e % DH;
    float mv[kMaxClusterSplits], lv[kMaxClusterSplits], av[kMaxClusterSplits];
#pragma unroll
    for (int sp = 0; sp < kMaxClusterSplits; sp++) {
      if (sp < n) {
        mv[sp] = ld_cluster_f32(cp + r * RS + DH, sp);
        lv[sp] = ld_cluster_f32(cp + r * RS + DH + 1, sp);
        av[sp] = ld_cluster_f32(cp + r * RS + d, sp);
      }
    }
    float M = -1e30f;
#pragma unroll
    for (int sp = 0; sp < kMaxClusterSplits; sp++)
      if (sp < n) M = fmaxf(M, mv[sp]);
    float L = 0.f, A = 0.f;
#pragma unroll
    for (int sp = 0; sp < kMaxClusterSplits; sp++) {
      if (sp < n) {
        const float w = exp2f(mv[sp] - M);
        L = fmaf(lv[sp], w, L);
        A = fmaf(av[sp], w, A);
      }
    }
    if (write && r < u.rows_valid) store_out(a, out_index(a, u, r, d, DH), A / L);
  }
}

// Launches a decode kernel `kern(maps..., args)`.  With args.cluster set, the
// split CTAs of each unit (gridDim.x of them, at most kMaxClusterSplits) form
// one thread-block cluster; if the device cannot schedule such a cluster, the
// launch-configuration error is cleared and the kernel runs in its ticket form
// instead (the handle's workspace holds the partials either way).
template <typename... KArgs, typename... Maps>
void launch_decode(void (*kern)(KArgs...), dim3 grid, int threads, size_t smem, cudaStream_t stream, AttnArgs args,
                   const Maps&... maps) {
  if (args.cluster) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = dim3((unsigned)threads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = grid.x;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, maps..., args) == cudaSuccess) return;
    (void)cudaGetLastError();
    args.cluster = 0;
  }
  kern<<<grid, threads, smem, stream>>>(maps..., args);
}

// Host launcher of the tcgen05 kernel (attention_decode_tc.cu).  Returns
// HCU_EUNSUPPORTED when the shape has no tensor-core variant.
int launch_attn_tc(hcu_context* h, int fmt, int R, const AttnArgs& args, dim3 grid, const CUtensorMap& tk,
                   const CUtensorMap& tv);
bool attn_tc_supported(int fmt, int Dh, int R);
// Host launcher of the Q8_0 tcgen05 kernel (attention_decode_q8tc.cu): R <= 4.
int launch_attn_q8tc(hcu_context* h, int R, const AttnArgs& args, dim3 grid, const CUtensorMap& tk,
                     const CUtensorMap& tv, const CUtensorMap& tks, const CUtensorMap& tvs);
constexpr int kTcTile = 128;  // tokens per tcgen05 tile

}  // namespace hcu
