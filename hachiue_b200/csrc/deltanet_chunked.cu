// deltanet_chunked.cu - chunked (WY-form) Gated DeltaNet prefill on tcgen05.
//
// Same recurrence as deltanet_recur (src/kernels.ts:1496-1573, JS
// src/wasm-backend.ts:1047-1102), per V head h (QK head h % HK) and token t:
//   k^ = k / sqrt(|k|^2 + 1e-6),  q^ = q / sqrt(|q|^2 + 1e-6) / sqrt(D)
//   S <- exp(g) S;  delta = (v - S^T k^) beta;  S <- S + k^ delta^T;  o = S^T q^
// evaluated 64 tokens at a time.  With S0 the state entering a chunk,
// gamma the in-chunk cumulative sum of g, Gamma = exp(gamma), ik / iq the
// norm factors (iq includes 1/sqrt(D)) and K, Q, V the raw chunk rows:
//   A_ij  = beta_i ik_i ik_j exp(gamma_i - gamma_j) (k_i . k_j)    (j < i)
//   T     = (I + A)^-1,   Tb = T diag(beta)
//   QKm_ij = iq_i ik_j exp(gamma_i - gamma_j) (q_i . k_j)            (j <= i)
//   c2 = Gamma ik,  c3 = Gamma iq,  c4 = ik exp(gamma_63 - gamma),  e = exp(gamma_63)
//   R'    = V - diag(c2) K S0                     (then Delta = Tb R')
//   O     = diag(c3) Q S0 + (QKm Tb) R'
//   S1    = e S0 + K^T diag(c4) Tb R'
//
// Two kernels per slab of chunks:
//   gdn_prep_kernel  - everything that does not depend on the state, for all
//     chunks of the slab in parallel: one CTA per (sequence, QK head, chunk)
//     computes [K;Q][K;Q]^T on the tensor cores once and, per V head that
//     reads this QK head (one 128-thread warpgroup each), the norms, decays,
//     A, T (16x16 blocks by substitution on the CUDA cores, combined to 32x32
//     there and to 64x64 on the tf32 tensor cores), QKm, and writes the
//     chunk's operand  W = [Tb ; QKm Tb]  (128 x 64 bf16, the second half a
//     tf32 tensor-core product) and the scalars c2, c3, c4, e to a scratch
//     buffer.
//   gdn_chain_kernel - the state recurrence: one CTA per (sequence, V head)
//     walks the chunks in order with three MMAs per chunk,
//     [X; QS] = [K; Q] S0,  [Tb R'; O] = [0; c3 QS] + W R',  S1 = e S0 + K^T Dsb
//     (Dsb = c4 Tb R'), keeping the f32 state in TMEM (MMA (e) accumulates
//     onto e S0) and its bf16 copy in shared memory as the next chunk's MMA
//     operand.  Two CTAs fit per SM, so a batch of up to 296 (sequence, V
//     head) pairs is one wave.
//   gdn_chain_split_kernel - the same recurrence with two CTAs per (sequence,
//     V head), 64 value columns each, the f32 state in registers (one state
//     row per thread).  Each CTA's chunk is shorter, so batches whose
//     2 x (sequence, V head) CTAs still fit one wave (at most 148 pairs) take
//     this kernel.
#include <stdlib.h>

#include "common.cuh"
#include "context.h"
#include "tcgen05.cuh"

namespace hcu {
namespace {

constexpr int GC = 64;   // chunk length
constexpr int GD = 128;  // DK = DV
// scratch per (sequence, V head, chunk) unit
constexpr int W_ELEMS = 128 * 64;  // bf16 operand W = [Tb; QKm Tb]
constexpr int SC_FLOATS = 4 * 64;  // c2, c3, c4, e (e repeated)
constexpr size_t UNIT_BYTES = W_ELEMS * 2 + SC_FLOATS * 4;

// ---------------- prep kernel layout ----------------
// The CUDA-core phases keep A and T in plain padded f32 arrays; the tf32 MMAs
// of the 64x64 combine read small 128-byte-swizzled K-major copies (A21, U11,
// T22), whose M = 64 reads run over 32 neighbouring rows that are not used.
// TMEM: [K;Q][K;Q]^T in columns 0-127 (whose lanes 64-127 later hold
// warpgroup w's QKm in columns 64w..64w+63, the A operand of QKm Tb), then per
// warpgroup 64 columns for the combine products and QKm Tb.
constexpr int PREP_THREADS = 256;
constexpr int AS = 68;           // row stride (floats) of T
constexpr int AD = 36;           // row stride (floats) of A's diagonal 32x32 blocks
constexpr int P_OFF_KQ = 0;      // K / Q chunk (32 KB); after (f) warpgroup w owns bytes [16w, 16w + 16) KB:
constexpr int P_KQ_U11 = 0;      //   U11 = T[0:32][0:32]^T, 32 swizzled rows
constexpr int P_KQ_X2T = 4096;   //   X2^T, 32 swizzled rows
constexpr int P_KQ_X1 = 8192;    //   X1 [2][16][20]
                                 //   and, once those are read, W = [Tb; QKm Tb] bf16 (128 swizzled rows)
constexpr int P_OFF_WG = 32768;  // per warpgroup:
constexpr int P_WG_A21 = 0;      //   A[32:64][0:32], 32 swizzled rows
constexpr int P_WG_T22 = 4096;   //   T[32:64][32:64], 32 swizzled rows (A21's rows precede it)
constexpr int P_WG_T = 8192;     //   T [64][AS]; later Tb^T as two swizzled 64 x 32 halves
constexpr int P_WG_A = 25600;    //   A's diagonal 32x32 blocks [2][32][AD]
constexpr int P_WG_SC = 34816;   //   gam2, beta, ik, iq, w [64] + misc[16]
constexpr int P_WG_STRIDE = 36864;
constexpr int P_OFF_BAR = P_OFF_WG + 2 * P_WG_STRIDE;
constexpr int P_NBAR = 8;
constexpr int P_SMEM = P_OFF_BAR + P_NBAR * 8 + 16;
static_assert(P_WG_T + 64 * AS * 4 <= P_WG_A && P_WG_A + 2 * 32 * AD * 4 <= P_WG_SC, "prep warpgroup layout");
static_assert(P_WG_SC + (5 * 64 + 16) * 4 <= P_WG_STRIDE, "prep warpgroup region");
static_assert(P_KQ_X1 + 2 * 16 * 20 * 4 <= 16384, "prep K/Q reuse");

// ---------------- chain kernel layout ----------------
constexpr int CHAIN_THREADS = 192;
constexpr int C_OFF_KQ = 0;         // [d0: K | Q][d1: K | Q] bf16: the A operand of [K;Q] S0; its K rows
                                    // are the MN-major A operand of K^T Dsb
constexpr int C_OFF_W = 32768;      // W, 128 rows K-major; after MMA (c), output boxes 0-1 (below)
constexpr int C_OFF_V = 49152;      // V [2 x 64 values][64 tokens] bf16; then R' in place (MN-major B of
                                    // W R'), then Dsb in place (MN-major B of K^T Dsb)
constexpr int C_OFF_S0B = 65536;    // [2 x 64 dv][128 dk] bf16 state, MN-major B operand of [K;Q] S0;
                                    // between MMA (c) and the state update, its second half holds output
                                    // boxes 2-3.  The chunk's f32 outputs are four boxes of [64 tokens][32
                                    // values] (128B-swizzled) for TMA stores: boxes 0-1 in W's buffer, 2-3
                                    // here, so the state update writes its first half without waiting
constexpr int C_OFF_SC = 98304;     // [2][4][64] f32
constexpr int C_OFF_BAR = C_OFF_SC + 2 * SC_FLOATS * 4;
constexpr int C_NBAR = 18;
constexpr int C_SMEM = C_OFF_BAR + C_NBAR * 8 + 16;
// TMEM columns of the chain kernel: P = [X; QS], then [Tb R'; O]; S = the f32 state
constexpr uint32_t TC_P = 0, TC_S = 128, C_TMEM_COLS = 256;

// ---------------- split chain kernel layout (64 value columns per CTA) ----------------
constexpr int R_COLS = 64;
constexpr int R_OFF_KQ = 0;         // [d0: K | Q][d1: K | Q] bf16, A operand of [K;Q] S0
constexpr int R_OFF_KE = 32768;     // [d0: K][d1: K] bf16, A operand (MN-major) of K^T Dsb
constexpr int R_OFF_W = 49152;      // W, 128 rows K-major; after MMA (c) the chunk's f32 outputs
                                    // [64 tokens][2 x 32 values] (two 128B-swizzled halves) for a TMA store
constexpr int R_OFF_S0B = 65536;    // [128 dk][64 dv] bf16 state, MN-major B operand
constexpr int R_OFF_V = 81920;      // [64 tokens][64 values] bf16
constexpr int R_OFF_RB = 90112;     // R', MN-major B operand
constexpr int R_OFF_DSB = 98304;    // Dsb, MN-major B operand
constexpr int R_OFF_SC = 106496;    // [2][4][64] f32
constexpr int R_OFF_BAR = R_OFF_SC + 2 * SC_FLOATS * 4;
constexpr int R_NBAR = 18;
constexpr int R_SMEM = R_OFF_BAR + R_NBAR * 8 + 16;
// TMEM columns of the split chain kernel: P = [X; QS] and later U, Q = [Tb R'; O2]
constexpr uint32_t RT_P = 0, RT_Q = 64, R_TMEM_COLS = 128;

struct PrepArgs {
  int T, NK, NV, c0, ns, ahead;
  const float* g;
  const float* beta;
  long long gb_row, gb_seq;
  float* sc;  // [units][4][64]
  uint32_t* status;
};

struct ChainArgs {
  int T, NK, NV, c0, ns, cnt, load_state;
  const float* state_in;
  float* core;
  float* state_out;
  uint32_t* status;
  // state snapshots (prefix reuse): snapshot j = the state after token
  // 64 * snap_every * (j + 1), f32 [B][snap_count][NV][D][D]; null for none
  float* snap;
  int snap_every;
  long long snap_count;
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

__device__ __forceinline__ float fast_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// 8 consecutive f32 values as one 16-byte bf16 chunk.
__device__ __forceinline__ uint4 pack8(const float* x) {
  uint4 w;
  w.x = pack2(x[0], x[1]);
  w.y = pack2(x[2], x[3]);
  w.z = pack2(x[4], x[5]);
  w.w = pack2(x[6], x[7]);
  return w;
}

// Writes 64 f32 values as one 128-byte bf16 row of a 128B-swizzled region.
__device__ __forceinline__ void store_row64(uint8_t* region, int row, const float (&x)[64]) {
#pragma unroll
  for (int u = 0; u < 8; u++) *reinterpret_cast<uint4*>(region + sw128_offset(row, 16 * u)) = pack8(x + 8 * u);
}

// Writes 32 f32 values as half hc (bytes 64 hc .. 64 hc + 63) of two 128-byte
// bf16 rows of 128B-swizzled regions: hi = bf16(x) and lo = bf16(x - hi).
__device__ __forceinline__ void store_row32_hilo(uint8_t* hi, uint8_t* lo, int row, int hc, const float (&x)[32]) {
#pragma unroll
  for (int u = 0; u < 4; u++) {
    const uint4 h = pack8(x + 8 * u);
    uint4 l;
    l.x = pack2(x[8 * u + 0] - bf16_lo(h.x), x[8 * u + 1] - bf16_hi(h.x));
    l.y = pack2(x[8 * u + 2] - bf16_lo(h.y), x[8 * u + 3] - bf16_hi(h.y));
    l.z = pack2(x[8 * u + 4] - bf16_lo(h.z), x[8 * u + 5] - bf16_hi(h.z));
    l.w = pack2(x[8 * u + 6] - bf16_lo(h.w), x[8 * u + 7] - bf16_hi(h.w));
    *reinterpret_cast<uint4*>(hi + sw128_offset(row, 64 * hc + 16 * u)) = h;
    *reinterpret_cast<uint4*>(lo + sw128_offset(row, 64 * hc + 16 * u)) = l;
  }
}

// 64 TMEM columns of this thread's lane as f32.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&x)[64]) {
  uint32_t r0[32], r1[32];
  tmem_ld32(taddr, r0);
  tmem_ld32(taddr + 32, r1);
  tmem_ld_wait();
#pragma unroll
  for (int i = 0; i < 32; i++) {
    x[i] = __uint_as_float(r0[i]);
    x[32 + i] = __uint_as_float(r1[i]);
  }
}

// =====================================================================
// prep: state-independent operands of every chunk of the slab
// =====================================================================
__global__ void __launch_bounds__(PREP_THREADS, 2)
    gdn_prep_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmW, const PrepArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + P_OFF_BAR);
  uint64_t* bar_kq = bars + 0;   // K / Q chunk landed
  uint64_t* bar_f = bars + 1;    // [K;Q][K;Q]^T done
  uint64_t* bar_l3a = bars + 2;  // [2] U11 A21^T done
  uint64_t* bar_l3b = bars + 4;  // [2] T22 X2 done
  uint64_t* bar_g = bars + 6;    // [2] QKm Tb done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + P_NBAR);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x, b = blockIdx.z;
  const int hk = blockIdx.y % a.NK, pair = blockIdx.y / a.NK;
  const int t0 = (a.c0 + c) * GC;
  const int wg = warp >> 2, quad = warp & 3, t = quad * 32 + lane;
  const int h = hk + (2 * pair + wg) * a.NK;
  const bool active = h < a.NV;
  // g and beta of this thread's row (t < 64), requested before the set-up
  float gi = 0.f, bi = 0.f;
  if (active && t < 64 && t0 + t < a.T) {
    const size_t idx = (size_t)b * a.gb_seq + (size_t)(t0 + t) * a.gb_row + h;
    gi = __ldg(a.g + idx);
    bi = __ldg(a.beta + idx);
  }

  if (tid == 0) {
    for (int i = 0; i < P_NBAR; i++) mbar_init(&bars[i], 1);
    fence_barrier_init();
    // The K / Q chunk is requested first of all, before the TMEM allocation
    // and the block barrier (only this thread uses bar_kq before that barrier).
    mbar_arrive_expect_tx(bar_kq, 32768);
    tma_load_4d(sm + P_OFF_KQ, &tmK, bar_kq, 0, hk, t0, b);
    tma_load_4d(sm + P_OFF_KQ + 8192, &tmQ, bar_kq, 0, hk, t0, b);
    tma_load_4d(sm + P_OFF_KQ + 16384, &tmK, bar_kq, 64, hk, t0, b);
    tma_load_4d(sm + P_OFF_KQ + 24576, &tmQ, bar_kq, 64, hk, t0, b);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // One elected lane issues the MMAs; the whole warp waits and forms the
    // (warp-uniform) descriptors.
    const bool leader = elect_one_sync();
    // warm L2 with the K / Q chunk that the CTA one wave later (a.ahead
    // blocks further in launch order) will load
    if (leader) {
      prefetch_tensormap(&tmW);
      const long long lin = blockIdx.x + (long long)gridDim.x * (blockIdx.y + (long long)gridDim.y * blockIdx.z) +
                            a.ahead;
      const int cf = (int)(lin % gridDim.x), yf = (int)((lin / gridDim.x) % gridDim.y);
      const long long bf = lin / ((long long)gridDim.x * gridDim.y);
      if (bf < gridDim.z) {
        const int tf = (a.c0 + cf) * GC, hf = yf % a.NK;
        tma_prefetch_l2_4d(&tmK, 0, hf, tf, (int)bf);
        tma_prefetch_l2_4d(&tmQ, 0, hf, tf, (int)bf);
        tma_prefetch_l2_4d(&tmK, 64, hf, tf, (int)bf);
        tma_prefetch_l2_4d(&tmQ, 64, hf, tf, (int)bf);
      }
    }
    if (__all_sync(0xffffffffu, mbar_wait(bar_kq, 0, a.status))) {
      tc_fence_after();
      constexpr uint32_t id_f = idesc_f16(128, 128, true, false, false);
      const uint32_t kq = smem_u32(sm + P_OFF_KQ);
#pragma unroll
      for (int ks = 0; ks < 8; ks++) {
        const uint64_t d = smem_desc_sw128(kq + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024);
        if (leader) mma_f16_ss(tmem, d, d, id_f, ks > 0);
      }
      if (leader) mma_commit(bar_f);
    }
  }

  {
    uint8_t* wreg = sm + P_OFF_WG + wg * P_WG_STRIDE;
    uint8_t* kqh = sm + P_OFF_KQ + wg * 16384;  // this warpgroup's half of the K/Q buffer, after (f)
    float* A21 = reinterpret_cast<float*>(wreg + P_WG_A21);
    float* T22 = reinterpret_cast<float*>(wreg + P_WG_T22);
    float* Tf = reinterpret_cast<float*>(wreg + P_WG_T);
    float* Ad = reinterpret_cast<float*>(wreg + P_WG_A);
    float* gam2 = reinterpret_cast<float*>(wreg + P_WG_SC);  // gamma * log2(e)
    float* betv = gam2 + 64;
    float* ikv = gam2 + 128;
    float* iqv = gam2 + 192;
    float* wv = gam2 + 256;  // gam2_j - log2(ik_j)
    float* misc = gam2 + 320;
    float* U11 = reinterpret_cast<float*>(kqh + P_KQ_U11);
    float* X2T = reinterpret_cast<float*>(kqh + P_KQ_X2T);
    float* X1 = reinterpret_cast<float*>(kqh + P_KQ_X1);
    uint8_t* wst = kqh;  // W staging
    const uint32_t lo = (uint32_t)(quad * 32) << 16;
    const uint32_t tl3 = tmem + 128 + 64 * wg;  // 64x64 combine products, later QKm Tb
    const uint32_t bid = 1 + wg;
    const size_t unit = ((size_t)b * a.NV + h) * a.ns + c;

    bool ok = active && named_bar_and(bid, 128, mbar_wait(bar_f, 0, a.status));
    float nrm2 = 0.f, f[64];  // f: G row t (t < 64) or P row t - 64: k_t . k_j / q_i . k_j
    if (ok) {
      tc_fence_after();
      // |k_t|^2 (t < 64) or |q_{t-64}|^2: the diagonal of [K;Q][K;Q]^T, column t
      uint32_t r[32];
      tmem_ld32(tmem + lo + quad * 32, r);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 32; j++) nrm2 = j == lane ? __uint_as_float(r[j]) : nrm2;
      tmem_ld64(tmem + lo, f);
    }
    // both warpgroups have read [K;Q][K;Q]^T before its columns take QKm
    tc_fence_before();
    named_bar(3, PREP_THREADS);
    if (ok) {
      tc_fence_after();
      float sc = gi;
      if (t < 64) {
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_up_sync(0xffffffffu, sc, o);
          if (lane >= o) sc += y;
        }
        if (t == 31) misc[0] = sc;
      }
      named_bar(bid, 128);
      if (t < 64) {
        const float g2 = (sc + (t >= 32 ? misc[0] : 0.f)) * kLog2e;
        const float ik = rsqrtf(nrm2 + 1e-6f);
        gam2[t] = g2;
        betv[t] = bi;
        ikv[t] = ik;
        wv[t] = g2 - __log2f(ik);
      } else {
        iqv[t - 64] = rsqrtf(nrm2 + 1e-6f) * rsqrtf((float)GD);
      }
      named_bar(bid, 128);
      // A_tj = 2^(z_t - w_j) f_j with z_t = gam2_t + log2(beta_t ik_t); QKm likewise
      // with z_i = gam2_i + log2(iq_i).  Entries outside the triangle are selected
      // away (their exponent may overflow).  All values are rounded to tf32.
      if (t < 64) {
        const float z = gam2[t] + __log2f(betv[t] * ikv[t]);
        const int r = t & 31;
        auto a4 = [&](int u) {
          const float4 w4 = reinterpret_cast<const float4*>(wv)[u];
          const int j = 4 * u;
          float4 o;
          o.x = j + 0 < t ? tf32_round(fast_ex2(z - w4.x) * f[j + 0]) : 0.f;
          o.y = j + 1 < t ? tf32_round(fast_ex2(z - w4.y) * f[j + 1]) : 0.f;
          o.z = j + 2 < t ? tf32_round(fast_ex2(z - w4.z) * f[j + 2]) : 0.f;
          o.w = j + 3 < t ? tf32_round(fast_ex2(z - w4.w) * f[j + 3]) : 0.f;
          return o;
        };
        if (quad == 0) {
#pragma unroll
          for (int u = 0; u < 8; u++) *reinterpret_cast<float4*>(Ad + r * AD + 4 * u) = a4(u);
        } else {
#pragma unroll
          for (int u = 0; u < 8; u++) *reinterpret_cast<float4*>(A21 + r * 32 + ((u ^ (r & 7)) << 2)) = a4(u);
#pragma unroll
          for (int u = 8; u < 16; u++) *reinterpret_cast<float4*>(Ad + 32 * AD + r * AD + 4 * (u - 8)) = a4(u);
        }
      } else {
        const int i = t - 64;
        const float z = gam2[i] + __log2f(iqv[i]);
        // QKm row i, the A operand of QKm Tb from TMEM lane 64 + i, as two bf16
        // terms: hi = bf16(x) in columns 64w..64w+31 and lo = bf16(x - hi) in the
        // next 32 (two elements per column, the even one in the low half);
        // 32 elements at a time
#pragma unroll
        for (int hh = 0; hh < 2; hh++) {
          uint32_t rh[16], rl[16];
#pragma unroll
          for (int u = 0; u < 8; u++) {
            const float4 w4 = reinterpret_cast<const float4*>(wv)[8 * hh + u];
            const int j = 32 * hh + 4 * u;
            const bool live = hh == 0 || quad == 3;
            const float y0 = live && j + 0 <= i ? fast_ex2(z - w4.x) * f[j + 0] : 0.f;
            const float y1 = live && j + 1 <= i ? fast_ex2(z - w4.y) * f[j + 1] : 0.f;
            const float y2 = live && j + 2 <= i ? fast_ex2(z - w4.z) * f[j + 2] : 0.f;
            const float y3 = live && j + 3 <= i ? fast_ex2(z - w4.w) * f[j + 3] : 0.f;
            rh[2 * u] = pack2(y0, y1);
            rh[2 * u + 1] = pack2(y2, y3);
            rl[2 * u] = pack2(y0 - bf16_lo(rh[2 * u]), y1 - bf16_hi(rh[2 * u]));
            rl[2 * u + 1] = pack2(y2 - bf16_lo(rh[2 * u + 1]), y3 - bf16_hi(rh[2 * u + 1]));
          }
          tmem_st16(tmem + lo + 64 * wg + 16 * hh, rh);
          tmem_st16(tmem + lo + 64 * wg + 32 + 16 * hh, rl);
        }
        tmem_st_wait();
        tc_fence_before();
      }
      named_bar(bid, 128);
      // (I + A)^-1: 16x16 diagonal blocks by forward substitution, thread cc of
      // a block computing its column
      if (t < 64) {
        const int base = (t >> 4) * 16, cc = t & 15;
        const float* ab = Ad + (base >> 5) * 32 * AD + (base & 31) * (AD + 1);  // A(base, base)
        float tc[16];
#pragma unroll
        for (int r = 0; r < 16; r++) {
          float s = 0.f;
#pragma unroll
          for (int j = 0; j < r; j++) s = fmaf(ab[r * AD + j], tc[j], s);
          tc[r] = tf32_round(r == cc ? 1.f : -s);
        }
#pragma unroll
        for (int r = 0; r < 16; r++) Tf[(base + r) * AS + base + cc] = tc[r];
        // the swizzled K-major operands of the 64x64 combine: U11 = T[0:32][0:32]^T
        // (column cc is U11's row base + cc) and T22 = T[32:64][32:64]
        if (base < 32) {
          const int j = base + cc;
#pragma unroll
          for (int u = 0; u < 4; u++)
            *reinterpret_cast<float4*>(U11 + j * 32 + ((((base >> 2) + u) ^ (j & 7)) << 2)) =
                make_float4(tc[4 * u], tc[4 * u + 1], tc[4 * u + 2], tc[4 * u + 3]);
        } else {
          const int b2 = base - 32, col = b2 + cc;
#pragma unroll
          for (int r = 0; r < 16; r++) {
            const int m = b2 + r;
            T22[m * 32 + (((col >> 2) ^ (m & 7)) << 2) + (col & 3)] = tc[r];
          }
        }
      } else {
        // zero the upper off-diagonal 16x16 blocks (0,1) and (2,3), in T and in
        // the combine operands (the 32x32 diagonal blocks are read whole below),
        // and T's upper 32x32 block, so that T's rows read whole
        for (int e = t - 64; e < 512; e += 64) {
          const int blk = e >> 8, r = (e >> 4) & 15, cc = e & 15;
          Tf[(blk * 32 + r) * AS + blk * 32 + 16 + cc] = 0.f;
          if (blk == 0) {
            const int j = 16 + cc;  // U11[16 + cc][r] = T[r][16 + cc]
            U11[j * 32 + (((r >> 2) ^ (j & 7)) << 2) + (r & 3)] = 0.f;
          } else {
            const int col = 16 + cc;  // T22[r][16 + cc]
            T22[r * 32 + (((col >> 2) ^ (r & 7)) << 2) + (col & 3)] = 0.f;
          }
        }
#pragma unroll
        for (int e = t - 64; e < 256; e += 64)
          *reinterpret_cast<float4*>(&Tf[(e >> 3) * AS + 32 + 4 * (e & 7)]) = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      named_bar(bid, 128);
      {
        // 32x32 blocks: T[2p+1][2p] = -T[2p+1][2p+1] A[2p+1][2p] T[2p][2p]
        const int p = t >> 6, rem = t & 63, r = rem >> 2, c4 = (rem & 3) * 4;
        const int rb = 16 * (2 * p + 1), cb = 16 * (2 * p);
        const float* arow = Ad + p * 32 * AD + (16 + r) * AD;  // A(rb + r, cb + k) = arow[k]
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int k = 0; k < 16; k++) {
          const float av = arow[k];
          const float4 tv = *reinterpret_cast<const float4*>(&Tf[(cb + k) * AS + cb + c4]);
          acc.x = fmaf(av, tv.x, acc.x);
          acc.y = fmaf(av, tv.y, acc.y);
          acc.z = fmaf(av, tv.z, acc.z);
          acc.w = fmaf(av, tv.w, acc.w);
        }
        *reinterpret_cast<float4*>(&X1[(p * 16 + r) * 20 + c4]) = acc;
        named_bar(bid, 128);
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int k = 0; k < 16; k++) {
          const float tv = Tf[(rb + r) * AS + rb + k];
          const float4 xv = *reinterpret_cast<const float4*>(&X1[(p * 16 + k) * 20 + c4]);
          o.x = fmaf(tv, xv.x, o.x);
          o.y = fmaf(tv, xv.y, o.y);
          o.z = fmaf(tv, xv.z, o.z);
          o.w = fmaf(tv, xv.w, o.w);
        }
        const float4 v = make_float4(tf32_round(-o.x), tf32_round(-o.y), tf32_round(-o.z), tf32_round(-o.w));
        *reinterpret_cast<float4*>(&Tf[(rb + r) * AS + cb + c4]) = v;
        if (p == 0) {
          // U11[c4 + e][16 + r] = T[16 + r][c4 + e]
          const int col = 16 + r;
#pragma unroll
          for (int e = 0; e < 4; e++) {
            const int j = c4 + e;
            U11[j * 32 + (((col >> 2) ^ (j & 7)) << 2) + (col & 3)] = (&v.x)[e];
          }
        } else {
          // T22[16 + r][c4 .. c4 + 3]
          const int m = 16 + r;
          *reinterpret_cast<float4*>(T22 + m * 32 + (((c4 >> 2) ^ (m & 7)) << 2)) = v;
        }
      }
      // 64x64 on the tensor cores (tf32, K-major operands):
      //   X2^T = U11 A[32:64][0:32]^T,  then  T[32:64][0:32] = -T[32:64][32:64] X2.
      fence_proxy_async();
      named_bar(bid, 128);
      constexpr uint32_t id_l3 = idesc_tf32(64, 32, false, false);
      if (quad == 0) {
        const bool leader = elect_one_sync();
        tc_fence_after();
        const uint32_t ub = smem_u32(U11), ab = smem_u32(A21);
#pragma unroll
        for (int ks = 0; ks < 4; ks++) {
          const uint64_t ad = smem_desc_sw128(ub + ks * 32, 16, 1024), bd = smem_desc_sw128(ab + ks * 32, 16, 1024);
          if (leader) mma_tf32_ss(tl3, ad, bd, id_l3, ks > 0);
        }
        if (leader) mma_commit(&bar_l3a[wg]);
      }
      ok = __all_sync(0xffffffffu, mbar_wait(&bar_l3a[wg], 0, a.status));
      if (ok && quad < 2) {
        tc_fence_after();
        uint32_t r[32];
        tmem_ld32(tl3 + lo, r);  // M = 64 rows 0-31 (X2^T): lanes 0-15 of quadrants 0, 1
        tmem_ld_wait();
        if (lane < 16) {
          const int j = 16 * quad + lane;
#pragma unroll
          for (int u = 0; u < 8; u++)
            *reinterpret_cast<float4*>(X2T + j * 32 + ((u ^ (j & 7)) << 2)) =
                make_float4(tf32_round(__uint_as_float(r[4 * u])), tf32_round(__uint_as_float(r[4 * u + 1])),
                            tf32_round(__uint_as_float(r[4 * u + 2])), tf32_round(__uint_as_float(r[4 * u + 3])));
        }
      }
      fence_proxy_async();
      tc_fence_before();
      ok = named_bar_and(bid, 128, ok);
      if (ok && quad == 0) {
        const bool leader = elect_one_sync();
        tc_fence_after();
        // A operand rows 32-63 are T22's; rows 0-31 read A21 and are not used
        const uint32_t tb = smem_u32(A21), xb = smem_u32(X2T);
#pragma unroll
        for (int ks = 0; ks < 4; ks++) {
          const uint64_t ad = smem_desc_sw128(tb + ks * 32, 16, 1024), bd = smem_desc_sw128(xb + ks * 32, 16, 1024);
          if (leader) mma_tf32_ss(tl3 + 32, ad, bd, id_l3, ks > 0);
        }
        if (leader) mma_commit(&bar_l3b[wg]);
      }
      if (ok && quad >= 2) {
        ok = __all_sync(0xffffffffu, mbar_wait(&bar_l3b[wg], 0, a.status));
        if (ok) {
          tc_fence_after();
          uint32_t r[32];
          tmem_ld32(tl3 + 32 + lo, r);  // rows 32-63: lanes 0-15 of quadrants 2, 3
          tmem_ld_wait();
          if (lane < 16) {
            const int m = 32 + 16 * (quad - 2) + lane;
#pragma unroll
            for (int u = 0; u < 8; u++)
              *reinterpret_cast<float4*>(&Tf[m * AS + 4 * u]) =
                  make_float4(-__uint_as_float(r[4 * u]), -__uint_as_float(r[4 * u + 1]),
                              -__uint_as_float(r[4 * u + 2]), -__uint_as_float(r[4 * u + 3]));
          }
        }
      }
      tc_fence_before();
      ok = named_bar_and(bid, 128, ok);
      // Tb = T diag(beta): row t is W row t.  As two bf16 terms (hi = W row t,
      // lo = the rounding residual in W's rows 64-127 until QKm Tb is done) it is
      // the MN-major B operand of QKm Tb.
      // Threads t and t + 64 take the two 32-column halves of row t % 64 (T's row:
      // unit diagonal, zeros or -0 above it) and two of its four scalars each.
      if (ok) {
        const int row = t & 63, hc = t >> 6;
        float yh[32];
#pragma unroll
        for (int u = 0; u < 8; u++) {
          const float4 v4 = *reinterpret_cast<const float4*>(&Tf[row * AS + 32 * hc + 4 * u]);
          const float4 b4 = reinterpret_cast<const float4*>(betv)[8 * hc + u];
          yh[4 * u] = v4.x * b4.x;
          yh[4 * u + 1] = v4.y * b4.y;
          yh[4 * u + 2] = v4.z * b4.z;
          yh[4 * u + 3] = v4.w * b4.w;
        }
        store_row32_hilo(wst, wst + 8192, row, hc, yh);
        float* scu = a.sc + unit * SC_FLOATS;
        if (hc == 0) {
          const float G = fast_ex2(gam2[row]);
          scu[row] = G * ikv[row];
          scu[64 + row] = G * iqv[row];
        } else {
          scu[128 + row] = ikv[row] * fast_ex2(gam2[63] - gam2[row]);
          scu[192 + row] = fast_ex2(gam2[63]);
        }
      }
      fence_proxy_async();
      tc_fence_before();
      ok = named_bar_and(bid, 128, ok);
      // W's rows 0-63 (Tb) are final: they go out now, read alongside QKm Tb
      if (ok && t == 0) {
        tma_store_2d(&tmW, wst, 0, (int)(unit * 128));
        tma_store_commit();
      }
      if (ok && quad == 0) {
        // QKm Tb = QKm_hi Tb_hi + QKm_hi Tb_lo + QKm_lo Tb_hi (M = 128: rows 64-127
        // are QKm's, from TMEM lanes 64-127; rows 0-63 read lanes 0-63 of the same
        // columns and are not used)
        const bool leader = elect_one_sync();
        tc_fence_after();
        constexpr uint32_t id_g = idesc_f16(128, 64, true, false, true);  // bf16, A from TMEM, B MN-major
        const uint32_t wb = smem_u32(wst);
        const uint32_t qh = tmem + 64 * wg, ql = qh + 32;
#pragma unroll
        for (int ks = 0; ks < 4; ks++) {
          const uint64_t bh = smem_desc_sw128(wb + ks * 2048, 8192, 1024);
          const uint64_t bl = smem_desc_sw128(wb + 8192 + ks * 2048, 8192, 1024);
          if (leader) {
            mma_f16_ts(tl3, qh + 8 * ks, bh, id_g, ks > 0);
            mma_f16_ts(tl3, qh + 8 * ks, bl, id_g, 1);
            mma_f16_ts(tl3, ql + 8 * ks, bh, id_g, 1);
          }
        }
        if (leader) mma_commit(&bar_g[wg]);
      }
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&bar_g[wg], 0, a.status));
      if (ok && quad >= 2) {
        float y[64];
        tc_fence_after();
        tmem_ld64(tl3 + lo, y);
        store_row64(wst, t, y);  // W row 64 + i = (QKm Tb) row i
        fence_proxy_async();
      }
      ok = named_bar_and(bid, 128, ok);
      if (ok && t == 0) {
        tma_store_2d(&tmW, wst + 8192, 0, (int)(unit * 128 + 64));
        tma_store_commit_and_wait_read();
      }
    }
  }
  // A timed-out wait can skip the final store: W's early store must still have
  // read shared memory before the CTA exits.
  if (t == 0) tma_store_wait_read();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) {
    __syncwarp();
    tmem_dealloc(tmem, 256);
  }
}

// =====================================================================
// chain: the state recurrence over the chunks of a slab
// =====================================================================
__global__ void __launch_bounds__(CHAIN_THREADS, 2)
    gdn_chain_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmW,
                     const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmO,
                     const ChainArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + C_OFF_BAR);
  uint64_t* kq_full = bars + 0;
  uint64_t* q_free = bars + 1;    // MMA (a) done: the Q rows may be refilled
  uint64_t* kv_free = bars + 2;   // MMA (e) done: the K rows and V's buffer may be refilled
  uint64_t* v_full = bars + 3;
  uint64_t* w_full = bars + 4;
  uint64_t* w_free = bars + 5;    // MMA (c) done
  uint64_t* o_ready = bars + 6;   // the chunk's outputs staged in the state buffer
  uint64_t* s0_free = bars + 7;   // those outputs stored: the state buffer may be rewritten
  uint64_t* sc_full = bars + 8;   // [2]
  uint64_t* sc_empty = bars + 10; // [2] the chunk's scalars no longer read
  uint64_t* bar_a = bars + 12;    // [X; QS] in TMEM
  uint64_t* bar_R = bars + 13;    // R' in shared memory, X zeroed and QS scaled in TMEM
  uint64_t* bar_c = bars + 14;    // [Tb R'; O] in TMEM
  uint64_t* bar_D = bars + 15;    // Dsb in shared memory and [Tb R'; O] read
  uint64_t* bar_e = bars + 16;    // the new state in TMEM
  uint64_t* bar_s0 = bars + 17;   // bf16 state written, e S in TMEM
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C_NBAR);
  float* scal = reinterpret_cast<float*>(sm + C_OFF_SC);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Grid (V heads per QK head, QK heads, sequences): the CTAs of one QK head's
  // V heads h = hk, hk + NK, ... are adjacent, so they run together and share
  // each chunk's K / Q tiles in L2.
  const int hk = blockIdx.y, b = blockIdx.z;
  const int h = hk + (int)blockIdx.x * a.NK;
  if (h >= a.NV) return;  // the whole CTA, before any barrier or allocation
  const int n = a.cnt;
  const size_t unit0 = ((size_t)b * a.NV + h) * a.ns;

  if (tid == 0) {
    mbar_init(kq_full, 1);
    mbar_init(q_free, 1);
    mbar_init(kv_free, 1);
    mbar_init(v_full, 1);
    mbar_init(w_full, 1);
    mbar_init(w_free, 1);
    mbar_init(o_ready, 2);
    mbar_init(s0_free, 1);
    for (int i = 0; i < 2; i++) {
      mbar_init(&sc_full[i], 1);
      mbar_init(&sc_empty[i], 4);
    }
    mbar_init(bar_a, 1);
    mbar_init(bar_R, 4);
    mbar_init(bar_c, 1);
    mbar_init(bar_D, 4);
    mbar_init(bar_e, 1);
    mbar_init(bar_s0, 4);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_tensormap(&tmK);
      prefetch_tensormap(&tmQ);
      prefetch_tensormap(&tmV);
      prefetch_tensormap(&tmW);
      prefetch_tensormap(&tmS);
      prefetch_tensormap(&tmO);
      // a chunk's outputs: boxes 2-3 (state buffer) as one store group, then
      // boxes 0-1 (W's buffer) as another
      auto store_outputs = [&](int tj) {
        tma_store_4d(&tmO, sm + C_OFF_S0B + 16384, 64, h, tj, b);
        tma_store_4d(&tmO, sm + C_OFF_S0B + 24576, 96, h, tj, b);
        tma_store_commit();
        tma_store_4d(&tmO, sm + C_OFF_W, 0, h, tj, b);
        tma_store_4d(&tmO, sm + C_OFF_W + 8192, 32, h, tj, b);
        tma_store_commit();
      };
      // chunk 0's scalars: the state set-up reads its e
      mbar_arrive_expect_tx(&sc_full[0], SC_FLOATS * 4);
      tma_load_2d(scal, &tmS, &sc_full[0], 0, (int)unit0 * 4);
      int c = 0;
      for (; c < n; c++) {
        const int t0 = (a.c0 + c) * GC;
        const int u = (int)(unit0 + c);
        const uint32_t pe = (c - 1) & 1;
        if (c + 1 < n) {
          // warm L2 with the next chunk's tiles: its loads below are issued only
          // when this chunk frees the buffers, a chunk's time before they are needed
          const int t1 = t0 + GC;
          tma_prefetch_l2_4d(&tmK, 0, hk, t1, b);
          tma_prefetch_l2_4d(&tmK, 64, hk, t1, b);
          tma_prefetch_l2_4d(&tmQ, 0, hk, t1, b);
          tma_prefetch_l2_4d(&tmQ, 64, hk, t1, b);
          tma_prefetch_l2_4d(&tmV, 0, h, t1, b);
          tma_prefetch_l2_4d(&tmV, 64, h, t1, b);
          tma_prefetch_l2_2d(&tmW, 0, (u + 1) * 128);
        }
        // Q rows as soon as the previous chunk's MMA (a) is done
        if (c >= 1 && !mbar_wait(q_free, pe, a.status)) break;
        mbar_arrive_expect_tx(kq_full, 32768);
        tma_load_4d(sm + C_OFF_KQ + 8192, &tmQ, kq_full, 0, hk, t0, b);
        tma_load_4d(sm + C_OFF_KQ + 24576, &tmQ, kq_full, 64, hk, t0, b);
        // the previous chunk's outputs, staged in W's buffer and the state buffer
        if (c >= 1) {
          if (!mbar_wait(o_ready, pe, a.status)) break;
          store_outputs(t0 - GC);
        }
        // K rows and V once the previous chunk's MMA (e) is done
        if (c >= 1 && !mbar_wait(kv_free, pe, a.status)) break;
        tma_load_4d(sm + C_OFF_KQ, &tmK, kq_full, 0, hk, t0, b);
        tma_load_4d(sm + C_OFF_KQ + 16384, &tmK, kq_full, 64, hk, t0, b);
        mbar_arrive_expect_tx(v_full, 16384);
        tma_load_4d(sm + C_OFF_V, &tmV, v_full, 0, h, t0, b);
        tma_load_4d(sm + C_OFF_V + 8192, &tmV, v_full, 64, h, t0, b);
        if (c >= 1) {
          tma_store_wait_read_all_but_last();  // the state buffer's half is read
          mbar_arrive(s0_free);
          tma_store_wait_read();  // and W's buffer
        }
        // W once the previous chunk's MMA (c) is done and its outputs left W's buffer
        if (c >= 1 && !mbar_wait(w_free, pe, a.status)) break;
        mbar_arrive_expect_tx(w_full, W_ELEMS * 2);
        tma_load_2d(sm + C_OFF_W, &tmW, w_full, 0, u * 128);
        // the next chunk's scalars, into the buffer chunk c - 1 used
        if (c + 1 < n) {
          const int nb = (c + 1) & 1;
          if (c >= 1 && !mbar_wait(&sc_empty[nb], ((c - 1) >> 1) & 1, a.status)) break;
          mbar_arrive_expect_tx(&sc_full[nb], SC_FLOATS * 4);
          tma_load_2d(scal + nb * SC_FLOATS, &tmS, &sc_full[nb], 0, (u + 1) * 4);
        }
      }
      if (c == n && n > 0 && mbar_wait(o_ready, (n - 1) & 1, a.status)) store_outputs((a.c0 + n - 1) * GC);
      tma_store_wait_all();
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    // The whole warp walks the loop (its values are warp-uniform); one
    // elected lane issues each tcgen05 instruction.
    {
      const bool leader = elect_one_sync();
      constexpr uint32_t id_k = idesc_f16(128, 128, true, false, true);  // K-major A, MN-major B
      constexpr uint32_t id_e = idesc_f16(128, 128, true, true, true);   // MN-major A (K^T)
      const uint32_t s0 = smem_u32(sm);
      for (int c = 0; c < n; c++) {
        const uint32_t ph = c & 1;
        // (a) [X; QS] = [K; Q] S0   (M = 128, N = 128, K = 128)
        if (!__all_sync(0xffffffffu, mbar_wait(kq_full, ph, a.status) && mbar_wait(bar_s0, ph, a.status))) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 8; ks++) {
          const uint64_t ad = smem_desc_sw128(s0 + C_OFF_KQ + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024);
          const uint64_t bd = smem_desc_sw128(s0 + C_OFF_S0B + ks * 2048, 16384, 1024);
          if (leader) mma_f16_ss(tmem + TC_P, ad, bd, id_k, ks > 0);
        }
        if (leader) {
          mma_commit(bar_a);
          mma_commit(q_free);
        }
        // (c) [Tb R'; O] += W R'   (M = 128, N = 128, K = 64), onto [0; c3 QS]
        if (!__all_sync(0xffffffffu, mbar_wait(bar_R, ph, a.status) && mbar_wait(w_full, ph, a.status))) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 4; ks++) {
          const uint64_t ad = smem_desc_sw128(s0 + C_OFF_W + ks * 32, 16, 1024);
          const uint64_t bd = smem_desc_sw128(s0 + C_OFF_V + ks * 2048, 8192, 1024);
          if (leader) mma_f16_ss(tmem + TC_P, ad, bd, id_k, 1);
        }
        if (leader) {
          mma_commit(bar_c);
          mma_commit(w_free);
        }
        // (e) S += K^T Dsb   (M = 128, N = 128, K = 64), onto e S
        if (!__all_sync(0xffffffffu, mbar_wait(bar_D, ph, a.status))) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 4; ks++) {
          const uint64_t ad = smem_desc_sw128(s0 + C_OFF_KQ + ks * 2048, 16384, 1024);
          const uint64_t bd = smem_desc_sw128(s0 + C_OFF_V + ks * 2048, 8192, 1024);
          if (leader) mma_f16_ss(tmem + TC_S, ad, bd, id_e, 1);
        }
        if (leader) {
          mma_commit(bar_e);
          mma_commit(kv_free);
        }
      }
    }
  } else {
    // ---------------- chain warps 2-5: TMEM lane quadrant = warp % 4 ----------------
    const int quad = warp & 3;
    const int t = quad * 32 + lane;  // state row (dk); row of [K; Q] / W results
    const uint32_t lo = (uint32_t)(quad * 32) << 16;
    const uint32_t tp = tmem + lo + TC_P, tsr = tmem + lo + TC_S;
    uint8_t* s0b = sm + C_OFF_S0B;
    uint8_t* vb = sm + C_OFF_V;
    const size_t row = ((size_t)b * a.NV + h) * GD + t;  // this thread's state row in [B][NV][D][D]
    // the state entering the slab: its bf16 copy for MMA (a), e_0 S for MMA (e)
    bool ok = __all_sync(0xffffffffu, mbar_wait(&sc_full[0], 0, a.status));
    if (ok) {
      const float e0 = scal[192];
      const float4* src = a.load_state ? reinterpret_cast<const float4*>(a.state_in + row * GD) : nullptr;
#pragma unroll
      for (int hf = 0; hf < 4; hf++) {
        float x[32];
#pragma unroll
        for (int i = 0; i < 8; i++) {
          const float4 v = src ? __ldg(src + 8 * hf + i) : make_float4(0.f, 0.f, 0.f, 0.f);
          x[4 * i] = v.x;
          x[4 * i + 1] = v.y;
          x[4 * i + 2] = v.z;
          x[4 * i + 3] = v.w;
        }
        uint32_t r[32];
#pragma unroll
        for (int u = 0; u < 4; u++)
          *reinterpret_cast<uint4*>(s0b + (hf >> 1) * 16384 + sw128_offset(t, 64 * (hf & 1) + 16 * u)) =
              pack8(x + 8 * u);
#pragma unroll
        for (int j = 0; j < 32; j++) r[j] = __float_as_uint(e0 * x[j]);
        tmem_st32(tsr + 32 * hf, r);
      }
      tmem_st_wait();
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_s0);
    }
    for (int c = 0; c < n && ok; c++) {
      const uint32_t ph = c & 1;
      const float* sc = scal + (c & 1) * SC_FLOATS;
      if (quad < 2) {
        // R'_t = V_t - c2_t X_t (token t), in place of V; X zeroed so that
        // MMA (c) leaves Tb R' in its rows
        ok = __all_sync(0xffffffffu,
                        mbar_wait(v_full, ph, a.status) && mbar_wait(&sc_full[c & 1], (c >> 1) & 1, a.status));
        if (!ok) break;
        const float c2 = sc[t];
        uint4 vrow[16];
#pragma unroll
        for (int u = 0; u < 16; u++)
          vrow[u] = *reinterpret_cast<const uint4*>(vb + (u >> 3) * 8192 + sw128_offset(t, 16 * (u & 7)));
        ok = __all_sync(0xffffffffu, mbar_wait(bar_a, ph, a.status));
        if (!ok) break;
        tc_fence_after();
        uint32_t zero[32];
#pragma unroll
        for (int j = 0; j < 32; j++) zero[j] = 0u;
#pragma unroll
        for (int hf = 0; hf < 4; hf++) {
          uint32_t xr[32];
          tmem_ld32(tp + 32 * hf, xr);
          tmem_ld_wait();
#pragma unroll
          for (int u = 0; u < 4; u++) {
            const int vu = 4 * hf + u;  // 16-byte chunk of the row: 64-value block vu / 8, chunk vu % 8
            const uint4 vw = vrow[vu];
            const uint32_t vs[4] = {vw.x, vw.y, vw.z, vw.w};
            float r[8];
#pragma unroll
            for (int e = 0; e < 4; e++) {
              r[2 * e] = fmaf(-c2, __uint_as_float(xr[8 * u + 2 * e]), bf16_lo(vs[e]));
              r[2 * e + 1] = fmaf(-c2, __uint_as_float(xr[8 * u + 2 * e + 1]), bf16_hi(vs[e]));
            }
            *reinterpret_cast<uint4*>(vb + (vu >> 3) * 8192 + sw128_offset(t, 16 * (vu & 7))) = pack8(r);
          }
          tmem_st32(tp + 32 * hf, zero);
        }
        tmem_st_wait();
        fence_proxy_async();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_R);
        // Dsb_t = c4_t (row t of Tb R'), in place of R', the B operand of MMA (e)
        ok = __all_sync(0xffffffffu, mbar_wait(bar_c, ph, a.status));
        if (!ok) break;
        tc_fence_after();
        const float c4 = sc[128 + t];
#pragma unroll
        for (int hf = 0; hf < 4; hf++) {
          uint32_t dr[32];
          tmem_ld32(tp + 32 * hf, dr);
          tmem_ld_wait();
#pragma unroll
          for (int u = 0; u < 4; u++) {
            const int vu = 4 * hf + u;
            uint4 w;
            w.x = pack2(c4 * __uint_as_float(dr[8 * u + 0]), c4 * __uint_as_float(dr[8 * u + 1]));
            w.y = pack2(c4 * __uint_as_float(dr[8 * u + 2]), c4 * __uint_as_float(dr[8 * u + 3]));
            w.z = pack2(c4 * __uint_as_float(dr[8 * u + 4]), c4 * __uint_as_float(dr[8 * u + 5]));
            w.w = pack2(c4 * __uint_as_float(dr[8 * u + 6]), c4 * __uint_as_float(dr[8 * u + 7]));
            *reinterpret_cast<uint4*>(vb + (vu >> 3) * 8192 + sw128_offset(t, 16 * (vu & 7))) = w;
          }
        }
        fence_proxy_async();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_D);
      } else {
        // QS_i *= c3_i (token i = t - 64): MMA (c) then leaves O_i = c3_i QS_i + O2_i
        ok = __all_sync(0xffffffffu,
                        mbar_wait(bar_a, ph, a.status) && mbar_wait(&sc_full[c & 1], (c >> 1) & 1, a.status));
        if (!ok) break;
        tc_fence_after();
        const int i = t - 64;
        const float c3 = sc[64 + i];
#pragma unroll
        for (int hf = 0; hf < 4; hf++) {
          uint32_t qs[32];
          tmem_ld32(tp + 32 * hf, qs);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; j++) qs[j] = __float_as_uint(c3 * __uint_as_float(qs[j]));
          tmem_st32(tp + 32 * hf, qs);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_R);
        // O_i staged as f32 for the TMA stores, four 32-value boxes of 64 token
        // rows: boxes 0-1 in W's buffer (read by MMA (c) already), 2-3 in the
        // state buffer's second half (read by MMA (a))
        ok = __all_sync(0xffffffffu, mbar_wait(bar_c, ph, a.status));
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int hf = 0; hf < 4; hf++) {
          uint32_t o[32];
          tmem_ld32(tp + 32 * hf, o);
          tmem_ld_wait();
          if (hf == 3) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_D);
          }
          uint8_t* orow = hf < 2 ? sm + C_OFF_W + hf * 8192 : s0b + 16384 + (hf - 2) * 8192;
#pragma unroll
          for (int u = 0; u < 8; u++)
            *reinterpret_cast<float4*>(orow + sw128_offset(i, 16 * u)) =
                make_float4(__uint_as_float(o[4 * u]), __uint_as_float(o[4 * u + 1]), __uint_as_float(o[4 * u + 2]),
                            __uint_as_float(o[4 * u + 3]));
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(o_ready);
      }
      // S1 = e S0 + U is in TMEM: snapshots and the final state from it, its
      // bf16 copy for the next chunk's MMA (a) and e' S1 for its MMA (e)
      const bool more = c + 1 < n;
      ok = __all_sync(0xffffffffu, mbar_wait(bar_e, ph, a.status) &&
                                       (!more || mbar_wait(&sc_full[(c + 1) & 1], ((c + 1) >> 1) & 1, a.status)));
      if (!ok) break;
      tc_fence_after();
      const float e1 = more ? scal[((c + 1) & 1) * SC_FLOATS + 192] : 0.f;
      float4* dst = nullptr;
      if (a.snap && (a.c0 + c + 1) % a.snap_every == 0) {
        const long long j = (a.c0 + c + 1) / a.snap_every - 1;  // < snap_count: the chunk is full
        if (j < a.snap_count)
          dst = reinterpret_cast<float4*>(a.snap + (((size_t)b * a.snap_count + j) * a.NV + h) * GD * GD +
                                          (size_t)t * GD);
      }
      float4* fin = more ? nullptr : reinterpret_cast<float4*>(a.state_out + row * GD);
#pragma unroll
      for (int hf = 0; hf < 4; hf++) {
        if (hf == 2 && more) {
          // the state buffer's second half: once this chunk's output boxes 2-3 left it
          ok = __all_sync(0xffffffffu, mbar_wait(s0_free, ph, a.status));
          if (!ok) break;
        }
        uint32_t sr[32];
        tmem_ld32(tsr + 32 * hf, sr);
        tmem_ld_wait();
        if (dst) {
#pragma unroll
          for (int i = 0; i < 8; i++)
            dst[8 * hf + i] = make_float4(__uint_as_float(sr[4 * i]), __uint_as_float(sr[4 * i + 1]),
                                          __uint_as_float(sr[4 * i + 2]), __uint_as_float(sr[4 * i + 3]));
        }
        if (fin) {
#pragma unroll
          for (int i = 0; i < 8; i++)
            fin[8 * hf + i] = make_float4(__uint_as_float(sr[4 * i]), __uint_as_float(sr[4 * i + 1]),
                                          __uint_as_float(sr[4 * i + 2]), __uint_as_float(sr[4 * i + 3]));
        }
        if (more) {
#pragma unroll
          for (int u = 0; u < 4; u++) {
            uint4 w;
            w.x = pack2(__uint_as_float(sr[8 * u + 0]), __uint_as_float(sr[8 * u + 1]));
            w.y = pack2(__uint_as_float(sr[8 * u + 2]), __uint_as_float(sr[8 * u + 3]));
            w.z = pack2(__uint_as_float(sr[8 * u + 4]), __uint_as_float(sr[8 * u + 5]));
            w.w = pack2(__uint_as_float(sr[8 * u + 6]), __uint_as_float(sr[8 * u + 7]));
            *reinterpret_cast<uint4*>(s0b + (hf >> 1) * 16384 + sw128_offset(t, 64 * (hf & 1) + 16 * u)) = w;
          }
#pragma unroll
          for (int j = 0; j < 32; j++) sr[j] = __float_as_uint(e1 * __uint_as_float(sr[j]));
          tmem_st32(tsr + 32 * hf, sr);
        }
      }
      if (!ok) break;
      if (more) {
        tmem_st_wait();
        fence_proxy_async();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_s0);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sc_empty[c & 1]);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, C_TMEM_COLS);
  }
}

// =====================================================================
// split chain: two CTAs per (sequence, V head), the state in registers
// =====================================================================
__global__ void __launch_bounds__(CHAIN_THREADS, 2)
    gdn_chain_split_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmW,
                     const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmO,
                     const ChainArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + R_OFF_BAR);
  uint64_t* kq_full = bars + 0;
  uint64_t* kq_empty = bars + 1;  // MMA a done
  uint64_t* ke_full = bars + 2;
  uint64_t* ke_empty = bars + 3;  // MMA e done
  uint64_t* v_full = bars + 4;
  uint64_t* v_empty = bars + 5;   // R' written
  uint64_t* w_full = bars + 6;
  uint64_t* o_ready = bars + 7;   // MMA c done and the chunk's outputs staged in W's place
  uint64_t* sc_full = bars + 8;   // [2]
  uint64_t* sc_empty = bars + 10; // [2] chunk finished by the chain warps
  uint64_t* bar_a = bars + 12;    // [X; QS] in TMEM
  uint64_t* bar_R = bars + 13;    // R' in shared memory
  uint64_t* bar_c = bars + 14;    // [Tb R'; O2] in TMEM
  uint64_t* bar_D = bars + 15;    // Dsb in shared memory, [X; QS] and [Tb R'; O2] read
  uint64_t* bar_e = bars + 16;    // U in TMEM
  uint64_t* bar_s0 = bars + 17;   // bf16 state written
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + R_NBAR);
  float* scal = reinterpret_cast<float*>(sm + R_OFF_SC);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Grid (2 x V heads per QK head, QK heads, sequences): the CTAs of one QK
  // head's V heads h = hk, hk + NK, ... and both value-column halves are
  // adjacent, so they run together and share each chunk's K / Q tiles in L2.
  const int dvb = blockIdx.x & 1, hk = blockIdx.y, b = blockIdx.z;
  const int h = hk + (int)(blockIdx.x >> 1) * a.NK;
  if (h >= a.NV) return;  // the whole CTA, before any barrier or allocation
  const int n = a.cnt;
  const size_t unit0 = ((size_t)b * a.NV + h) * a.ns;

  if (tid == 0) {
    mbar_init(kq_full, 1);
    mbar_init(kq_empty, 1);
    mbar_init(ke_full, 1);
    mbar_init(ke_empty, 1);
    mbar_init(v_full, 1);
    mbar_init(v_empty, 2);
    mbar_init(w_full, 1);
    mbar_init(o_ready, 2);
    for (int i = 0; i < 2; i++) {
      mbar_init(&sc_full[i], 1);
      mbar_init(&sc_empty[i], 4);
    }
    mbar_init(bar_a, 1);
    mbar_init(bar_R, 2);
    mbar_init(bar_c, 1);
    mbar_init(bar_D, 4);
    mbar_init(bar_e, 1);
    mbar_init(bar_s0, 4);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, R_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_tensormap(&tmK);
      prefetch_tensormap(&tmQ);
      prefetch_tensormap(&tmV);
      prefetch_tensormap(&tmW);
      prefetch_tensormap(&tmS);
      prefetch_tensormap(&tmO);
      // outputs of chunk j: staged by the output warps in W's buffer, stored here
      auto store_outputs = [&](int j) {
        const int tj = (a.c0 + j) * GC;
        tma_store_4d(&tmO, sm + R_OFF_W, dvb * R_COLS, h, tj, b);
        tma_store_4d(&tmO, sm + R_OFF_W + 8192, dvb * R_COLS + 32, h, tj, b);
        tma_store_commit();
        tma_store_wait_read();
      };
      int c = 0;
      for (; c < n; c++) {
        const int t0 = (a.c0 + c) * GC;
        const int u = (int)(unit0 + c);
        const uint32_t pe = (c - 1) & 1;
        if (c + 1 < n) {
          // warm L2 with the next chunk's tiles: its loads below are issued only
          // when this chunk frees the buffers, a chunk's time before they are needed
          const int t1 = t0 + GC;
          tma_prefetch_l2_4d(&tmK, 0, hk, t1, b);
          tma_prefetch_l2_4d(&tmK, 64, hk, t1, b);
          tma_prefetch_l2_4d(&tmQ, 0, hk, t1, b);
          tma_prefetch_l2_4d(&tmQ, 64, hk, t1, b);
          tma_prefetch_l2_4d(&tmV, dvb * R_COLS, h, t1, b);
          tma_prefetch_l2_2d(&tmW, 0, (u + 1) * 128);
          tma_prefetch_l2_2d(&tmS, 0, (u + 1) * 4);
        }
        if (c >= 1 && !mbar_wait(kq_empty, pe, a.status)) break;
        mbar_arrive_expect_tx(kq_full, 32768);
        tma_load_4d(sm + R_OFF_KQ, &tmK, kq_full, 0, hk, t0, b);
        tma_load_4d(sm + R_OFF_KQ + 8192, &tmQ, kq_full, 0, hk, t0, b);
        tma_load_4d(sm + R_OFF_KQ + 16384, &tmK, kq_full, 64, hk, t0, b);
        tma_load_4d(sm + R_OFF_KQ + 24576, &tmQ, kq_full, 64, hk, t0, b);
        if (c >= 1 && !mbar_wait(v_empty, pe, a.status)) break;
        mbar_arrive_expect_tx(v_full, 8192);
        tma_load_4d(sm + R_OFF_V, &tmV, v_full, dvb * R_COLS, h, t0, b);
        if (c >= 2 && !mbar_wait(&sc_empty[c & 1], ((c - 2) >> 1) & 1, a.status)) break;
        mbar_arrive_expect_tx(&sc_full[c & 1], SC_FLOATS * 4);
        tma_load_2d(scal + (c & 1) * SC_FLOATS, &tmS, &sc_full[c & 1], 0, u * 4);
        if (c >= 1) {
          if (!mbar_wait(o_ready, pe, a.status)) break;
          store_outputs(c - 1);
        }
        mbar_arrive_expect_tx(w_full, W_ELEMS * 2);
        tma_load_2d(sm + R_OFF_W, &tmW, w_full, 0, u * 128);
        if (c >= 1 && !mbar_wait(ke_empty, pe, a.status)) break;
        mbar_arrive_expect_tx(ke_full, 16384);
        tma_load_4d(sm + R_OFF_KE, &tmK, ke_full, 0, hk, t0, b);
        tma_load_4d(sm + R_OFF_KE + 8192, &tmK, ke_full, 64, hk, t0, b);
      }
      if (c == n && n > 0 && mbar_wait(o_ready, (n - 1) & 1, a.status)) store_outputs(n - 1);
      tma_store_wait_all();
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    // The whole warp walks the loop (its values are warp-uniform); one
    // elected lane issues each tcgen05 instruction.
    {
      const bool leader = elect_one_sync();
      constexpr uint32_t id_n64 = idesc_f16(128, 64, true, false, true);  // K-major A, MN-major B
      constexpr uint32_t id_e = idesc_f16(128, 64, true, true, true);     // MN-major A (K^T)
      const uint32_t s0 = smem_u32(sm);
      for (int c = 0; c < n; c++) {
        const uint32_t ph = c & 1;
        // (a) [X; QS] = [K; Q] S0   (M = 128, N = 64, K = 128)
        if (!__all_sync(0xffffffffu, mbar_wait(kq_full, ph, a.status) && mbar_wait(bar_s0, ph, a.status))) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 8; ks++) {
          const uint64_t ad = smem_desc_sw128(s0 + R_OFF_KQ + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024);
          const uint64_t bd = smem_desc_sw128(s0 + R_OFF_S0B + ks * 2048, 8192, 1024);
          if (leader) mma_f16_ss(tmem + RT_P, ad, bd, id_n64, ks > 0);
        }
        if (leader) {
          mma_commit(bar_a);
          mma_commit(kq_empty);
        }
        // (c) [Tb R'; O2] = W R'   (M = 128, N = 64, K = 64)
        if (!__all_sync(0xffffffffu, mbar_wait(bar_R, ph, a.status) && mbar_wait(w_full, ph, a.status))) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 4; ks++) {
          const uint64_t ad = smem_desc_sw128(s0 + R_OFF_W + ks * 32, 16, 1024);
          const uint64_t bd = smem_desc_sw128(s0 + R_OFF_RB + ks * 2048, 8192, 1024);
          if (leader) mma_f16_ss(tmem + RT_Q, ad, bd, id_n64, ks > 0);
        }
        if (leader) mma_commit(bar_c);
        // (e) U = K^T Dsb   (M = 128, N = 64, K = 64)
        if (!__all_sync(0xffffffffu, mbar_wait(bar_D, ph, a.status) && mbar_wait(ke_full, ph, a.status))) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 4; ks++) {
          const uint64_t ad = smem_desc_sw128(s0 + R_OFF_KE + ks * 2048, 8192, 1024);
          const uint64_t bd = smem_desc_sw128(s0 + R_OFF_DSB + ks * 2048, 8192, 1024);
          if (leader) mma_f16_ss(tmem + RT_P, ad, bd, id_e, ks > 0);
        }
        if (leader) {
          mma_commit(bar_e);
          mma_commit(ke_empty);
        }
      }
    }
  } else {
    // ---------------- chain warps 2-5: TMEM lane quadrant = warp % 4 ----------------
    const int quad = warp & 3;
    const int t = quad * 32 + lane;  // state row (dk); row of [K; Q] / W results
    const uint32_t lo = (uint32_t)(quad * 32) << 16;
    uint8_t* s0b = sm + R_OFF_S0B;
    float st[64];
    if (a.load_state) {
      const float4* src =
          reinterpret_cast<const float4*>(a.state_in + (((size_t)b * a.NV + h) * GD + t) * GD + dvb * R_COLS);
#pragma unroll
      for (int i = 0; i < 16; i++) {
        const float4 v = __ldg(src + i);
        st[4 * i] = v.x;
        st[4 * i + 1] = v.y;
        st[4 * i + 2] = v.z;
        st[4 * i + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 64; i++) st[i] = 0.f;
    }
    store_row64(s0b, t, st);
    fence_proxy_async();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(bar_s0);
    bool ok = true;
    for (int c = 0; c < n && ok; c++) {
      const uint32_t ph = c & 1;
      const float* sc = scal + (c & 1) * SC_FLOATS;
      if (quad < 2) {
        // R'_t = V_t - c2_t X_t   (token t); V's row is read before X lands
        ok = __all_sync(0xffffffffu,
                        mbar_wait(v_full, ph, a.status) && mbar_wait(&sc_full[c & 1], (c >> 1) & 1, a.status));
        if (!ok) break;
        const float c2 = sc[t];
        uint4 vrow[8];
#pragma unroll
        for (int u = 0; u < 8; u++) vrow[u] = *reinterpret_cast<const uint4*>(sm + R_OFF_V + sw128_offset(t, 16 * u));
        ok = __all_sync(0xffffffffu, mbar_wait(bar_a, ph, a.status));
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int hf = 0; hf < 2; hf++) {
          uint32_t xr[32];
          tmem_ld32(tmem + lo + RT_P + 32 * hf, xr);
          tmem_ld_wait();
#pragma unroll
          for (int u = 0; u < 4; u++) {
            const uint32_t off = sw128_offset(t, 64 * hf + 16 * u);
            const uint4 vw = vrow[4 * hf + u];
            const uint32_t vs[4] = {vw.x, vw.y, vw.z, vw.w};
            float r[8];
#pragma unroll
            for (int e = 0; e < 4; e++) {
              r[2 * e] = fmaf(-c2, __uint_as_float(xr[8 * u + 2 * e]), bf16_lo(vs[e]));
              r[2 * e + 1] = fmaf(-c2, __uint_as_float(xr[8 * u + 2 * e + 1]), bf16_hi(vs[e]));
            }
            *reinterpret_cast<uint4*>(sm + R_OFF_RB + off) = pack8(r);
          }
        }
        fence_proxy_async();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(bar_R);
          mbar_arrive(v_empty);
        }
        // Dsb_t = c4_t (row t of Tb R'), the bf16 operand of the state update
        ok = __all_sync(0xffffffffu, mbar_wait(bar_c, ph, a.status));
        if (!ok) break;
        tc_fence_after();
        const float c4 = sc[128 + t];
#pragma unroll
        for (int hf = 0; hf < 2; hf++) {
          uint32_t dr[32];
          tmem_ld32(tmem + lo + RT_Q + 32 * hf, dr);
          tmem_ld_wait();
#pragma unroll
          for (int u = 0; u < 4; u++) {
            uint4 w;
            w.x = pack2(c4 * __uint_as_float(dr[8 * u + 0]), c4 * __uint_as_float(dr[8 * u + 1]));
            w.y = pack2(c4 * __uint_as_float(dr[8 * u + 2]), c4 * __uint_as_float(dr[8 * u + 3]));
            w.z = pack2(c4 * __uint_as_float(dr[8 * u + 4]), c4 * __uint_as_float(dr[8 * u + 5]));
            w.w = pack2(c4 * __uint_as_float(dr[8 * u + 6]), c4 * __uint_as_float(dr[8 * u + 7]));
            *reinterpret_cast<uint4*>(sm + R_OFF_DSB + sw128_offset(t, 64 * hf + 16 * u)) = w;
          }
        }
        fence_proxy_async();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_D);
      } else {
        // O_i = c3_i QS_i + O2_i   (token i = t - 64)
        ok = __all_sync(0xffffffffu,
                        mbar_wait(bar_c, ph, a.status) && mbar_wait(&sc_full[c & 1], (c >> 1) & 1, a.status));
        if (!ok) break;
        tc_fence_after();
        const int i = t - 64;
        const float c3 = sc[64 + i];
#pragma unroll
        for (int hf = 0; hf < 2; hf++) {
          uint32_t qs[32], o2[32];
          tmem_ld32(tmem + lo + RT_P + 32 * hf, qs);
          tmem_ld32(tmem + lo + RT_Q + 32 * hf, o2);
          tmem_ld_wait();
          if (hf == 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_D);
          }
          // row i of the staged outputs: 32 f32 = one 128-byte swizzled row of half hf
          uint8_t* orow = sm + R_OFF_W + hf * 8192;
#pragma unroll
          for (int u = 0; u < 8; u++)
            *reinterpret_cast<float4*>(orow + sw128_offset(i, 16 * u)) =
                make_float4(fmaf(c3, __uint_as_float(qs[4 * u]), __uint_as_float(o2[4 * u])),
                            fmaf(c3, __uint_as_float(qs[4 * u + 1]), __uint_as_float(o2[4 * u + 1])),
                            fmaf(c3, __uint_as_float(qs[4 * u + 2]), __uint_as_float(o2[4 * u + 2])),
                            fmaf(c3, __uint_as_float(qs[4 * u + 3]), __uint_as_float(o2[4 * u + 3])));
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(o_ready);
      }
      // S1 = e S0 + U, and its bf16 copy for the next chunk
      ok = __all_sync(0xffffffffu, mbar_wait(bar_e, ph, a.status));
      if (!ok) break;
      tc_fence_after();
      const float e = sc[192];
#pragma unroll
      for (int hf = 0; hf < 2; hf++) {
        uint32_t ur[32];
        tmem_ld32(tmem + lo + RT_P + 32 * hf, ur);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; j++) st[32 * hf + j] = fmaf(e, st[32 * hf + j], __uint_as_float(ur[j]));
#pragma unroll
        for (int u = 0; u < 4; u++)
          *reinterpret_cast<uint4*>(s0b + sw128_offset(t, 64 * hf + 16 * u)) = pack8(st + 32 * hf + 8 * u);
      }
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(bar_s0);
        mbar_arrive(&sc_empty[c & 1]);
      }
      if (a.snap && (a.c0 + c + 1) % a.snap_every == 0) {
        const long long j = (a.c0 + c + 1) / a.snap_every - 1;  // < snap_count: the chunk is full
        if (j < a.snap_count) {
          float4* dst = reinterpret_cast<float4*>(
              a.snap + ((((size_t)b * a.snap_count + j) * a.NV + h) * GD + t) * GD + dvb * R_COLS);
#pragma unroll
          for (int i = 0; i < 16; i++) dst[i] = make_float4(st[4 * i], st[4 * i + 1], st[4 * i + 2], st[4 * i + 3]);
        }
      }
    }
    if (ok) {
      float4* dst = reinterpret_cast<float4*>(a.state_out + (((size_t)b * a.NV + h) * GD + t) * GD + dvb * R_COLS);
#pragma unroll
      for (int i = 0; i < 16; i++) dst[i] = make_float4(st[4 * i], st[4 * i + 1], st[4 * i + 2], st[4 * i + 3]);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, R_TMEM_COLS);
  }
}

}  // namespace
}  // namespace hcu

using hcu::fail;

namespace {

int chunked_prefill(hcu_handle h, const hcu_gdn_prefill_params* p, const void* q, const void* k, const void* v,
                    const float* g, const float* beta, const float* state_in, float* core, float* state_out,
                    uint32_t snap_every, float* snapshots) {
  if (!p || !q || !k || !v || !g || !beta || !core || !state_out || (p->load_state && !state_in))
    return fail(HCU_EINVAL, "hcu_deltanet_chunked_prefill: null argument");
  const long long B = p->B, T = p->T, NK = p->NK, NV = p->NV;
  if (B < 1 || T < 1 || NK < 1 || NV < 1) return fail(HCU_EINVAL, "hcu_deltanet_chunked_prefill: empty shape");
  if (p->D != hcu::GD) return fail(HCU_EUNSUPPORTED, "hcu_deltanet_chunked_prefill: D=%u (built: 128)", p->D);
  if (B > 65535 || NV > 65535 || NK > 65535)
    return fail(HCU_EINVAL, "hcu_deltanet_chunked_prefill: B, NK or NV > 65535");
  const long long qrow = p->q_row_stride ? (long long)p->q_row_stride : NK * 128;
  const long long krow = p->k_row_stride ? (long long)p->k_row_stride : NK * 128;
  const long long vrow = p->v_row_stride ? (long long)p->v_row_stride : NV * 128;
  const long long qseq = p->q_seq_stride ? (long long)p->q_seq_stride : T * qrow;
  const long long kseq = p->k_seq_stride ? (long long)p->k_seq_stride : T * krow;
  const long long vseq = p->v_seq_stride ? (long long)p->v_seq_stride : T * vrow;
  if (reinterpret_cast<uintptr_t>(core) % 16 || reinterpret_cast<uintptr_t>(state_out) % 16 ||
      (p->load_state && reinterpret_cast<uintptr_t>(state_in) % 16) ||
      reinterpret_cast<uintptr_t>(snapshots) % 16)
    return fail(HCU_EINVAL, "hcu_deltanet_chunked_prefill: core / state buffers must be 16-byte aligned");
  const long long snap_count = snap_every ? T / (hcu::GC * (long long)snap_every) : 0;
  CUtensorMap tq, tk, tv, tw, twh, ts, to;
  {
    uint64_t dims[4] = {128, (uint64_t)NK, (uint64_t)T, (uint64_t)B};
    uint64_t st[3] = {256, (uint64_t)qrow * 2, (uint64_t)qseq * 2};
    uint32_t box[4] = {64, 1, 64, 1};
    HCU_TRY(hcu::make_tensor_map(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(q), dims, st, box,
                                 CU_TENSOR_MAP_SWIZZLE_128B));
    uint64_t stk[3] = {256, (uint64_t)krow * 2, (uint64_t)kseq * 2};
    HCU_TRY(hcu::make_tensor_map(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(k), dims, stk, box,
                                 CU_TENSOR_MAP_SWIZZLE_128B));
  }
  {
    uint64_t dims[4] = {128, (uint64_t)NV, (uint64_t)T, (uint64_t)B};
    uint64_t st[3] = {256, (uint64_t)vrow * 2, (uint64_t)vseq * 2};
    uint32_t box[4] = {64, 1, 64, 1};
    HCU_TRY(hcu::make_tensor_map(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(v), dims, st, box,
                                 CU_TENSOR_MAP_SWIZZLE_128B));
    // outputs core [B][T][NV][128] f32, stored 32 values x 64 tokens at a time
    uint64_t ost[3] = {512, (uint64_t)NV * 512, (uint64_t)T * NV * 512};
    uint32_t obox[4] = {32, 1, 64, 1};
    HCU_TRY(hcu::make_tensor_map(&to, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, core, dims, ost, obox,
                                 CU_TENSOR_MAP_SWIZZLE_128B));
  }
  // Scratch: the prep outputs of one slab of chunks (17 KB per sequence, V head
  // and chunk).  The slab is as long as the scratch budget allows
  // (HCU_OPT_GDN_SCRATCH_MB, default 1 GiB: one slab for 8 x 8192 tokens x 32 heads).
  const long long nchunks = (T + hcu::GC - 1) / hcu::GC;
  const long long per_chunk = B * NV * (long long)hcu::UNIT_BYTES;
  const long long budget = (h->opt_gdn_scratch_mb > 0 ? (long long)h->opt_gdn_scratch_mb : 1024ll) << 20;
  long long ns = budget / per_chunk;
  if (ns < 1) ns = 1;
  if (ns > nchunks) ns = nchunks;
  const long long nslab = (nchunks + ns - 1) / ns;
  ns = (nchunks + nslab - 1) / nslab;  // even slabs
  const long long units = B * NV * ns;
  if (units * 128 > 0x7fffffffll)
    return fail(HCU_EINVAL, "hcu_deltanet_chunked_prefill: %lld units per slab exceed the TMA range", units);
  HCU_TRY(hcu::ensure_scratch(h, (size_t)units * hcu::UNIT_BYTES, "hcu_deltanet_chunked_prefill"));
  auto* wbuf = reinterpret_cast<__nv_bfloat16*>(h->scratch);  // [units][128][64] bf16
  auto* sbuf = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(h->scratch) + (size_t)units * hcu::W_ELEMS * 2);
  {
    uint64_t dims[2] = {64, (uint64_t)units * 128};
    uint64_t st[1] = {128};
    uint32_t box[2] = {64, 128};
    HCU_TRY(hcu::make_tensor_map(&tw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, wbuf, dims, st, box,
                                 CU_TENSOR_MAP_SWIZZLE_128B));
    uint32_t hbox[2] = {64, 64};  // the prep stores W as two 64-row halves
    HCU_TRY(hcu::make_tensor_map(&twh, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, wbuf, dims, st, hbox,
                                 CU_TENSOR_MAP_SWIZZLE_128B));
    uint64_t sdims[2] = {64, (uint64_t)units * 4};
    uint64_t sst[1] = {256};
    uint32_t sbox[2] = {64, 4};
    HCU_TRY(hcu::make_tensor_map(&ts, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, sbuf, sdims, sst, sbox,
                                 CU_TENSOR_MAP_SWIZZLE_NONE));
  }
  static std::atomic<uint64_t> attr_done{0};  // per device
  HCU_TRY(hcu::once_per_device(attr_done, h->device, [&]() -> int {
    HCU_TRY(hcu::check_cuda(cudaFuncSetAttribute(hcu::gdn_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 hcu::P_SMEM + 1024),
                            "hcu_deltanet_chunked_prefill: smem attribute"));
    HCU_TRY(hcu::check_cuda(cudaFuncSetAttribute(hcu::gdn_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 hcu::C_SMEM + 1024),
                            "hcu_deltanet_chunked_prefill: smem attribute"));
    HCU_TRY(hcu::check_cuda(cudaFuncSetAttribute(hcu::gdn_chain_split_kernel,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, hcu::R_SMEM + 1024),
                            "hcu_deltanet_chunked_prefill: smem attribute"));
    return HCU_OK;
  }));
  const long long gb_row = p->gb_row_stride ? (long long)p->gb_row_stride : NV;
  const long long gb_seq = p->gb_seq_stride ? (long long)p->gb_seq_stride : T * gb_row;
  // The recurrence kernel: two 64-column CTAs per (sequence, V head) walk the
  // chunks faster than one 128-column CTA, so they are used while the batch
  // still fits one wave of two CTAs per SM; larger batches take one CTA per head.
  const long long ncol = h->opt_gdn_chain_cols ? h->opt_gdn_chain_cols
                         : (2 * B * NV <= 2LL * h->sm_count ? 64 : 128);
  const long long npair = ((NV + NK - 1) / NK + 1) / 2;  // V heads per QK head, two per prep CTA
  if (NK * npair > 65535) return fail(HCU_EINVAL, "hcu_deltanet_chunked_prefill: too many heads");
  for (long long s = 0; s < nslab; s++) {
    const long long c0 = s * ns;
    const long long cnt = nchunks - c0 < ns ? nchunks - c0 : ns;
    hcu::PrepArgs pa{};
    pa.T = (int)T;
    pa.NK = (int)NK;
    pa.NV = (int)NV;
    pa.c0 = (int)c0;
    pa.ns = (int)ns;
    pa.ahead = 2 * h->sm_count;  // two prep CTAs are resident per SM
    pa.g = g;
    pa.beta = beta;
    pa.gb_row = gb_row;
    pa.gb_seq = gb_seq;
    pa.sc = sbuf;
    pa.status = h->dev_status;
    hcu::gdn_prep_kernel<<<dim3((unsigned)cnt, (unsigned)(NK * npair), (unsigned)B), hcu::PREP_THREADS,
                           hcu::P_SMEM + 1024, h->stream>>>(tq, tk, twh, pa);
    HCU_TRY(hcu::after_launch("hcu_deltanet_chunked_prefill: prep launch"));
    hcu::ChainArgs ca{};
    ca.T = (int)T;
    ca.NK = (int)NK;
    ca.NV = (int)NV;
    ca.c0 = (int)c0;
    ca.ns = (int)ns;
    ca.cnt = (int)cnt;
    ca.load_state = (s > 0 || p->load_state) ? 1 : 0;
    ca.state_in = s > 0 ? state_out : state_in;
    ca.core = core;
    ca.state_out = state_out;
    ca.status = h->dev_status;
    ca.snap = snap_count > 0 ? snapshots : nullptr;
    ca.snap_every = (int)snap_every;
    ca.snap_count = snap_count;
    const long long nvper = (NV + NK - 1) / NK;  // V heads per QK head (the last QK heads may have fewer)
    if (ncol == 128) {
      const dim3 cgrid((unsigned)nvper, (unsigned)NK, (unsigned)B);
      hcu::gdn_chain_kernel<<<cgrid, hcu::CHAIN_THREADS, hcu::C_SMEM + 1024, h->stream>>>(tq, tk, tv, tw, ts, to, ca);
    } else {
      const dim3 cgrid((unsigned)(hcu::GD / hcu::R_COLS * nvper), (unsigned)NK, (unsigned)B);
      hcu::gdn_chain_split_kernel<<<cgrid, hcu::CHAIN_THREADS, hcu::R_SMEM + 1024, h->stream>>>(tq, tk, tv, tw, ts,
                                                                                                 to, ca);
    }
    HCU_TRY(hcu::after_launch("hcu_deltanet_chunked_prefill: chain launch"));
  }
  return HCU_OK;
}

}  // namespace

extern "C" int hcu_deltanet_chunked_prefill(hcu_handle h, const hcu_gdn_prefill_params* p, const void* q,
                                            const void* k, const void* v, const float* g, const float* beta,
                                            const float* state_in, float* core, float* state_out) {
  HCU_TRY(hcu::begin_op(h, "hcu_deltanet_chunked_prefill"));
  return chunked_prefill(h, p, q, k, v, g, beta, state_in, core, state_out, 0, nullptr);
}

extern "C" int hcu_deltanet_chunked_prefill_snap(hcu_handle h, const hcu_gdn_prefill_params* p, const void* q,
                                                 const void* k, const void* v, const float* g, const float* beta,
                                                 const float* state_in, float* core, float* state_out,
                                                 uint32_t snap_every, float* snapshots) {
  HCU_TRY(hcu::begin_op(h, "hcu_deltanet_chunked_prefill_snap"));
  if (!snap_every || !snapshots)
    return fail(HCU_EINVAL, "hcu_deltanet_chunked_prefill_snap: snap_every must be >= 1 and snapshots non-null");
  return chunked_prefill(h, p, q, k, v, g, beta, state_in, core, state_out, snap_every, snapshots);
}
