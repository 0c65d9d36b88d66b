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
//   R     = diag(beta) (V - diag(Gamma ik) K S0)
//   Delta = (I + A)^-1 R                          (the per-token deltas)
//   O     = diag(Gamma iq) Q S0 + QKm Delta,  QKm_ij = iq_i ik_j exp(gamma_i - gamma_j) (q_i . k_j)  (j <= i)
//   S1    = exp(gamma_63) S0 + K^T diag(ik_j exp(gamma_63 - gamma_j)) Delta
// The products run on the tensor cores (bf16 operands, f32 accumulation in
// TMEM); the state S is kept in f32 in TMEM across chunks (its bf16 copy is
// the MMA operand); (I + A)^-1 is solved in f32 on the CUDA cores by 16x16
// diagonal blocks combined twice.
//
// One CTA per (sequence, V head, 64-wide block of value columns): the state's
// value columns evolve independently.  Warp 0 streams K / Q / V chunks with
// TMA (double-buffered), warp 1 allocates TMEM and issues the MMAs, warps 4-7
// (one TMEM lane each) do the element-wise work and the solve.
#include "common.cuh"
#include "context.h"
#include "tcgen05.cuh"

namespace hcu {
namespace {

constexpr int GC = 64;        // chunk length
constexpr int GD = 128;       // DK = DV
constexpr int DVB = 64;       // value columns per CTA
constexpr int GT_THREADS = 256;
// shared memory layout (bytes)
constexpr int KQ_BYTES = 32768;  // per buffer: [d-block 0: K rows 0-63 | Q rows 0-63][d-block 1: same]
constexpr int V_BYTES = 8192;    // per buffer: [64 tokens x 64 values] bf16
constexpr int OFF_KQ = 0;
constexpr int OFF_V = OFF_KQ + 2 * KQ_BYTES;
constexpr int OFF_S0B = OFF_V + 2 * V_BYTES;   // [128 dk x 64 dv] bf16, MN-major B operand
constexpr int OFF_TB = OFF_S0B + 16384;        // [64 x 64] bf16 (I+A)^-1, K-major A operand
constexpr int OFF_QKM = OFF_TB + 8192;         // [64 x 64] bf16, K-major A operand
constexpr int OFF_RB = OFF_QKM + 8192;         // [64 tok x 64 dv] bf16, MN-major B operand
constexpr int OFF_DB = OFF_RB + 8192;          // Delta
constexpr int OFF_DSB = OFF_DB + 8192;         // diag(ik exp(g63 - g)) Delta
constexpr int OFF_AF = OFF_DSB + 8192;         // [64][65] f32 A (and G)
constexpr int OFF_TF = OFF_AF + 64 * 65 * 4;   // [64][65] f32 (I+A)^-1
constexpr int OFF_X1 = OFF_TF + 64 * 65 * 4;   // [2][16][17] f32
constexpr int OFF_X2 = OFF_X1 + 2 * 16 * 17 * 4;  // [32][33] f32
constexpr int OFF_SC = OFF_X2 + 32 * 33 * 4;   // gam2[64] beta[64] ik[64] iq[64] misc[8]
constexpr int OFF_BAR = OFF_SC + (4 * 64 + 8) * 4;
constexpr int NBAR = 13;
constexpr int SMEM_BYTES = OFF_BAR + NBAR * 8 + 16;
// TMEM columns
constexpr uint32_t TC_F = 0, TC_X = 64, TC_D = 128, TC_O = 192, TC_S = 256, TMEM_COLS = 512;

struct GdnArgs {
  int B, T, NK, NV, load_state, nchunks;
  const float* g;
  const float* beta;
  long long gb_row, gb_seq;
  const float* state_in;
  float* core;
  float* state_out;
  uint32_t* status;
};

__device__ __forceinline__ float fast_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// Writes 64 f32 values as one 128-byte bf16 row of a 128B-swizzled region.
__device__ __forceinline__ void store_row64(uint8_t* region, int row, const float (&x)[64]) {
#pragma unroll
  for (int u = 0; u < 8; u++) {
    uint4 w;
    w.x = pack2(x[8 * u + 0], x[8 * u + 1]);
    w.y = pack2(x[8 * u + 2], x[8 * u + 3]);
    w.z = pack2(x[8 * u + 4], x[8 * u + 5]);
    w.w = pack2(x[8 * u + 6], x[8 * u + 7]);
    *reinterpret_cast<uint4*>(region + sw128_offset(row, 16 * u)) = w;
  }
}

// Reads one 128-byte bf16 row (64 values) of a 128B-swizzled region.
__device__ __forceinline__ void load_row64(const uint8_t* region, int row, float (&x)[64]) {
#pragma unroll
  for (int u = 0; u < 8; u++) {
    const uint4 w = *reinterpret_cast<const uint4*>(region + sw128_offset(row, 16 * u));
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int e = 0; e < 4; e++) {
      x[8 * u + 2 * e] = __uint_as_float(ws[e] << 16);
      x[8 * u + 2 * e + 1] = __uint_as_float(ws[e] & 0xffff0000u);
    }
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

__device__ __forceinline__ void tmem_st64(uint32_t taddr, const float (&x)[64]) {
  uint32_t r0[32], r1[32];
#pragma unroll
  for (int i = 0; i < 32; i++) {
    r0[i] = __float_as_uint(x[i]);
    r1[i] = __float_as_uint(x[32 + i]);
  }
  tmem_st32(taddr, r0);
  tmem_st32(taddr + 32, r1);
  tmem_st_wait();
}

__global__ void __launch_bounds__(GT_THREADS, 1)
    gdn_chunked_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const GdnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint64_t* kv_full = bars + 0;   // [2]
  uint64_t* kv_empty = bars + 2;  // [2]
  uint64_t* bar_f = bars + 4;     // MMA (f) done
  uint64_t* bar_a = bars + 5;     // MMA (a) done
  uint64_t* bar_c = bars + 6;     // MMA (c) done
  uint64_t* bar_d = bars + 7;     // MMA (d) done
  uint64_t* bar_e = bars + 8;     // MMA (e) done
  uint64_t* bar_T = bars + 9;     // (I+A)^-1, QKm, Q' written
  uint64_t* bar_R = bars + 10;    // R written
  uint64_t* bar_D = bars + 11;    // Delta copies written, state rescaled
  uint64_t* bar_s0 = bars + 12;   // S0 (bf16) written
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NBAR);
  float* Af = reinterpret_cast<float*>(sm + OFF_AF);
  float* Tf = reinterpret_cast<float*>(sm + OFF_TF);
  float* X1 = reinterpret_cast<float*>(sm + OFF_X1);
  float* X2 = reinterpret_cast<float*>(sm + OFF_X2);
  float* gam2 = reinterpret_cast<float*>(sm + OFF_SC);  // gamma * log2(e)
  float* betv = gam2 + 64;
  float* ikv = betv + 64;
  float* iqv = ikv + 64;
  float* misc = iqv + 64;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int dvb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h % a.NK;

  if (tid == 0) {
    for (int i = 0; i < 2; i++) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 4; i <= 8; i++) mbar_init(&bars[i], 1);
    for (int i = 9; i <= 12; i++) mbar_init(&bars[i], 4);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_tensormap(&tmQ);
      prefetch_tensormap(&tmK);
      prefetch_tensormap(&tmV);
      for (int c = 0; c < a.nchunks; c++) {
        const int buf = c & 1;
        if (c >= 2 && !mbar_wait(&kv_empty[buf], ((c - 2) >> 1) & 1, a.status)) break;
        uint8_t* kq = sm + OFF_KQ + buf * KQ_BYTES;
        const int t0 = c * GC;
        mbar_arrive_expect_tx(&kv_full[buf], KQ_BYTES + V_BYTES);
        tma_load_4d(kq, &tmK, &kv_full[buf], 0, hk, t0, b);
        tma_load_4d(kq + 8192, &tmQ, &kv_full[buf], 0, hk, t0, b);
        tma_load_4d(kq + 16384, &tmK, &kv_full[buf], 64, hk, t0, b);
        tma_load_4d(kq + 24576, &tmQ, &kv_full[buf], 64, hk, t0, b);
        tma_load_4d(sm + OFF_V + buf * V_BYTES, &tmV, &kv_full[buf], dvb * DVB, h, t0, b);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t id_f = idesc_f16(128, 64, true, false, false);  // [K;Q] K^T
      constexpr uint32_t id_kb = idesc_f16(64, 64, true, false, true);   // 64-row A (K-major) x MN-major B
      constexpr uint32_t id_e = idesc_f16(128, 64, true, true, true);    // K^T (MN-major) x MN-major B
      const uint32_t s0 = smem_u32(sm);
      bool ok = true;
      for (int c = 0; c < a.nchunks && ok; c++) {
        const int buf = c & 1;
        const uint32_t kq = s0 + OFF_KQ + buf * KQ_BYTES;
        ok = mbar_wait(&kv_full[buf], (c >> 1) & 1, a.status);
        if (!ok) break;
        tc_fence_after();
        // (f) D_f = [K; Q] . K^T   (M = 128, N = 64, K = 128)
#pragma unroll
        for (int ks = 0; ks < 8; ks++) {
          const uint32_t off = (ks >> 2) * 16384 + (ks & 3) * 32;
          mma_f16_ss(tmem + TC_F, smem_desc_sw128(kq + off, 16, 1024), smem_desc_sw128(kq + off, 16, 1024), id_f,
                     ks > 0);
        }
        mma_commit(bar_f);
        // (a) X = K . S0   (M = 64, N = 64, K = 128)
        ok = mbar_wait(bar_s0, c & 1, a.status);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 8; ks++) {
          const uint32_t off = (ks >> 2) * 16384 + (ks & 3) * 32;
          mma_f16_ss(tmem + TC_X, smem_desc_sw128(kq + off, 16, 1024),
                     smem_desc_sw128(s0 + OFF_S0B + ks * 2048, 8192, 1024), id_kb, ks > 0);
        }
        mma_commit(bar_a);
        // (c) Delta = (I+A)^-1 . R   (M = 64, N = 64, K = 64)
        ok = mbar_wait(bar_T, c & 1, a.status) && mbar_wait(bar_R, c & 1, a.status);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 4; ks++)
          mma_f16_ss(tmem + TC_D, smem_desc_sw128(s0 + OFF_TB + ks * 32, 16, 1024),
                     smem_desc_sw128(s0 + OFF_RB + ks * 2048, 8192, 1024), id_kb, ks > 0);
        mma_commit(bar_c);
        // (d) O = Q' . S0 + QKm . Delta   (M = 64, N = 64, K = 128 + 64)
        ok = mbar_wait(bar_D, c & 1, a.status);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 8; ks++) {
          const uint32_t off = (ks >> 2) * 16384 + 8192 + (ks & 3) * 32;
          mma_f16_ss(tmem + TC_O, smem_desc_sw128(kq + off, 16, 1024),
                     smem_desc_sw128(s0 + OFF_S0B + ks * 2048, 8192, 1024), id_kb, ks > 0);
        }
#pragma unroll
        for (int ks = 0; ks < 4; ks++)
          mma_f16_ss(tmem + TC_O, smem_desc_sw128(s0 + OFF_QKM + ks * 32, 16, 1024),
                     smem_desc_sw128(s0 + OFF_DB + ks * 2048, 8192, 1024), id_kb, 1);
        mma_commit(bar_d);
        // (e) S += K^T . Dsb   (M = 128, N = 64, K = 64; S pre-scaled by the math warps)
#pragma unroll
        for (int ks = 0; ks < 4; ks++)
          mma_f16_ss(tmem + TC_S, smem_desc_sw128(kq + ks * 2048, 16384, 1024),
                     smem_desc_sw128(s0 + OFF_DSB + ks * 2048, 8192, 1024), id_e, 1);
        mma_commit(bar_e);
        mma_commit(&kv_empty[buf]);
      }
    }
  } else if (warp >= 4) {
    // ---------------- element-wise work and the solve (128 threads) ----------------
    const int q4 = warp - 4;                 // TMEM lane quarter
    const int t = q4 * 32 + lane;            // 0..127
    const uint32_t lo = (uint32_t)(q4 * 32) << 16;
    const int r64 = q4 * 16 + lane;          // row of an M = 64 accumulator (valid when lane < 16)
    const float inv_sqrt_d = rsqrtf((float)GD);
    uint8_t* s0b = sm + OFF_S0B;
    bool ok = true;

    // initial state: TMEM (f32 master) and its bf16 copy
    {
      float x[64];
      if (a.load_state) {
        const float4* src = reinterpret_cast<const float4*>(
            a.state_in + (((size_t)b * a.NV + h) * GD + t) * GD + dvb * DVB);
#pragma unroll
        for (int i = 0; i < 16; i++) {
          const float4 v = __ldg(src + i);
          x[4 * i] = v.x;
          x[4 * i + 1] = v.y;
          x[4 * i + 2] = v.z;
          x[4 * i + 3] = v.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 64; i++) x[i] = 0.f;
      }
      tmem_st64(tmem + lo + TC_S, x);
      store_row64(s0b, t, x);
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_s0);
    }

    for (int c = 0; c < a.nchunks && ok; c++) {
      const int buf = c & 1;
      const int t0 = c * GC;
      uint8_t* kq = sm + OFF_KQ + buf * KQ_BYTES;
      const uint8_t* vt = sm + OFF_V + buf * V_BYTES;

      // ---- (f) landed: G = K K^T (rows 0-63), P = Q K^T (rows 64-127) ----
      if (!__all_sync(0xffffffffu, mbar_wait(bar_f, c & 1, a.status))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float f[64];
      tmem_ld64(tmem + lo + TC_F, f);
      float gi = 0.f, bi = 0.f;
      if (t < 64) {
#pragma unroll
        for (int j = 0; j < 64; j++) Af[t * 65 + j] = f[j];
        const int tok = t0 + t;
        if (tok < a.T) {
          const size_t gi_idx = (size_t)b * a.gb_seq + (size_t)tok * a.gb_row + h;
          gi = __ldg(a.g + gi_idx);
          bi = __ldg(a.beta + gi_idx);
        }
        // inclusive scan of g over the chunk (two warps)
        float sc = gi;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_up_sync(0xffffffffu, sc, o);
          if (lane >= o) sc += y;
        }
        if (t == 31) misc[0] = sc;
        gi = sc;
      }
      named_bar(1, 128);
      if (t < 64) {
        const float gam = gi + (t >= 32 ? misc[0] : 0.f);
        gam2[t] = gam * kLog2e;
        betv[t] = bi;
        ikv[t] = rsqrtf(Af[t * 65 + t] + 1e-6f);
      } else {
        // |q_i|^2 from the Q rows of the tile (both 64-element blocks)
        const int i = t - 64;
        float x0[64], x1[64];
        load_row64(kq, 64 + i, x0);
        load_row64(kq + 16384, 64 + i, x1);
        float s2 = 0.f;
#pragma unroll
        for (int j = 0; j < 64; j++) s2 = fmaf(x0[j], x0[j], fmaf(x1[j], x1[j], s2));
        iqv[i] = rsqrtf(s2 + 1e-6f) * inv_sqrt_d;
      }
      named_bar(1, 128);
      if (t < 64) {
        // A (strictly lower) in place of G
        const float gi2 = gam2[t], cb = betv[t] * ikv[t];
#pragma unroll
        for (int j = 0; j < 64; j++)
          Af[t * 65 + j] = j < t ? cb * ikv[j] * fast_ex2(gi2 - gam2[j]) * f[j] : 0.f;
      } else {
        // QKm row (lower incl. diagonal) and Q' = diag(Gamma iq) Q
        const int i = t - 64;
        const float gi2 = gam2[i], cq = iqv[i];
        float x[64];
#pragma unroll
        for (int j = 0; j < 64; j++) x[j] = j <= i ? cq * ikv[j] * fast_ex2(gi2 - gam2[j]) * f[j] : 0.f;
        store_row64(sm + OFF_QKM, i, x);
        const float sq = fast_ex2(gi2) * cq;
        float y[64];
        load_row64(kq, 64 + i, y);
#pragma unroll
        for (int j = 0; j < 64; j++) y[j] *= sq;
        store_row64(kq, 64 + i, y);
        load_row64(kq + 16384, 64 + i, y);
#pragma unroll
        for (int j = 0; j < 64; j++) y[j] *= sq;
        store_row64(kq + 16384, 64 + i, y);
      }
      named_bar(1, 128);

      // ---- (I + A)^-1: 16x16 diagonal blocks by forward substitution ----
      if (t < 64) {
        const int blk = t >> 4, cc = t & 15, base = blk * 16;
        float tc[16];
#pragma unroll
        for (int r = 0; r < 16; r++) {
          float s = 0.f;
#pragma unroll
          for (int j = 0; j < r; j++) s = fmaf(Af[(base + r) * 65 + base + j], tc[j], s);
          tc[r] = r == cc ? 1.f : -s;
        }
#pragma unroll
        for (int r = 0; r < 16; r++) Tf[(base + r) * 65 + base + cc] = tc[r];
      } else {
        // The block combines below read whole 32x32 blocks: zero the upper
        // off-diagonal 16x16 blocks (0,1), (2,3) that nothing else writes.
        const int u = t - 64;  // 0..63
        for (int e = u; e < 2 * 256; e += 64) {
          const int blk = e >> 8, r = (e >> 4) & 15, cc = e & 15;
          const int rb = blk * 32, cb = blk * 32 + 16;
          Tf[(rb + r) * 65 + cb + cc] = 0.f;
        }
      }
      named_bar(1, 128);
      // combine into 32x32 blocks: T[2p+1][2p] = -T[2p+1][2p+1] A[2p+1][2p] T[2p][2p]
      {
        const int p = t >> 6, rem = t & 63, r = rem >> 2, c4 = (rem & 3) * 4;
        const int rb = 16 * (2 * p + 1), cb = 16 * (2 * p);
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int k = 0; k < 16; k++) {
          const float av = Af[(rb + r) * 65 + cb + k];
#pragma unroll
          for (int u = 0; u < 4; u++) acc[u] = fmaf(av, Tf[(cb + k) * 65 + cb + c4 + u], acc[u]);
        }
#pragma unroll
        for (int u = 0; u < 4; u++) X1[(p * 16 + r) * 17 + c4 + u] = acc[u];
        named_bar(1, 128);
        float o4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int k = 0; k < 16; k++) {
          const float tv = Tf[(rb + r) * 65 + rb + k];
#pragma unroll
          for (int u = 0; u < 4; u++) o4[u] = fmaf(tv, X1[(p * 16 + k) * 17 + c4 + u], o4[u]);
        }
#pragma unroll
        for (int u = 0; u < 4; u++) Tf[(rb + r) * 65 + cb + c4 + u] = -o4[u];
      }
      named_bar(1, 128);
      // combine into 64x64: T[32:64][0:32] = -T[32:64][32:64] A[32:64][0:32] T[0:32][0:32]
      {
        const int r = t >> 2, c8 = (t & 3) * 8;
        float acc[8];
#pragma unroll
        for (int u = 0; u < 8; u++) acc[u] = 0.f;
#pragma unroll 4
        for (int k = 0; k < 32; k++) {
          const float av = Af[(32 + r) * 65 + k];
#pragma unroll
          for (int u = 0; u < 8; u++) acc[u] = fmaf(av, Tf[k * 65 + c8 + u], acc[u]);
        }
#pragma unroll
        for (int u = 0; u < 8; u++) X2[r * 33 + c8 + u] = acc[u];
        named_bar(1, 128);
#pragma unroll
        for (int u = 0; u < 8; u++) acc[u] = 0.f;
#pragma unroll 4
        for (int k = 0; k < 32; k++) {
          const float tv = Tf[(32 + r) * 65 + 32 + k];
#pragma unroll
          for (int u = 0; u < 8; u++) acc[u] = fmaf(tv, X2[k * 33 + c8 + u], acc[u]);
        }
#pragma unroll
        for (int u = 0; u < 8; u++) Tf[(32 + r) * 65 + c8 + u] = -acc[u];
      }
      named_bar(1, 128);
      if (t < 64) {
        float x[64];
#pragma unroll
        for (int j = 0; j < 64; j++) x[j] = j < t ? Tf[t * 65 + j] : (j == t ? 1.f : 0.f);
        store_row64(sm + OFF_TB, t, x);
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_T);

      // ---- (a) landed: R = diag(beta) (V - diag(Gamma ik) X) ----
      if (!__all_sync(0xffffffffu, mbar_wait(bar_a, c & 1, a.status))) {
        ok = false;
        break;
      }
      tc_fence_after();
      {
        float xr[64];
        tmem_ld64(tmem + lo + TC_X, xr);
        if (lane < 16) {
          const int i = r64;
          float v[64];
          load_row64(vt, i, v);
          const float bi2 = betv[i], ci = fast_ex2(gam2[i]) * ikv[i];
#pragma unroll
          for (int j = 0; j < 64; j++) v[j] = bi2 * fmaf(-ci, xr[j], v[j]);
          store_row64(sm + OFF_RB, i, v);
        }
      }
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_R);

      // ---- (c) landed: Delta copies for (d) and (e); state *= exp(gamma_63) ----
      if (!__all_sync(0xffffffffu, mbar_wait(bar_c, c & 1, a.status))) {
        ok = false;
        break;
      }
      tc_fence_after();
      {
        float dl[64];
        tmem_ld64(tmem + lo + TC_D, dl);
        const float g63 = gam2[63];
        if (lane < 16) {
          const int i = r64;
          store_row64(sm + OFF_DB, i, dl);
          const float si = ikv[i] * fast_ex2(g63 - gam2[i]);
#pragma unroll
          for (int j = 0; j < 64; j++) dl[j] *= si;
          store_row64(sm + OFF_DSB, i, dl);
        }
        float st[64];
        tmem_ld64(tmem + lo + TC_S, st);
        const float dec = fast_ex2(g63);
#pragma unroll
        for (int j = 0; j < 64; j++) st[j] *= dec;
        tmem_st64(tmem + lo + TC_S, st);
      }
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_D);

      // ---- (d) landed: outputs ----
      if (!__all_sync(0xffffffffu, mbar_wait(bar_d, c & 1, a.status))) {
        ok = false;
        break;
      }
      tc_fence_after();
      {
        float o[64];
        tmem_ld64(tmem + lo + TC_O, o);
        const int tok = t0 + r64;
        if (lane < 16 && tok < a.T) {
          float4* dst = reinterpret_cast<float4*>(a.core + (((size_t)b * a.T + tok) * a.NV + h) * GD + dvb * DVB);
#pragma unroll
          for (int i = 0; i < 16; i++) dst[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
        }
      }
      // ---- (e) landed: new state -> bf16 copy for the next chunk ----
      if (!__all_sync(0xffffffffu, mbar_wait(bar_e, c & 1, a.status))) {
        ok = false;
        break;
      }
      tc_fence_after();
      {
        float st[64];
        tmem_ld64(tmem + lo + TC_S, st);
        store_row64(s0b, t, st);
        if (c == a.nchunks - 1) {
          float4* dst = reinterpret_cast<float4*>(a.state_out + (((size_t)b * a.NV + h) * GD + t) * GD + dvb * DVB);
#pragma unroll
          for (int i = 0; i < 16; i++) dst[i] = make_float4(st[4 * i], st[4 * i + 1], st[4 * i + 2], st[4 * i + 3]);
        }
      }
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_s0);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace
}  // namespace hcu

using hcu::fail;

extern "C" int hcu_deltanet_chunked_prefill(hcu_handle h, const hcu_gdn_prefill_params* p, const void* q,
                                            const void* k, const void* v, const float* g, const float* beta,
                                            const float* state_in, float* core, float* state_out) {
  HCU_TRY(hcu::begin_op(h, "hcu_deltanet_chunked_prefill"));
  if (!p || !q || !k || !v || !g || !beta || !core || !state_out || (p->load_state && !state_in))
    return fail(HCU_EINVAL, "hcu_deltanet_chunked_prefill: null argument");
  const long long B = p->B, T = p->T, NK = p->NK, NV = p->NV;
  if (B < 1 || T < 1 || NK < 1 || NV < 1) return fail(HCU_EINVAL, "hcu_deltanet_chunked_prefill: empty shape");
  if (p->D != hcu::GD) return fail(HCU_EUNSUPPORTED, "hcu_deltanet_chunked_prefill: D=%u (built: 128)", p->D);
  if (B > 65535 || NV > 65535) return fail(HCU_EINVAL, "hcu_deltanet_chunked_prefill: B or NV > 65535");
  const long long qrow = p->q_row_stride ? (long long)p->q_row_stride : NK * 128;
  const long long krow = p->k_row_stride ? (long long)p->k_row_stride : NK * 128;
  const long long vrow = p->v_row_stride ? (long long)p->v_row_stride : NV * 128;
  const long long qseq = p->q_seq_stride ? (long long)p->q_seq_stride : T * qrow;
  const long long kseq = p->k_seq_stride ? (long long)p->k_seq_stride : T * krow;
  const long long vseq = p->v_seq_stride ? (long long)p->v_seq_stride : T * vrow;
  if (reinterpret_cast<uintptr_t>(core) % 16 || reinterpret_cast<uintptr_t>(state_out) % 16 ||
      (p->load_state && reinterpret_cast<uintptr_t>(state_in) % 16))
    return fail(HCU_EINVAL, "hcu_deltanet_chunked_prefill: core / state buffers must be 16-byte aligned");
  CUtensorMap tq, tk, tv;
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
  }
  hcu::GdnArgs args{};
  args.B = (int)B;
  args.T = (int)T;
  args.NK = (int)NK;
  args.NV = (int)NV;
  args.load_state = p->load_state ? 1 : 0;
  args.nchunks = (int)((T + hcu::GC - 1) / hcu::GC);
  args.g = g;
  args.beta = beta;
  args.gb_row = p->gb_row_stride ? (long long)p->gb_row_stride : NV;
  args.gb_seq = p->gb_seq_stride ? (long long)p->gb_seq_stride : T * args.gb_row;
  args.state_in = state_in;
  args.core = core;
  args.state_out = state_out;
  args.status = h->dev_status;
  static bool attr_done = false;
  if (!attr_done) {
    HCU_TRY(hcu::check_cuda(cudaFuncSetAttribute(hcu::gdn_chunked_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 hcu::SMEM_BYTES + 1024),
                            "hcu_deltanet_chunked_prefill: smem attribute"));
    attr_done = true;
  }
  hcu::gdn_chunked_kernel<<<dim3(hcu::GD / hcu::DVB, (unsigned)NV, (unsigned)B), hcu::GT_THREADS,
                            hcu::SMEM_BYTES + 1024, h->stream>>>(tq, tk, tv, args);
  return hcu::after_launch("hcu_deltanet_chunked_prefill: launch");
}
