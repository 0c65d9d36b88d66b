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
// TMA (double-buffered), warp 1 allocates TMEM and issues the MMAs.  Two
// 128-thread warpgroups (one TMEM lane per thread) split the element-wise
// work so consecutive chunks overlap: warps 4-7 prepare the state-independent
// part of chunk c+1 (norms, decays, A, (I+A)^-1, QKm) while warps 8-11 run
// the state-dependent chain of chunk c (R, Delta, outputs, state update).
#include "common.cuh"
#include "context.h"
#include "tcgen05.cuh"

namespace hcu {
namespace {

constexpr int GC = 64;        // chunk length
constexpr int GD = 128;       // DK = DV
constexpr int DVB = 64;       // value columns per CTA
constexpr int GT_THREADS = 384;
// shared memory layout (bytes)
constexpr int KQ_BYTES = 32768;  // per buffer: [d-block 0: K rows 0-63 | Q rows 0-63][d-block 1: same]
constexpr int V_BYTES = 8192;    // per buffer: [64 tokens x 64 values] bf16
constexpr int AS = 68;           // row stride (floats) of the f32 scratch matrices
constexpr int OFF_KQ = 0;
constexpr int OFF_V = OFF_KQ + 2 * KQ_BYTES;
constexpr int OFF_S0B = OFF_V + 2 * V_BYTES;   // [128 dk x 64 dv] bf16, MN-major B operand
constexpr int OFF_TB = OFF_S0B + 16384;        // [2][64 x 64] bf16 (I+A)^-1, K-major A operand
constexpr int OFF_QKM = OFF_TB + 2 * 8192;     // [2][64 x 64] bf16, K-major A operand
constexpr int OFF_RB = OFF_QKM + 2 * 8192;     // [64 tok x 64 dv] bf16, MN-major B operand
constexpr int OFF_DB = OFF_RB + 8192;          // Delta
constexpr int OFF_DSB = OFF_DB + 8192;         // diag(ik exp(g63 - g)) Delta
constexpr int OFF_AF = OFF_DSB + 8192;         // [64][AS] f32 A
constexpr int OFF_TF = OFF_AF + 64 * AS * 4;   // [64][AS] f32 (I+A)^-1
constexpr int OFF_X1 = OFF_TF + 64 * AS * 4;   // [2][16][20] f32
constexpr int OFF_X2 = OFF_X1 + 2 * 16 * 20 * 4;  // [32][36] f32
constexpr int OFF_SC = OFF_X2 + 32 * 36 * 4;   // [2][gam2, beta, ik, iq][64] + misc[16]
constexpr int OFF_BAR = OFF_SC + (2 * 4 * 64 + 16) * 4;
constexpr int NBAR = 16;
constexpr int SMEM_BYTES = OFF_BAR + NBAR * 8 + 16;
// TMEM columns: [K;Q][K;Q]^T (128), K S0, Q S0, Delta, QKm Delta, state (64 each)
constexpr uint32_t TC_F = 0, TC_X = 128, TC_QS = 192, TC_DL = 256, TC_O2 = 320, TC_S = 384, TMEM_COLS = 512;

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

// Value of register-array element `idx` (runtime index) without local memory.
__device__ __forceinline__ float pick64(const float (&x)[64], int idx) {
  float v = 0.f;
#pragma unroll
  for (int j = 0; j < 64; j++) v = j == idx ? x[j] : v;
  return v;
}

__global__ void __launch_bounds__(GT_THREADS, 1)
    gdn_chunked_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const GdnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint64_t* kv_full = bars + 0;   // [2] TMA landed
  uint64_t* kv_empty = bars + 2;  // [2] inputs of a chunk no longer read
  uint64_t* bar_f = bars + 4;     // (f) [K;Q][K;Q]^T done
  uint64_t* f_free = bars + 5;    // prep warps have read (f)
  uint64_t* bar_T = bars + 6;     // [2] prep outputs (scalars, QKm, (I+A)^-1) of a chunk written
  uint64_t* pfree = bars + 8;     // [2] chain warps done with those prep outputs
  uint64_t* bar_a = bars + 10;    // (a) K S0, Q S0 done
  uint64_t* bar_R = bars + 11;    // R written
  uint64_t* bar_c = bars + 12;    // (c) Delta done
  uint64_t* bar_D = bars + 13;    // Delta copies written, state rescaled
  uint64_t* bar_d = bars + 14;    // (d) QKm Delta and (e) state update done
  uint64_t* bar_s0 = bars + 15;   // bf16 state written (and initial state)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NBAR);
  float* Af = reinterpret_cast<float*>(sm + OFF_AF);
  float* Tf = reinterpret_cast<float*>(sm + OFF_TF);
  float* X1 = reinterpret_cast<float*>(sm + OFF_X1);
  float* X2 = reinterpret_cast<float*>(sm + OFF_X2);
  float* scal = reinterpret_cast<float*>(sm + OFF_SC);  // [2][4][64]
  float* misc = scal + 2 * 4 * 64;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int dvb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h % a.NK;
  const int n = a.nchunks;

  if (tid == 0) {
    for (int i = 0; i < 2; i++) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&bar_T[i], 4);
      mbar_init(&pfree[i], 4);
    }
    mbar_init(bar_f, 1);
    mbar_init(f_free, 4);
    mbar_init(bar_a, 1);
    mbar_init(bar_R, 4);
    mbar_init(bar_c, 1);
    mbar_init(bar_D, 4);
    mbar_init(bar_d, 1);
    mbar_init(bar_s0, 4);
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
      for (int c = 0; c < n; c++) {
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
      constexpr uint32_t id_f = idesc_f16(128, 128, true, false, false);  // [K;Q] [K;Q]^T
      constexpr uint32_t id_kb = idesc_f16(64, 64, true, false, true);    // 64-row A (K-major) x MN-major B
      constexpr uint32_t id_e = idesc_f16(128, 64, true, true, true);     // K^T (MN-major) x MN-major B
      const uint32_t s0 = smem_u32(sm);
      auto issue_f = [&](int c) {
        const uint32_t kq = s0 + OFF_KQ + (c & 1) * KQ_BYTES;
#pragma unroll
        for (int ks = 0; ks < 8; ks++) {
          const uint64_t d = smem_desc_sw128(kq + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024);
          mma_f16_ss(tmem + TC_F, d, d, id_f, ks > 0);
        }
        mma_commit(bar_f);
      };
      bool ok = mbar_wait(&kv_full[0], 0, a.status);
      if (ok) {
        tc_fence_after();
        issue_f(0);
      }
      for (int c = 0; c < n && ok; c++) {
        const int buf = c & 1, x = c & 1;
        const uint32_t kq = s0 + OFF_KQ + buf * KQ_BYTES;
        // state-independent MMA of the next chunk, once the prep warps hold chunk c's
        if (c + 1 < n) {
          ok = mbar_wait(&kv_full[(c + 1) & 1], ((c + 1) >> 1) & 1, a.status) && mbar_wait(f_free, c & 1, a.status);
          if (!ok) break;
          tc_fence_after();
          issue_f(c + 1);
        }
        // (a) X = K S0 and QS = Q S0   (M = 64, N = 64, K = 128)
        ok = mbar_wait(bar_s0, c & 1, a.status);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 8; ks++) {
          const uint32_t off = (ks >> 2) * 16384 + (ks & 3) * 32;
          const uint64_t bd = smem_desc_sw128(s0 + OFF_S0B + ks * 2048, 8192, 1024);
          mma_f16_ss(tmem + TC_X, smem_desc_sw128(kq + off, 16, 1024), bd, id_kb, ks > 0);
          mma_f16_ss(tmem + TC_QS, smem_desc_sw128(kq + off + 8192, 16, 1024), bd, id_kb, ks > 0);
        }
        mma_commit(bar_a);
        // (c) Delta = (I+A)^-1 R   (M = 64, N = 64, K = 64)
        ok = mbar_wait(bar_R, c & 1, a.status);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 4; ks++)
          mma_f16_ss(tmem + TC_DL, smem_desc_sw128(s0 + OFF_TB + x * 8192 + ks * 32, 16, 1024),
                     smem_desc_sw128(s0 + OFF_RB + ks * 2048, 8192, 1024), id_kb, ks > 0);
        mma_commit(bar_c);
        // (d) O2 = QKm Delta; (e) S += K^T Dsb   (S pre-scaled by the chain warps)
        ok = mbar_wait(bar_D, c & 1, a.status);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 4; ks++) {
          mma_f16_ss(tmem + TC_O2, smem_desc_sw128(s0 + OFF_QKM + x * 8192 + ks * 32, 16, 1024),
                     smem_desc_sw128(s0 + OFF_DB + ks * 2048, 8192, 1024), id_kb, ks > 0);
          mma_f16_ss(tmem + TC_S, smem_desc_sw128(kq + ks * 2048, 16384, 1024),
                     smem_desc_sw128(s0 + OFF_DSB + ks * 2048, 8192, 1024), id_e, 1);
        }
        mma_commit(bar_d);
        mma_commit(&kv_empty[buf]);
      }
    }
  } else if (warp >= 4 && warp < 8) {
    // ---------------- prep warpgroup: state-independent part of each chunk ----------------
    const int t = (warp - 4) * 32 + lane;
    const uint32_t lo = (uint32_t)((warp - 4) * 32) << 16;
    const float inv_sqrt_d = rsqrtf((float)GD);
    for (int c = 0; c < n; c++) {
      const int x = c & 1;
      float* gam2 = scal + x * 256;
      float* betv = gam2 + 64;
      float* ikv = gam2 + 128;
      float* iqv = gam2 + 192;
      if (!__all_sync(0xffffffffu, mbar_wait(bar_f, c & 1, a.status))) break;
      tc_fence_after();
      float f[64], dg[64];
      tmem_ld64(tmem + lo + TC_F, f);         // G row t (t < 64) / P row t-64
      tmem_ld64(tmem + lo + TC_F + 64, dg);   // K Q^T row / Q Q^T row
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(f_free);
      const float nrm2 = t < 64 ? pick64(f, t) : pick64(dg, t - 64);  // |k_t|^2 or |q_t-64|^2
      float gi = 0.f, bi = 0.f;
      const int t0 = c * GC;
      if (t < 64 && t0 + t < a.T) {
        const size_t idx = (size_t)b * a.gb_seq + (size_t)(t0 + t) * a.gb_row + h;
        gi = __ldg(a.g + idx);
        bi = __ldg(a.beta + idx);
      }
      if (c >= 2 && !__all_sync(0xffffffffu, mbar_wait(&pfree[x], ((c - 2) >> 1) & 1, a.status))) break;
      if (t < 64) {
        float sc = gi;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_up_sync(0xffffffffu, sc, o);
          if (lane >= o) sc += y;
        }
        if (t == 31) misc[x] = sc;
        gi = sc;
      }
      named_bar(2, 128);
      if (t < 64) {
        gam2[t] = (gi + (t >= 32 ? misc[x] : 0.f)) * kLog2e;
        betv[t] = bi;
        ikv[t] = rsqrtf(nrm2 + 1e-6f);
      } else {
        iqv[t - 64] = rsqrtf(nrm2 + 1e-6f) * inv_sqrt_d;
      }
      named_bar(2, 128);
      if (t < 64) {
        // A (strictly lower), f32
        const float gi2 = gam2[t], cb = betv[t] * ikv[t];
#pragma unroll
        for (int j = 0; j < 64; j++) Af[t * AS + j] = j < t ? cb * ikv[j] * fast_ex2(gi2 - gam2[j]) * f[j] : 0.f;
      } else {
        // QKm row (lower including the diagonal), bf16
        const int i = t - 64;
        const float gi2 = gam2[i], cq = iqv[i];
        float y[64];
#pragma unroll
        for (int j = 0; j < 64; j++) y[j] = j <= i ? cq * ikv[j] * fast_ex2(gi2 - gam2[j]) * f[j] : 0.f;
        store_row64(sm + OFF_QKM + x * 8192, i, y);
      }
      named_bar(2, 128);
      // (I + A)^-1: 16x16 diagonal blocks by forward substitution
      if (t < 64) {
        const int base = (t >> 4) * 16, cc = t & 15;
        float tc[16];
#pragma unroll
        for (int r = 0; r < 16; r++) {
          float s = 0.f;
#pragma unroll
          for (int j = 0; j < r; j++) s = fmaf(Af[(base + r) * AS + base + j], tc[j], s);
          tc[r] = r == cc ? 1.f : -s;
        }
#pragma unroll
        for (int r = 0; r < 16; r++) Tf[(base + r) * AS + base + cc] = tc[r];
      } else {
        // zero the upper off-diagonal 16x16 blocks (0,1) and (2,3): the
        // combines below read whole 32x32 blocks
        for (int e = t - 64; e < 512; e += 64) {
          const int blk = e >> 8, r = (e >> 4) & 15, cc = e & 15;
          Tf[(blk * 32 + r) * AS + blk * 32 + 16 + cc] = 0.f;
        }
      }
      named_bar(2, 128);
      {
        // 32x32 blocks: T[2p+1][2p] = -T[2p+1][2p+1] A[2p+1][2p] T[2p][2p]
        const int p = t >> 6, rem = t & 63, r = rem >> 2, c4 = (rem & 3) * 4;
        const int rb = 16 * (2 * p + 1), cb = 16 * (2 * p);
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int k = 0; k < 16; k++) {
          const float av = Af[(rb + r) * AS + cb + k];
          const float4 tv = *reinterpret_cast<const float4*>(&Tf[(cb + k) * AS + cb + c4]);
          acc.x = fmaf(av, tv.x, acc.x);
          acc.y = fmaf(av, tv.y, acc.y);
          acc.z = fmaf(av, tv.z, acc.z);
          acc.w = fmaf(av, tv.w, acc.w);
        }
        *reinterpret_cast<float4*>(&X1[(p * 16 + r) * 20 + c4]) = acc;
        named_bar(2, 128);
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
        *reinterpret_cast<float4*>(&Tf[(rb + r) * AS + cb + c4]) = make_float4(-o.x, -o.y, -o.z, -o.w);
      }
      named_bar(2, 128);
      {
        // 64x64: T[32:64][0:32] = -T[32:64][32:64] A[32:64][0:32] T[0:32][0:32]
        const int r = t >> 2, c8 = (t & 3) * 8;
        float acc[8];
#pragma unroll
        for (int u = 0; u < 8; u++) acc[u] = 0.f;
#pragma unroll 8
        for (int k = 0; k < 32; k++) {
          const float av = Af[(32 + r) * AS + k];
          const float4 t0v = *reinterpret_cast<const float4*>(&Tf[k * AS + c8]);
          const float4 t1v = *reinterpret_cast<const float4*>(&Tf[k * AS + c8 + 4]);
          acc[0] = fmaf(av, t0v.x, acc[0]);
          acc[1] = fmaf(av, t0v.y, acc[1]);
          acc[2] = fmaf(av, t0v.z, acc[2]);
          acc[3] = fmaf(av, t0v.w, acc[3]);
          acc[4] = fmaf(av, t1v.x, acc[4]);
          acc[5] = fmaf(av, t1v.y, acc[5]);
          acc[6] = fmaf(av, t1v.z, acc[6]);
          acc[7] = fmaf(av, t1v.w, acc[7]);
        }
        *reinterpret_cast<float4*>(&X2[r * 36 + c8]) = make_float4(acc[0], acc[1], acc[2], acc[3]);
        *reinterpret_cast<float4*>(&X2[r * 36 + c8 + 4]) = make_float4(acc[4], acc[5], acc[6], acc[7]);
        named_bar(2, 128);
#pragma unroll
        for (int u = 0; u < 8; u++) acc[u] = 0.f;
#pragma unroll 8
        for (int k = 0; k < 32; k++) {
          const float tv = Tf[(32 + r) * AS + 32 + k];
          const float4 x0 = *reinterpret_cast<const float4*>(&X2[k * 36 + c8]);
          const float4 x1 = *reinterpret_cast<const float4*>(&X2[k * 36 + c8 + 4]);
          acc[0] = fmaf(tv, x0.x, acc[0]);
          acc[1] = fmaf(tv, x0.y, acc[1]);
          acc[2] = fmaf(tv, x0.z, acc[2]);
          acc[3] = fmaf(tv, x0.w, acc[3]);
          acc[4] = fmaf(tv, x1.x, acc[4]);
          acc[5] = fmaf(tv, x1.y, acc[5]);
          acc[6] = fmaf(tv, x1.z, acc[6]);
          acc[7] = fmaf(tv, x1.w, acc[7]);
        }
        *reinterpret_cast<float4*>(&Tf[(32 + r) * AS + c8]) = make_float4(-acc[0], -acc[1], -acc[2], -acc[3]);
        *reinterpret_cast<float4*>(&Tf[(32 + r) * AS + c8 + 4]) = make_float4(-acc[4], -acc[5], -acc[6], -acc[7]);
      }
      named_bar(2, 128);
      if (t < 64) {
        float y[64];
#pragma unroll
        for (int j = 0; j < 64; j++) y[j] = j < t ? Tf[t * AS + j] : (j == t ? 1.f : 0.f);
        store_row64(sm + OFF_TB + x * 8192, t, y);
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_T[x]);
    }
  } else if (warp >= 8) {
    // ---------------- chain warpgroup: state-dependent part of each chunk ----------------
    const int q4 = warp - 8;
    const int t = q4 * 32 + lane;            // state row (dk) for M = 128 accumulators
    const uint32_t lo = (uint32_t)(q4 * 32) << 16;
    const int r64 = q4 * 16 + lane;          // row of an M = 64 accumulator (valid when lane < 16)
    uint8_t* s0b = sm + OFF_S0B;
    {
      float st[64];
      if (a.load_state) {
        const float4* src = reinterpret_cast<const float4*>(
            a.state_in + (((size_t)b * a.NV + h) * GD + t) * GD + dvb * DVB);
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
      tmem_st64(tmem + lo + TC_S, st);
      store_row64(s0b, t, st);
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_s0);
    }
    for (int c = 0; c < n; c++) {
      const int x = c & 1;
      const float* gam2 = scal + x * 256;
      const float* betv = gam2 + 64;
      const float* ikv = gam2 + 128;
      const float* iqv = gam2 + 192;
      const uint8_t* vt = sm + OFF_V + (c & 1) * V_BYTES;
      // R = diag(beta) (V - diag(Gamma ik) K S0)
      if (!__all_sync(0xffffffffu, mbar_wait(bar_a, c & 1, a.status))) break;
      tc_fence_after();
      float xr[64];
      tmem_ld64(tmem + lo + TC_X, xr);
      if (!__all_sync(0xffffffffu, mbar_wait(&bar_T[x], (c >> 1) & 1, a.status))) break;
      if (lane < 16) {
        const int i = r64;
        float v[64];
        load_row64(vt, i, v);
        const float bi = betv[i], ci = fast_ex2(gam2[i]) * ikv[i];
#pragma unroll
        for (int j = 0; j < 64; j++) v[j] = bi * fmaf(-ci, xr[j], v[j]);
        store_row64(sm + OFF_RB, i, v);
      }
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_R);
      // Delta for (d) and (e); state *= exp(gamma_63)
      if (!__all_sync(0xffffffffu, mbar_wait(bar_c, c & 1, a.status))) break;
      tc_fence_after();
      const float g63 = gam2[63];
      {
        float dl[64];
        tmem_ld64(tmem + lo + TC_DL, dl);
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
      // outputs O = diag(Gamma iq) Q S0 + QKm Delta, and the next bf16 state
      if (!__all_sync(0xffffffffu, mbar_wait(bar_d, c & 1, a.status))) break;
      tc_fence_after();
      {
        float qs[64], o2[64];
        tmem_ld64(tmem + lo + TC_QS, qs);
        tmem_ld64(tmem + lo + TC_O2, o2);
        const int tok = c * GC + r64;
        if (lane < 16 && tok < a.T) {
          const float cq = fast_ex2(gam2[r64]) * iqv[r64];
          float4* dst = reinterpret_cast<float4*>(a.core + (((size_t)b * a.T + tok) * a.NV + h) * GD + dvb * DVB);
#pragma unroll
          for (int i = 0; i < 16; i++)
            dst[i] = make_float4(fmaf(cq, qs[4 * i], o2[4 * i]), fmaf(cq, qs[4 * i + 1], o2[4 * i + 1]),
                                 fmaf(cq, qs[4 * i + 2], o2[4 * i + 2]), fmaf(cq, qs[4 * i + 3], o2[4 * i + 3]));
        }
        float st[64];
        tmem_ld64(tmem + lo + TC_S, st);
        store_row64(s0b, t, st);
        if (c == n - 1) {
          float4* dst = reinterpret_cast<float4*>(a.state_out + (((size_t)b * a.NV + h) * GD + t) * GD + dvb * DVB);
#pragma unroll
          for (int i = 0; i < 16; i++) dst[i] = make_float4(st[4 * i], st[4 * i + 1], st[4 * i + 2], st[4 * i + 3]);
        }
      }
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(bar_s0);
        mbar_arrive(&pfree[x]);
      }
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
