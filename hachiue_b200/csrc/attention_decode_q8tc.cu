// attention_decode_q8tc.cu - tcgen05 split-K decode attention over the
// reference's Q8_0 KV cache (int8 values plus one f32 scale per 32 elements,
// src/engine.ts:483-492), head_dim 128, with int8 tensor-core MMAs
// (kind::i8) reading the cache bytes exactly as TMA lands them: no int8 to
// floating-point conversion pass, no converted copy in shared memory.
//
// Replaces attention_q8 (src/kernels.ts:1341-1426) / runAttentionQ8
// (src/wasm-backend.ts:826-895) on the engine's own cache format.  Same
// split-K / ticket-merge structure and partial format as the other decode
// kernels (attention.cuh).
//
// The arithmetic.  With b the 32-dimension blocks of a head,
//   score_r(t) = sum_b ks[t][b] * (q_r[b] . kq[t][b])
//   o_r[d]     = sum_t p_r(t) * vs[t][b(d)] * vq[t][d]
// * q_r (f32) is scaled by sigma_r = 2^26 / max|q_r|, rounded to an integer
//   and written as four balanced base-128 digits in [-64, 64] (the rounding
//   error is at most 2^-27 max|q_r| per element).  Per tile, one kind::i8 MMA
//   per block b (K = 32 = the block) forms the exact int32 dot products of
//   every digit row with the tile's 128 keys in its own 16-column TMEM group;
//   the softmax thread of key t combines digits and blocks with the K scales
//   in f32.
// * For the output, per tile and block b, y = p * vs[t][b] / max_t vs[t][b]
//   lies in [0, 1]; it is rounded to 21 bits and written as three base-128
//   digits in [0, 127].  The four blocks' digit rows are stacked along N
//   (16 rows each), so ONE MMA chain per tile (M = 128 head dims, N = 64,
//   K = 128 tokens in four K = 32 steps) reads the V tile once, as the
//   MN-major A operand straight from its TMA layout; the thread holding head
//   dimension d reads only the 16 columns of d's block.
// Results keep the fp32 tolerance of the decode path.
//
// Warps (224 threads): 0 loads K tiles + K scales (TMA, 2-slot ring), 1
// allocates TMEM and issues the MMAs (one thread), 2-5 (one TMEM lane each:
// a key of the tile for S, a head dimension for O) run the online softmax and
// accumulate O in registers, 6 loads V tiles + V scales (2-slot ring).  Two
// S and two O accumulators (256 TMEM columns) let Q.K^T of tile j+1 and P.V
// of tile j-1 overlap the softmax of tile j; ~94 KB of shared memory and 256
// columns put two CTAs on an SM.
#include "attention.cuh"
#include "tcgen05.cuh"

namespace hcu {
namespace {

constexpr int Q8_THREADS = 224;
constexpr int Q8_TT = kTcTile;                  // 128 tokens per tile
constexpr int Q8_DH = 128;
constexpr int TILE_BYTES = Q8_TT * Q8_DH;       // 16 KB of int8
constexpr int SC_BYTES = Q8_TT * 4 * 4;         // [128 tokens][4 blocks] f32 scales
constexpr int SLOT_BYTES = TILE_BYTES + SC_BYTES;  // 18 KB, a multiple of 1024
constexpr int KST = 2, VST = 2;
constexpr int NQ = 16;                          // q digit rows: R x 4, padded to 16
constexpr int GP = 16;                          // p digit rows per head-dim block: R x 3, padded
constexpr int NP = 4 * GP;                      // 64
constexpr int QS_BYTES = NQ * 128;
constexpr int PS_BYTES = NP * 128;
constexpr uint32_t TMEM_COLS = 256;
constexpr uint32_t S_COL = 0;                   // 2 buffers x 4 blocks x 16 columns
constexpr uint32_t O_COL = 128;                 // 2 buffers x 64 columns
constexpr float P_ONE = 2097151.f;              // 2^21 - 1
constexpr float Q_ONE = 67108864.f;             // 2^26
constexpr size_t SMEM_BYTES = 1024 + (KST + VST) * SLOT_BYTES + QS_BYTES + 2 * PS_BYTES + 1024;

// An int32 accumulator |x| < 2^22 as f32, exactly, with two ALU operations:
// x added to the bit pattern of 1.5 * 2^23 (whose spacing is 1) is 1.5 * 2^23 + x.
__device__ __forceinline__ float i22f(uint32_t bits) {
  return __int_as_float((int)bits + 0x4B400000) - 12582912.f;
}

template <int R>
__global__ void __launch_bounds__(Q8_THREADS, 2)
    attn_decode_q8tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                            const __grid_constant__ CUtensorMap tmKs, const __grid_constant__ CUtensorMap tmVs,
                            const AttnArgs a) {
  static_assert(R == 1 || R == 2 || R == 4, "rows per CTA");
  static_assert(4 * R <= NQ && 3 * R <= GP, "digit rows");
  constexpr int RB = R + 4;  // per warp and tile: R row maxima, then the 4 blocks' V-scale maxima

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* kslots = smem;                       // KST x [tile | scales]
  uint8_t* vslots = kslots + KST * SLOT_BYTES;  // VST x [tile | scales]
  uint8_t* qs = vslots + VST * SLOT_BYTES;      // [NQ digit rows x 128 dims] int8, SW128
  uint8_t* ps = qs + QS_BYTES;                  // 2 x [NP digit rows x 128 tokens] int8, SW128
  uint64_t* bars = reinterpret_cast<uint64_t*>(ps + 2 * PS_BYTES);
  uint64_t* k_full = bars;       // [KST]
  uint64_t* k_empty = bars + 2;  // [KST]: the QK MMA's commit + the 4 softmax warps (K scales read)
  uint64_t* v_full = bars + 4;   // [VST]
  uint64_t* v_empty = bars + 6;  // [VST]
  uint64_t* s_full = bars + 8;
  uint64_t* s_free = bars + 10;
  uint64_t* p_full = bars + 12;
  uint64_t* o_full = bars + 14;
  uint64_t* o_free = bars + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);
  int* s_last = reinterpret_cast<int*>(tmem_slot + 1);
  float* red = reinterpret_cast<float*>(tmem_slot + 4);  // [2][4 warps][RB]
  float* lred = red + 2 * 4 * RB;                         // [4][R] row sums
  float* qred = lred + 4 * R;                             // [4][R] max |q|

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.x;
  const AttnUnit u = attn_unit(a, split);
  if (u.nsplit > (int)gridDim.x) {
    if (split == 0 && tid == 0) atomicOr(a.status, HCU_DEVERR_BADARG);
    return;
  }
  if (split >= u.nsplit) return;
  const int ntiles = (u.k_hi - u.k_lo + Q8_TT - 1) / Q8_TT;
  const bool softmax_warp = warp >= 2 && warp <= 5;

  if (tid == 0) {
    for (int i = 0; i < 2; i++) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1 + 4);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_free[i], 4);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  // Softmax threads: t = TMEM lane (a key of the tile for S, a head dimension for O).
  const int quarter = warp & 3;
  const int t = quarter * 32 + lane;
  int jlo[R], jhi[R];
  float rs[R];  // score = rs[r] * (sum_b ks_b * digit combination): qscale * smul / sigma_r
  if (softmax_warp) {
    const int sw = warp - 2;
    float qv[R];
#pragma unroll
    for (int r = 0; r < R; r++) {
      const int qi = u.q0 + r / a.G;
      const bool valid = (r < a.QB * a.G) && (r / a.G < u.qn);
      const int pos = u.pb + qi;
      jlo[r] = valid ? ((a.window > 0 && pos + 1 > a.window) ? pos + 1 - a.window : 0) : 1;
      jhi[r] = valid ? pos : 0;
      qv[r] = valid ? __ldg(a.q + out_index(a, u, r, t, Q8_DH)) : 0.f;
      const float mx = warp_max(fabsf(qv[r]));
      if (lane == 0) qred[sw * R + r] = mx;
    }
    named_bar(1, 128);
#pragma unroll
    for (int r = 0; r < R; r++) {
      const float qm = fmaxf(fmaxf(qred[r], qred[R + r]), fmaxf(qred[2 * R + r], qred[3 * R + r]));
      const float sigma = qm > 0.f ? Q_ONE / qm : 0.f;
      rs[r] = qm > 0.f ? a.qscale * a.q8_smul * (qm / Q_ONE) : 0.f;
      int xi = __float2int_rn(qv[r] * sigma);  // |xi| <= 2^26
      int dg[4];
#pragma unroll
      for (int k = 3; k >= 1; k--) {  // balanced digits: xi = d0 2^21 + d1 2^14 + d2 2^7 + d3
        dg[k] = ((xi + 64) & 127) - 64;
        xi = (xi - dg[k]) >> 7;
      }
      dg[0] = xi;
#pragma unroll
      for (int k = 0; k < 4; k++) qs[sw128_offset(r * 4 + k, t)] = (uint8_t)(int8_t)dg[k];
    }
    for (int n = 4 * R; n < NQ; n++) qs[sw128_offset(n, t)] = 0;
    for (int i = t; i < 2 * PS_BYTES / 16; i += 128) reinterpret_cast<uint4*>(ps)[i] = make_uint4(0, 0, 0, 0);
    fence_proxy_async();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool aborted = false;

  if (warp == 0 || warp == 6) {
    // ---------------- TMA producers: warp 0 K, warp 6 V ----------------
    if (lane == 0) {
      const bool isk = warp == 0;
      const CUtensorMap* tm = isk ? &tmK : &tmV;
      const CUtensorMap* tms = isk ? &tmKs : &tmVs;
      uint64_t* full = isk ? k_full : v_full;
      uint64_t* empty = isk ? k_empty : v_empty;
      uint8_t* slots = isk ? kslots : vslots;
      prefetch_tensormap(tm);
      prefetch_tensormap(tms);
      for (int it = 0; it < ntiles; ++it) {
        const int s = it & 1, rnd = it >> 1;
        if (rnd > 0 && !mbar_wait(&empty[s], (rnd - 1) & 1, a.status)) break;
        uint8_t* st = slots + s * SLOT_BYTES;
        const int row = (int)(u.roff + u.k_lo + it * Q8_TT);
        mbar_arrive_expect_tx(&full[s], SLOT_BYTES);
        tma_load_3d(st, tm, &full[s], 0, u.g, row);
        tma_load_3d(st + TILE_BYTES, tms, &full[s], 0, u.g, row);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_s8(128, NQ, false, false);
      constexpr uint32_t idesc_pv = idesc_s8(128, NP, true, false);
      const uint32_t k0 = smem_u32(kslots), v0 = smem_u32(vslots), qs0 = smem_u32(qs), ps0 = smem_u32(ps);
      for (int j = 0; j <= ntiles; ++j) {
        if (j < ntiles) {
          const int s = j & 1, x = j & 1;
          if (!mbar_wait(&k_full[s], (j >> 1) & 1, a.status)) break;
          if (j >= 2 && !mbar_wait(&s_free[x], ((j - 2) >> 1) & 1, a.status)) break;
          tc_fence_after();
          const uint32_t kb = k0 + s * SLOT_BYTES;
#pragma unroll
          for (int b = 0; b < 4; b++) {  // block b = K step b (32 dims = 32 bytes of each row)
            const uint64_t ad = smem_desc_sw128(kb + b * 32, 16, 1024);
            const uint64_t bd = smem_desc_sw128(qs0 + b * 32, 16, 1024);
            mma_s8_ss(tmem + S_COL + x * 64 + b * 16, ad, bd, idesc_qk, 0);
          }
          mma_commit(&s_full[x]);
          mma_commit(&k_empty[s]);
        }
        if (j >= 1) {
          const int jp = j - 1, xp = jp & 1, sv = jp & 1;
          if (!mbar_wait(&v_full[sv], (jp >> 1) & 1, a.status)) break;
          if (!mbar_wait(&p_full[xp], (jp >> 1) & 1, a.status)) break;
          if (jp >= 2 && !mbar_wait(&o_free[xp], ((jp - 2) >> 1) & 1, a.status)) break;
          tc_fence_after();
          const uint32_t vb = v0 + sv * SLOT_BYTES;
          const uint32_t pb = ps0 + xp * PS_BYTES;
#pragma unroll
          for (int ks = 0; ks < 4; ks++) {  // 32 tokens per step: 32 rows of 128 B of V, 32 B of each P row
            const uint64_t ad = smem_desc_sw128(vb + ks * 4096, TILE_BYTES, 1024);  // MN-major V^T
            const uint64_t bd = smem_desc_sw128(pb + ks * 32, 16, 1024);
            mma_s8_ss(tmem + O_COL + xp * 64, ad, bd, idesc_pv, ks > 0);
          }
          mma_commit(&o_full[xp]);
          mma_commit(&v_empty[sv]);
        }
      }
    }
  } else {
    // ---------------- softmax / accumulation (warps 2-5) ----------------
    const int sw = warp - 2;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    float m[R], lsum[R], acc[R], corr0[R], corr1[R];
    float osc0 = 0.f, osc1 = 0.f;  // O scale of the last tile with even / odd index (this thread's block)
#pragma unroll
    for (int r = 0; r < R; r++) {
      m[r] = -1e30f;
      lsum[r] = 0.f;
      acc[r] = 0.f;
      corr0[r] = corr1[r] = 1.f;
    }
    for (int j = 0; j < ntiles + 2; ++j) {
      if (j >= 2) {
        const int jo = j - 2, xo = jo & 1;
        if (!__all_sync(0xffffffffu, mbar_wait(&o_full[xo], (jo >> 1) & 1, a.status))) {
          aborted = true;
          break;
        }
        tc_fence_after();
        uint32_t o[16];
        tmem_ld16(tmem + lane_off + O_COL + xo * 64 + quarter * GP, o);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&o_free[xo]);
        const float osc = xo ? osc1 : osc0;
#pragma unroll
        for (int r = 0; r < R; r++) {
          const float v = fmaf(fmaf(i22f(o[3 * r]), 128.f, i22f(o[3 * r + 1])), 128.f, i22f(o[3 * r + 2]));
          acc[r] = fmaf(acc[r], xo ? corr1[r] : corr0[r], v * osc);
        }
      }
      if (j < ntiles) {
        const int x = j & 1, s = j & 1;
        const bool okw = mbar_wait(&s_full[x], (j >> 1) & 1, a.status) && mbar_wait(&v_full[s], (j >> 1) & 1, a.status);
        if (!__all_sync(0xffffffffu, okw)) {
          aborted = true;
          break;
        }
        tc_fence_after();
        uint32_t sv[64];
        tmem_ld16(tmem + lane_off + S_COL + x * 64, *reinterpret_cast<uint32_t(*)[16]>(sv));
        tmem_ld16(tmem + lane_off + S_COL + x * 64 + 16, *reinterpret_cast<uint32_t(*)[16]>(sv + 16));
        tmem_ld16(tmem + lane_off + S_COL + x * 64 + 32, *reinterpret_cast<uint32_t(*)[16]>(sv + 32));
        tmem_ld16(tmem + lane_off + S_COL + x * 64 + 48, *reinterpret_cast<uint32_t(*)[16]>(sv + 48));
        tmem_ld_wait();
        tc_fence_before();
        const float4 ks = *reinterpret_cast<const float4*>(kslots + s * SLOT_BYTES + TILE_BYTES + t * 16);
        float4 vs = *reinterpret_cast<const float4*>(vslots + s * SLOT_BYTES + TILE_BYTES + t * 16);
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&s_free[x]);
          mbar_arrive(&k_empty[s]);  // the K scales are in registers
        }
        const int key = u.k_lo + j * Q8_TT + t;
        if (key >= u.k_hi) vs = make_float4(0.f, 0.f, 0.f, 0.f);  // rows past the split: any bits
        const float ksb[4] = {ks.x, ks.y, ks.z, ks.w};
        float sc[R];
#pragma unroll
        for (int r = 0; r < R; r++) {
          float dot = 0.f;
#pragma unroll
          for (int b = 0; b < 4; b++) {
            const uint32_t* d = sv + b * 16 + r * 4;
            const float c = fmaf(fmaf(fmaf(i22f(d[0]), 128.f, i22f(d[1])), 128.f, i22f(d[2])), 128.f, i22f(d[3]));
            dot = fmaf(ksb[b], c, dot);
          }
          const bool ok = key >= jlo[r] && key <= jhi[r] && key < u.k_hi;
          sc[r] = ok ? dot * rs[r] : -INFINITY;
          const float mx = warp_max(sc[r]);
          if (lane == 0) red[(x * 4 + sw) * RB + r] = mx;
        }
        {
          const float vb[4] = {warp_max(vs.x), warp_max(vs.y), warp_max(vs.z), warp_max(vs.w)};
          if (lane == 0)
#pragma unroll
            for (int b = 0; b < 4; b++) red[(x * 4 + sw) * RB + R + b] = vb[b];
        }
        named_bar(1, 128);
        float p[R];
#pragma unroll
        for (int r = 0; r < R; r++) {
          float mt = red[(x * 4) * RB + r];
#pragma unroll
          for (int w = 1; w < 4; w++) mt = fmaxf(mt, red[(x * 4 + w) * RB + r]);
          const float mnew = fmaxf(m[r], mt);
          const float corr = exp2f(m[r] - mnew);
          if (x) corr1[r] = corr; else corr0[r] = corr;
          m[r] = mnew;
          p[r] = exp2f(sc[r] - mnew);
          lsum[r] = fmaf(lsum[r], corr, p[r]);
        }
        const float vsb[4] = {vs.x, vs.y, vs.z, vs.w};
        uint8_t* pbuf = ps + x * PS_BYTES;
#pragma unroll
        for (int b = 0; b < 4; b++) {
          float vmax = red[(x * 4) * RB + R + b];
#pragma unroll
          for (int w = 1; w < 4; w++) vmax = fmaxf(vmax, red[(x * 4 + w) * RB + R + b]);
          if (b == quarter) {
            if (x) osc1 = vmax * a.q8_smul * (1.f / P_ONE); else osc0 = vmax * a.q8_smul * (1.f / P_ONE);
          }
          const float f = vmax > 0.f ? vsb[b] / vmax : 0.f;  // in [0, 1]
#pragma unroll
          for (int r = 0; r < R; r++) {
            const int xi = __float_as_int(fmaf(p[r] * f, P_ONE, 12582912.f)) - 0x4B400000;  // round(y (2^21 - 1))
            pbuf[sw128_offset(b * GP + r * 3 + 0, t)] = (uint8_t)(xi >> 14);
            pbuf[sw128_offset(b * GP + r * 3 + 1, t)] = (uint8_t)((xi >> 7) & 127);
            pbuf[sw128_offset(b * GP + r * 3 + 2, t)] = (uint8_t)(xi & 127);
          }
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[x]);
      }
    }
    // row sums over the tile keys
#pragma unroll
    for (int r = 0; r < R; r++) {
      const float v = warp_sum(lsum[r]);
      if (lane == 0) lred[sw * R + r] = v;
    }
    // One decision for the four softmax warps (a bounded wait may give up in
    // some of them only): the merge below synchronises them on named barriers.
    aborted = !named_bar_and(1, 128, !aborted);
#pragma unroll
    for (int r = 0; r < R; r++) lsum[r] = lred[r] + lred[R + r] + lred[2 * R + r] + lred[3 * R + r];
    tc_fence_before();
    __syncthreads();
    if (aborted) {
      // The status word holds the timeout; the unit's tickets stay consistent.
      if (u.nsplit > 1) ticket_merge<R, Q8_DH, 128>(a, u, t, 1, reinterpret_cast<float*>(kslots), s_last);
      return;
    }
    if (u.nsplit == 1) {
#pragma unroll
      for (int r = 0; r < R; r++)
        if (r < u.rows_valid) store_out(a, out_index(a, u, r, t, Q8_DH), acc[r] / lsum[r]);
      return;
    }
    float* part = a.part + ((size_t)u.unit * a.max_splits + split) * R * (Q8_DH + 2);
#pragma unroll
    for (int r = 0; r < R; r++) {
      part[r * (Q8_DH + 2) + t] = acc[r];
      if (t == 0) {
        part[r * (Q8_DH + 2) + Q8_DH] = m[r];
        part[r * (Q8_DH + 2) + Q8_DH + 1] = lsum[r];
      }
    }
    ticket_merge<R, Q8_DH, 128>(a, u, t, 1, reinterpret_cast<float*>(kslots), s_last);
    return;
  }
  // producers and the MMA warp: wait for the softmax warps, then release TMEM
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

template <int R>
int launch(hcu_context* h, const AttnArgs& args, dim3 grid, const CUtensorMap& tk, const CUtensorMap& tv,
           const CUtensorMap& tks, const CUtensorMap& tvs) {
  auto kern = attn_decode_q8tc_kernel<R>;
  static std::atomic<uint64_t> attr_done{0};  // per device
  HCU_TRY(once_per_device(attr_done, h->device, [&]() -> int {
    HCU_TRY(check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES),
                       "hcu_attention: q8 tc smem attribute"));
    return HCU_OK;
  }));
  kern<<<grid, Q8_THREADS, SMEM_BYTES, h->stream>>>(tk, tv, tks, tvs, args);
  return after_launch("hcu_attention: q8 tc launch");
}

}  // namespace

int launch_attn_q8tc(hcu_context* h, int R, const AttnArgs& args, dim3 grid, const CUtensorMap& tk,
                     const CUtensorMap& tv, const CUtensorMap& tks, const CUtensorMap& tvs) {
  switch (R) {
    case 1: return launch<1>(h, args, grid, tk, tv, tks, tvs);
    case 2: return launch<2>(h, args, grid, tk, tv, tks, tvs);
    case 4: return launch<4>(h, args, grid, tk, tv, tks, tvs);
  }
  return fail(HCU_EUNSUPPORTED, "hcu_attention: no Q8_0 tensor-core variant with %d rows", R);
}

}  // namespace hcu
