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
// * q_r (f32) is scaled by sigma_r = 2^20 / max|q_r|, rounded to an integer
//   and written as three balanced base-128 digits in [-64, 64] (the rounding
//   error is at most 2^-21 max|q_r| per element).  Per tile, one kind::i8 MMA
//   per block b (K = 32 = the block) forms the exact int32 dot products of
//   every digit row with the tile's 128 keys in its own 16-column TMEM group;
//   the softmax thread of key t combines digits and blocks with the K scales
//   in f32.
// * For the output, per tile and block b, y = p * vs[t][b] / max_t vs[t][b]
//   lies in [0, 1]; it is rounded to 22 bits, whose three bytes are the
//   unsigned base-256 digits (a u8 B operand).  The four blocks' digit columns are stacked along N
//   (16 each), so ONE MMA chain per tile (M = 128 head dims, N = 64,
//   K = 128 tokens in four K = 32 steps) reads the V tile once, as the
//   MN-major A operand straight from its TMA layout; the thread holding head
//   dimension d reads only the 16 columns of d's block.  P is the MN-major B
//   operand (64-byte rows, one per key, 64-byte swizzle), so the thread of key
//   t writes its digits of a block as one 8-byte store.
// Results keep the fp32 tolerance of the decode path.
//
// Warps: 0 loads K tiles with the K and V scales of the tile (TMA, 3-slot
// ring), 1 allocates TMEM and issues the MMAs (one thread), then one or two
// softmax warpgroups (one TMEM lane each: a key of the tile for S, a head
// dimension for O) that run the online softmax and accumulate O in registers,
// then a warp loading V tiles (2-slot ring).  The softmax of a tile needs its
// V scales but not its V values: carrying the V scales in the K slot, which
// the softmax frees as soon as it has read them, keeps the V ring's longer
// round trip (a V slot frees only when P.V has read it) off the softmax's
// path.  With R >= 2 the rows are split between two
// warpgroups (R / 2 each): every tile's softmax work per thread halves and
// each SM sub-partition holds twice the softmax warps, which hides the
// latency of the per-tile chain (TMEM load, digit combination, maxima, exp2,
// digit stores).  The digit rows are laid out so that warpgroup w owns
// columns 8w .. 8w+7 of every 16-column group.  Two S and two O accumulators
// (256 TMEM columns) let Q.K^T of tile j+1 and P.V of tile j-1 overlap the
// softmax of tile j; ~94 KB of shared memory and 256 columns put two CTAs on
// an SM.
#include "attention.cuh"
#include "tcgen05.cuh"

namespace hcu {
namespace {

constexpr int Q8_TT = kTcTile;                  // 128 tokens per tile
constexpr int Q8_DH = 128;
constexpr int TILE_BYTES = Q8_TT * Q8_DH;       // 16 KB of int8
constexpr int SC_BYTES = Q8_TT * 4 * 4;         // [128 tokens][4 blocks] f32 scales
constexpr int KSLOT_BYTES = TILE_BYTES + 2 * SC_BYTES;  // K tile, K scales, V scales: 20 KB
constexpr int VSLOT_BYTES = TILE_BYTES;                 // V tile
constexpr int KST = 3, VST = 2;
constexpr int NQD = 3;                          // q digits per row
constexpr int NQ = 16;                          // q digit rows (8 per warpgroup)
constexpr int GP = 16;                          // p digit rows per head-dim block (8 per warpgroup)
constexpr int NP = 4 * GP;                      // 64
constexpr int QS_BYTES = NQ * 128;
constexpr int PS_BYTES = NP * Q8_TT;             // [128 keys][64 digit columns] int8
constexpr uint32_t TMEM_COLS = 256;
constexpr uint32_t S_COL = 0;                   // 2 buffers x 4 blocks x 16 columns
constexpr uint32_t O_COL = 128;                 // 2 buffers x 64 columns
constexpr float P_ONE = 4194303.f;              // 2^22 - 1: y (2^22 - 1) rounds with the 1.5 * 2^23 trick
constexpr float Q_ONE = 1048576.f;              // 2^20
constexpr size_t SMEM_BYTES = 1024 + KST * KSLOT_BYTES + VST * VSLOT_BYTES + QS_BYTES + 2 * PS_BYTES + 1024;
static_assert(KSLOT_BYTES % 1024 == 0 && VSLOT_BYTES % 1024 == 0, "slot alignment");
static_assert(2 * (SMEM_BYTES + 1024) <= 228 * 1024, "two CTAs per SM");

__host__ __device__ constexpr int nwg_of(int R) { return R >= 2 ? 2 : 1; }
__host__ __device__ constexpr int threads_of(int R) { return 32 * (3 + 4 * nwg_of(R)); }

// An int32 accumulator |x| < 2^22 as f32, exactly, with two ALU operations:
// x added to the bit pattern of 1.5 * 2^23 (whose spacing is 1) is 1.5 * 2^23 + x.
__device__ __forceinline__ float i22f(uint32_t bits) {
  return __int_as_float((int)bits + 0x4B400000) - 12582912.f;
}

template <int R>
__global__ void __launch_bounds__(threads_of(R), 2)
    attn_decode_q8tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                            const __grid_constant__ CUtensorMap tmKs, const __grid_constant__ CUtensorMap tmVs,
                            const AttnArgs a) {
  static_assert(R == 1 || R == 2 || R == 4, "rows per CTA");
  constexpr int NWG = nwg_of(R);   // softmax warpgroups
  constexpr int RL = R / NWG;      // rows per warpgroup
  constexpr int NSW = 4 * NWG;     // softmax warps
  constexpr int VWARP = 2 + NSW;   // V producer warp
  static_assert(NQD * RL <= 8 && 3 * RL <= 8 && RL <= 2, "digit rows of a warpgroup");
  constexpr int RB = 8;  // per warp and tile: the 4 blocks' V-scale maxima (16-B aligned), then RL row maxima

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* kslots = smem;                        // KST x [K tile | K scales | V scales]
  uint8_t* vslots = kslots + KST * KSLOT_BYTES;  // VST x [V tile]
  uint8_t* qs = vslots + VST * VSLOT_BYTES;      // [NQ digit rows x 128 dims] int8, SW128
  uint8_t* ps = qs + QS_BYTES;                   // 2 x [128 keys x NP digit columns] int8, SW64
  uint64_t* bars = reinterpret_cast<uint64_t*>(ps + 2 * PS_BYTES);
  uint64_t* k_full = bars;       // [KST]
  uint64_t* k_empty = bars + 3;  // [KST]: the QK MMA's commit + the softmax warps (scales read)
  uint64_t* v_full = bars + 6;   // [VST]
  uint64_t* v_empty = bars + 8;  // [VST]
  uint64_t* s_full = bars + 10;
  uint64_t* s_free = bars + 12;
  uint64_t* p_full = bars + 14;
  uint64_t* o_full = bars + 16;
  uint64_t* o_free = bars + 18;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 20);
  int* s_last = reinterpret_cast<int*>(tmem_slot + 1);
  float* red_all = reinterpret_cast<float*>(tmem_slot + 4);  // [NWG][2][4 warps][RB]
  float* lred_all = red_all + NWG * 2 * 4 * RB;               // [NWG][4][RL] row sums
  float* qred_all = lred_all + NWG * 4 * RL;                  // [NWG][4][RL] max |q|

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.x;
  const AttnUnit u = attn_unit(a, split);
  const bool softmax_warp = warp >= 2 && warp < 2 + NSW;
  // In the cluster form every CTA of the unit's cluster reaches the two
  // cluster barriers; a CTA without work only contributes an empty partial.
  const bool clus = a.cluster != 0;
  const bool badarg = u.nsplit > (int)gridDim.x;
  if (badarg && split == 0 && tid == 0) atomicOr(a.status, HCU_DEVERR_BADARG);
  if (badarg || split >= u.nsplit) {
    if (!clus) return;
    float* cp = reinterpret_cast<float*>(kslots);  // [R][Dh + 2]: acc, m, l
    for (int e = tid; e < R * (Q8_DH + 2); e += threads_of(R)) cp[e] = e % (Q8_DH + 2) == Q8_DH ? -1e30f : 0.f;
    cluster_sync_all();
    if (softmax_warp)
      cluster_merge<R, Q8_DH, 32 * NSW>(a, u, badarg ? 0 : min(u.nsplit, (int)gridDim.x), cp, tid - 64, !badarg);
    cluster_sync_all();
    return;
  }
  const int ntiles = (u.k_hi - u.k_lo + Q8_TT - 1) / Q8_TT;

  if (tid == 0) {
    for (int i = 0; i < KST; i++) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1 + NSW);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], NSW);
      mbar_init(&p_full[i], NSW);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_free[i], NSW);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  // Softmax threads: warpgroup wg, warp sw of it; t = TMEM lane (a key of the
  // tile for S, a head dimension for O).  Row i of the warpgroup is row
  // r = wg * RL + i of the CTA; its digits sit at row / column 8 wg + 3 i + k
  // of each 16-wide group.
  const int quarter = warp & 3;
  const int t = quarter * 32 + lane;
  const int wg = softmax_warp ? (warp - 2) >> 2 : 0;
  const int sw = (warp - 2) & 3;
  float* red = red_all + wg * 2 * 4 * RB;
  float* lred = lred_all + wg * 4 * RL;
  float* qred = qred_all + wg * 4 * RL;
  const uint32_t wbar = 1 + wg;  // this warpgroup's named barrier
  int jlo[RL], jhi[RL];
  float rs[RL];  // score = rs[i] * (sum_b ks_b * digit combination): qscale * smul / sigma
  if (softmax_warp) {
    float qv[RL];
#pragma unroll
    for (int i = 0; i < RL; i++) {
      const int r = wg * RL + i;
      const int qi = u.q0 + r / a.G;
      const bool valid = (r < a.QB * a.G) && (r / a.G < u.qn);
      const int pos = u.pb + qi;
      jlo[i] = valid ? ((a.window > 0 && pos + 1 > a.window) ? pos + 1 - a.window : 0) : 1;
      jhi[i] = valid ? pos : 0;
      qv[i] = valid ? __ldg(a.q + out_index(a, u, r, t, Q8_DH)) : 0.f;
      const float mx = warp_max_nonneg(fabsf(qv[i]));
      if (lane == 0) qred[sw * RL + i] = mx;
    }
    named_bar(wbar, 128);
#pragma unroll
    for (int i = 0; i < RL; i++) {
      const float qm = fmaxf(fmaxf(qred[i], qred[RL + i]), fmaxf(qred[2 * RL + i], qred[3 * RL + i]));
      const float sigma = qm > 0.f ? Q_ONE / qm : 0.f;
      rs[i] = qm > 0.f ? a.qscale * a.q8_smul * (qm / Q_ONE) : 0.f;
      int xi = __float2int_rn(qv[i] * sigma);  // |xi| <= 2^20
      int dg[NQD];
#pragma unroll
      for (int k = NQD - 1; k >= 1; k--) {  // balanced digits: xi = d0 2^14 + d1 2^7 + d2
        dg[k] = ((xi + 64) & 127) - 64;
        xi = (xi - dg[k]) >> 7;
      }
      dg[0] = xi;
#pragma unroll
      for (int k = 0; k < NQD; k++) qs[sw128_offset(wg * 8 + i * NQD + k, t)] = (uint8_t)(int8_t)dg[k];
    }
    for (int n = NQD * RL; n < 8; n++) qs[sw128_offset(wg * 8 + n, t)] = 0;
    if (NWG == 1)
      for (int n = 8; n < NQ; n++) qs[sw128_offset(n, t)] = 0;
    for (int i = (tid - 64); i < 2 * PS_BYTES / 16; i += 32 * NSW) reinterpret_cast<uint4*>(ps)[i] = make_uint4(0, 0, 0, 0);
    fence_proxy_async();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool aborted = false;

  if (warp == 0 || warp == VWARP) {
    // ---------------- TMA producers: warp 0 K, the last warp V ----------------
    if (lane == 0 && warp == 0) {
      prefetch_tensormap(&tmK);
      prefetch_tensormap(&tmKs);
      prefetch_tensormap(&tmVs);
      for (int it = 0; it < ntiles; ++it) {
        const int s = it % KST, rnd = it / KST;
        if (rnd > 0 && !mbar_wait(&k_empty[s], (rnd - 1) & 1, a.status)) break;
        uint8_t* st = kslots + s * KSLOT_BYTES;
        const int row = (int)(u.roff + u.k_lo + it * Q8_TT);
        mbar_arrive_expect_tx(&k_full[s], KSLOT_BYTES);
        tma_load_3d(st, &tmK, &k_full[s], 0, u.g, row);
        tma_load_3d(st + TILE_BYTES, &tmKs, &k_full[s], 0, u.g, row);
        tma_load_3d(st + TILE_BYTES + SC_BYTES, &tmVs, &k_full[s], 0, u.g, row);
      }
    } else if (lane == 0) {
      prefetch_tensormap(&tmV);
      for (int it = 0; it < ntiles; ++it) {
        const int s = it & 1, rnd = it >> 1;
        if (rnd > 0 && !mbar_wait(&v_empty[s], (rnd - 1) & 1, a.status)) break;
        const int row = (int)(u.roff + u.k_lo + it * Q8_TT);
        mbar_arrive_expect_tx(&v_full[s], VSLOT_BYTES);
        tma_load_3d(vslots + s * VSLOT_BYTES, &tmV, &v_full[s], 0, u.g, row);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_s8(128, NQ, false, false);
      constexpr uint32_t idesc_pv = idesc_s8(128, NP, true, true, true);
      const uint32_t k0 = smem_u32(kslots), v0 = smem_u32(vslots), qs0 = smem_u32(qs), ps0 = smem_u32(ps);
      for (int j = 0; j <= ntiles; ++j) {
        if (j < ntiles) {
          const int s = j % KST, x = j & 1;
          if (!mbar_wait_poll(&k_full[s], (j / KST) & 1, a.status)) break;
          if (j >= 2 && !mbar_wait_poll(&s_free[x], ((j - 2) >> 1) & 1, a.status)) break;
          tc_fence_after();
          const uint32_t kb = k0 + s * KSLOT_BYTES;
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
          if (!mbar_wait_poll(&v_full[sv], (jp >> 1) & 1, a.status)) break;
          if (!mbar_wait_poll(&p_full[xp], (jp >> 1) & 1, a.status)) break;
          if (jp >= 2 && !mbar_wait_poll(&o_free[xp], ((jp - 2) >> 1) & 1, a.status)) break;
          tc_fence_after();
          const uint32_t vb = v0 + sv * VSLOT_BYTES;
          const uint32_t pb = ps0 + xp * PS_BYTES;
#pragma unroll
          for (int ks = 0; ks < 4; ks++) {  // 32 tokens per step: 32 rows of 128 B of V, 32 rows of 64 B of P
            const uint64_t ad = smem_desc_sw128(vb + ks * 4096, TILE_BYTES, 1024);  // MN-major V^T
            const uint64_t bd = smem_desc_sw64(pb + ks * 2048, PS_BYTES, 512);       // MN-major P^T
            mma_s8_ss(tmem + O_COL + xp * 64, ad, bd, idesc_pv, ks > 0);
          }
          mma_commit(&o_full[xp]);
          mma_commit(&v_empty[sv]);
        }
      }
    }
  } else {
    // ---------------- softmax / accumulation ----------------
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int stid = tid - 64;  // 0 .. 32 NSW - 1
    float m[RL], lsum[RL], acc[RL], corr0[RL], corr1[RL];
    float osc0 = 0.f, osc1 = 0.f;  // O scale of the last tile with even / odd index (this thread's block)
#pragma unroll
    for (int i = 0; i < RL; i++) {
      m[i] = -1e30f;
      lsum[i] = 0.f;
      acc[i] = 0.f;
      corr0[i] = corr1[i] = 1.f;
    }
    for (int j = 0; j < ntiles + 2; ++j) {
      if (j >= 2) {
        const int jo = j - 2, xo = jo & 1;
        if (!__all_sync(0xffffffffu, mbar_wait(&o_full[xo], (jo >> 1) & 1, a.status))) {
          aborted = true;
          break;
        }
        tc_fence_after();
        uint32_t o[8];
        tmem_ld8(tmem + lane_off + O_COL + xo * 64 + quarter * GP + wg * 8, o);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&o_free[xo]);
        const float osc = xo ? osc1 : osc0;
#pragma unroll
        for (int i = 0; i < RL; i++) {
          const float v = fmaf(fmaf(i22f(o[3 * i + 2]), 256.f, i22f(o[3 * i + 1])), 256.f, i22f(o[3 * i]));
          acc[i] = fmaf(acc[i], xo ? corr1[i] : corr0[i], v * osc);
        }
      }
      if (j < ntiles) {
        const int x = j & 1, s = j % KST;
        // S(j) complete implies K slot s (K values and both scales) landed:
        // Q.K^T(j) was issued after k_full.
        if (!__all_sync(0xffffffffu, mbar_wait(&s_full[x], (j >> 1) & 1, a.status))) {
          aborted = true;
          break;
        }
        tc_fence_after();
        uint32_t sv[32];
#pragma unroll
        for (int b = 0; b < 4; b++) tmem_ld8(tmem + lane_off + S_COL + x * 64 + b * 16 + wg * 8, sv + 8 * b);
        tmem_ld_wait();
        tc_fence_before();
        const float4 ks = *reinterpret_cast<const float4*>(kslots + s * KSLOT_BYTES + TILE_BYTES + t * 16);
        float4 vs = *reinterpret_cast<const float4*>(kslots + s * KSLOT_BYTES + TILE_BYTES + SC_BYTES + t * 16);
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&s_free[x]);
          mbar_arrive(&k_empty[s]);  // both scales are in registers
        }
        const int key = u.k_lo + j * Q8_TT + t;
        if (key >= u.k_hi) vs = make_float4(0.f, 0.f, 0.f, 0.f);  // rows past the split: any bits
        const float ksb[4] = {ks.x, ks.y, ks.z, ks.w};
        float sc[RL];
#pragma unroll
        for (int i = 0; i < RL; i++) {
          float dot = 0.f;
#pragma unroll
          for (int b = 0; b < 4; b++) {
            const uint32_t* d = sv + b * 8 + i * NQD;
            const float c = fmaf(fmaf(i22f(d[0]), 128.f, i22f(d[1])), 128.f, i22f(d[2]));
            dot = fmaf(ksb[b], c, dot);
          }
          const bool ok = key >= jlo[i] && key <= jhi[i] && key < u.k_hi;
          sc[i] = ok ? dot * rs[i] : -INFINITY;
          const float mx = warp_max_redux(sc[i]);
          if (lane == 0) red[(x * 4 + sw) * RB + 4 + i] = mx;
        }
        {
          const float vb[4] = {warp_max_nonneg(vs.x), warp_max_nonneg(vs.y), warp_max_nonneg(vs.z),
                               warp_max_nonneg(vs.w)};
          if (lane == 0)
            *reinterpret_cast<float4*>(red + (x * 4 + sw) * RB) = make_float4(vb[0], vb[1], vb[2], vb[3]);
        }
        named_bar(wbar, 128);
        float p[RL];
#pragma unroll
        for (int i = 0; i < RL; i++) {
          float mt = red[(x * 4) * RB + 4 + i];
#pragma unroll
          for (int w = 1; w < 4; w++) mt = fmaxf(mt, red[(x * 4 + w) * RB + 4 + i]);
          const float mnew = fmaxf(m[i], mt);
          const float corr = ex2_approx(m[i] - mnew);
          if (x) corr1[i] = corr; else corr0[i] = corr;
          m[i] = mnew;
          p[i] = ex2_approx(sc[i] - mnew);
          lsum[i] = fmaf(lsum[i], corr, p[i]);
        }
        const float vsb[4] = {vs.x, vs.y, vs.z, vs.w};
        float vmx[4];
        {
          float4 v4 = *reinterpret_cast<const float4*>(red + (x * 4) * RB);
#pragma unroll
          for (int w = 1; w < 4; w++) {
            const float4 u4 = *reinterpret_cast<const float4*>(red + (x * 4 + w) * RB);
            v4 = make_float4(fmaxf(v4.x, u4.x), fmaxf(v4.y, u4.y), fmaxf(v4.z, u4.z), fmaxf(v4.w, u4.w));
          }
          vmx[0] = v4.x;
          vmx[1] = v4.y;
          vmx[2] = v4.z;
          vmx[3] = v4.w;
        }
        // this key's row of the P buffer (64-byte swizzle: chunk c at c ^ ((t >> 1) & 3))
        uint8_t* prow = ps + x * PS_BYTES + t * 64 + wg * 8;
        const int swz = (t >> 1) & 3;
#pragma unroll
        for (int b = 0; b < 4; b++) {
          const float vmax = vmx[b];
          if (b == quarter) {
            if (x) osc1 = vmax * a.q8_smul * (1.f / P_ONE); else osc0 = vmax * a.q8_smul * (1.f / P_ONE);
          }
          const float f = vmax > 0.f ? vsb[b] * rcp_approx(vmax) : 0.f;  // in [0, 1] up to rounding
          // row i's digits are the three low bytes of xi, at bytes 3i .. 3i + 2
          // of this warpgroup's 8 bytes (least significant first)
          uint32_t xi[2] = {0u, 0u};
#pragma unroll
          for (int i = 0; i < RL; i++) {
            const float y = fminf(p[i] * f, 1.f);
            xi[i] = (uint32_t)(__float_as_int(fmaf(y, P_ONE, 12582912.f)) - 0x4B400000);  // round(y (2^22 - 1))
          }
          const uint2 w = make_uint2(__byte_perm(xi[0], xi[1], 0x4210), __byte_perm(xi[1], 0u, 0x4421));
          *reinterpret_cast<uint2*>(prow + ((b ^ swz) << 4)) = w;
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[x]);
      }
    }
    // row sums over the tile keys
#pragma unroll
    for (int i = 0; i < RL; i++) {
      const float v = warp_sum(lsum[i]);
      if (lane == 0) lred[sw * RL + i] = v;
    }
    // One decision for all softmax warps (a bounded wait may give up in some
    // of them only): the merge below synchronises them on named barriers.
    aborted = !named_bar_and(3, 32 * NSW, !aborted);
#pragma unroll
    for (int i = 0; i < RL; i++) lsum[i] = lred[i] + lred[RL + i] + lred[2 * RL + i] + lred[3 * RL + i];
    tc_fence_before();
    __syncthreads();
    if (clus) {
      // This CTA's partial into its own shared memory (the K slots are free),
      // then the merge across the cluster.
      float* cp = reinterpret_cast<float*>(kslots);
#pragma unroll
      for (int i = 0; i < RL; i++) {
        const int r = wg * RL + i;
        cp[r * (Q8_DH + 2) + t] = aborted ? 0.f : acc[i];
        if (t == 0) {
          cp[r * (Q8_DH + 2) + Q8_DH] = aborted ? -1e30f : m[i];
          cp[r * (Q8_DH + 2) + Q8_DH + 1] = aborted ? 0.f : lsum[i];
        }
      }
      cluster_sync_all();
      cluster_merge<R, Q8_DH, 32 * NSW>(a, u, u.nsplit, cp, stid, true);
      cluster_sync_all();
      return;
    }
    if (aborted) {
      // The status word holds the timeout; the unit's tickets stay consistent.
      if (u.nsplit > 1) ticket_merge<R, Q8_DH, 32 * NSW>(a, u, stid, 3, reinterpret_cast<float*>(kslots), s_last);
      return;
    }
    if (u.nsplit == 1) {
#pragma unroll
      for (int i = 0; i < RL; i++) {
        const int r = wg * RL + i;
        if (r < u.rows_valid) store_out(a, out_index(a, u, r, t, Q8_DH), acc[i] / lsum[i]);
      }
      return;
    }
    float* part = a.part + ((size_t)u.unit * a.max_splits + split) * R * (Q8_DH + 2);
#pragma unroll
    for (int i = 0; i < RL; i++) {
      const int r = wg * RL + i;
      part[r * (Q8_DH + 2) + t] = acc[i];
      if (t == 0) {
        part[r * (Q8_DH + 2) + Q8_DH] = m[i];
        part[r * (Q8_DH + 2) + Q8_DH + 1] = lsum[i];
      }
    }
    ticket_merge<R, Q8_DH, 32 * NSW>(a, u, stid, 3, reinterpret_cast<float*>(kslots), s_last);
    return;
  }
  // producers and the MMA warp: wait for the softmax warps, then release TMEM
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (clus) {
    cluster_sync_all();
    cluster_sync_all();
  }
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
    HCU_TRY(check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1),
                       "hcu_attention: q8 tc cluster attribute"));
    return HCU_OK;
  }));
  launch_decode(kern, grid, threads_of(R), SMEM_BYTES, h->stream, args, tk, tv, tks, tvs);
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
