// swa_prefill.cu - causal sliding-window attention prefill on tcgen05 (plamo3).
//
// Semantics of attention_q8 / runAttentionQ8 over a whole prompt
// (src/kernels.ts:1341-1426, src/wasm-backend.ts:826-895 with S = T,
// posBase = 0): query i attends keys j with max(0, i - W + 1) <= j <= i
// (W = windowSize; W = 0 is full causal), scale 1/sqrt(D), grouped head map
// kvh = h / (H / KV).  bf16 Q / K / V (RoPE applied), f32 accumulation,
// bf16 or f32 output.  The reference runs this 8 tokens at a time through the
// decode kernel (PREFILL_CHUNK, src/engine.ts:29).
//
// B200 design (flash-attention on the 5th-gen tensor cores):
//  * CTA = (sequence, KV head, 128-query tile, pair of query heads of that KV
//    head).  Both heads use every K / V tile the TMA brings in.
//  * Per 128-key tile and head: S = Q.K^T (tcgen05.mma, M=N=K=128, Q and K
//    K-major from 128B-swizzled smem, S in TMEM); the softmax warpgroup of the
//    head reads its S rows from TMEM (one thread per query row), writes
//    P = exp2(S*scale - m) as bf16 back into the same TMEM columns, and
//    O += P.V runs with A = P from TMEM and B = V (MN-major) from smem.
//  * The two heads ping-pong: while one head's softmax runs, the tensor core
//    works on the other head's MMAs.
//  * O stays in TMEM across key tiles.  It is rescaled only when a row's
//    running max grows by more than 8 (log2 units): until then P is computed
//    against the stale max, P <= 2^8, which the final O / l cancels exactly.
//  * Only key tiles that intersect the causal window band are visited; tiles
//    entirely inside the band skip per-element masking.
#include <stdlib.h>

#include "common.cuh"
#include "context.h"
#include "tcgen05.cuh"

namespace hcu {
namespace {

// Warpgroup 0: warp 0 TMA, warp 1 MMA + TMEM (warps 2, 3 idle); warpgroup 1 + hd:
// softmax of head hd.  With two heads the 384 threads launch with 168
// registers each (64,512); the control warpgroup drops to 56 and the softmax
// warpgroups rise to 224: 128 * 56 + 256 * 224 = 64,512.
__host__ __device__ constexpr int sw_threads(int nhd) { return 128 + 128 * nhd; }
constexpr uint32_t REG_CTRL = 56, REG_SOFTMAX = 224;
static_assert(128 * REG_CTRL + 256 * REG_SOFTMAX == 384 * 168, "register split of the two-head kernel");
constexpr int BM = 128, BN = 128, HD = 128;
constexpr int BOX = BM * 128;                 // [128 rows x 64 bf16] = 16 KB
constexpr int TILE = 2 * BOX;                 // [128 x 128] bf16 tile
constexpr int KV_STAGES = 2;
constexpr int KV_STAGE = 2 * TILE;            // K tile + V tile
constexpr int OSTAGE = BOX;                   // output staging per head: [128 rows x 64 bf16]
constexpr int NBARS = 18;
constexpr float RESCALE_LOG2 = 8.f;

struct SwaArgs {
  int B, T, H, KV, W, G, nqt;
  int n_items;       // B * KV * (G / NHD) * nqt work items
  float scale_log2;  // log2(e) / sqrt(D)
  void* out;
  int out_bf16;
  uint32_t* status;
};

// lo in the low 16 bits, hi in the high 16 bits (one cvt.rn.bf16x2.f32).
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// 2^x on the SFU (ex2.approx.ftz.f32; 2^-inf = +0).  P is rounded to bf16
// for the P.V product, far coarser than the instruction's error.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// max(a, b, c) in one instruction (three-input max.f32, sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Sets the scores of columns outside this row's valid range lo..hi (tile
// column indices) to -inf, in one 32-column chunk starting at column C0, and
// returns whether no row of the warp keeps any column of it (warp-uniform;
// the chunk is then left as it is and skipped by the max and P).  Chunks
// that every row of the warp keeps whole are left alone too, so only the one
// or two chunks a causal diagonal or window edge cuts through pay a compare
// and select per element.
template <int C0>
__device__ __forceinline__ bool mask_chunk(uint32_t (&r)[32], int lo, int hi) {
  if (__all_sync(0xffffffffu, lo <= C0 && hi >= C0 + 31)) return false;
  if (__all_sync(0xffffffffu, hi < C0 || lo > C0 + 31)) return true;
  const int a = lo - C0, b = hi - C0;
#pragma unroll
  for (int i = 0; i < 32; i++) r[i] = (i >= a && i <= b) ? r[i] : 0xff800000u;  // -inf
  return false;
}

// Row max of one 32-column chunk; `lo`..`hi` is the valid column range (all
// columns when FULL).
template <bool FULL>
__device__ __forceinline__ void chunk_max(const uint32_t (&r)[32], int col0, int lo, int hi, float (&mx)[4]) {
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    float v0 = __uint_as_float(r[i]), v1 = __uint_as_float(r[i + 1]);
    if (!FULL) {
      v0 = (col0 + i >= lo && col0 + i <= hi) ? v0 : -INFINITY;
      v1 = (col0 + i + 1 >= lo && col0 + i + 1 <= hi) ? v1 : -INFINITY;
    }
    mx[(i >> 1) & 3] = fmax3(mx[(i >> 1) & 3], v0, v1);
  }
}

// Packed f32x2 arithmetic (sm_100): one instruction for two lanes of a
// 64-bit register pair, half the issue slots of two scalar instructions.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// P for one 32-column chunk packed as 16 bf16x2 words pk[OFF..OFF+15]; adds
// to the row sum (two packed accumulators).  A chunk that no row of the warp
// keeps (EMPTY, warp-uniform) is all zeros without an exponential.
template <int OFF>
__device__ __forceinline__ void chunk_p(const uint32_t (&r)[32], bool empty, uint64_t scale2, uint64_t negm2,
                                        uint64_t (&ls2)[2], uint32_t (&pk)[32]) {
  if (empty) {
#pragma unroll
    for (int i = 0; i < 16; i++) pk[OFF + i] = 0u;
    return;
  }
#pragma unroll
  for (int i = 0; i < 16; i++) {
    float v0, v1;
    f2_unpack(fma2(f2_pack(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])), scale2, negm2), v0, v1);
    const float p0 = fast_exp2(v0), p1 = fast_exp2(v1);
    ls2[i & 1] = add2(ls2[i & 1], f2_pack(p0, p1));
    pk[OFF + i] = pack_bf16x2(p0, p1);
  }
}

// One work item: a 128-query tile of NHD query heads of one sequence.
struct SwaItem {
  int b, g, h0, m0, n_first, ntiles;
};

// Items are numbered in decreasing cost (query tiles from the last, whose key
// range is longest, to the first); within a query tile, the head pairs that
// share a KV head are adjacent, so CTAs running them together share K / V
// tiles in L2.
template <int NHD>
__device__ __forceinline__ SwaItem swa_item(const SwaArgs& a, int idx) {
  const int hpairs = a.G / NHD;
  const int per_qt = a.B * a.KV * hpairs;
  const int qt = a.nqt - 1 - idx / per_qt;
  int r = idx % per_qt;
  SwaItem it;
  it.b = r / (a.KV * hpairs);
  r %= a.KV * hpairs;
  it.g = r / hpairs;
  it.h0 = it.g * a.G + (r % hpairs) * NHD;
  it.m0 = qt * BM;
  const int kfirst = a.W > 0 ? max(0, it.m0 - a.W + 1) : 0;
  it.n_first = (kfirst / BN) * BN;
  const int n_last = min(it.m0 + BM - 1, a.T - 1);
  it.ntiles = (n_last - it.n_first) / BN + 1;
  return it;
}

// The k-th item of this CTA: rounds of gridDim.x items, walked forwards in
// even rounds and backwards in odd ones (costs decrease with the index, so
// every CTA gets a near-equal share of the key tiles).
__device__ __forceinline__ int swa_item_index(int k) {
  const int P = (int)gridDim.x, c = (int)blockIdx.x;
  return k * P + ((k & 1) ? P - 1 - c : c);
}

// Persistent kernel: one CTA per SM loops over its items.  All barriers run
// continuously across items; their parities come from item and tile counters
// that every role advances identically:
//   q_full / q_empty  once per item and head (Q of the head's next item loads
//                     as soon as its last Q.K^T of the current item has read
//                     the Q tiles),
//   kv_full / kv_empty once per key tile, ring index over all items,
//   s_full / p_half / p_full once per key tile and head,
//   o_free            once per item and head: the epilogue has moved O out of
//                     TMEM, so the next item's first P.V may overwrite it,
//   o_done            once per head, after the CTA's last P.V.
template <int NHD>
__global__ void __launch_bounds__(sw_threads(NHD), 1)
    swa_prefill_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const SwaArgs a) {
  constexpr uint32_t TMEM_COLS = NHD == 2 ? 512 : 256;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qsm = smem;                      // [NHD][TILE]
  uint8_t* kvsm = qsm + NHD * TILE;         // [KV_STAGES][K tile | V tile]
  uint8_t* osm = kvsm + KV_STAGES * KV_STAGE;  // [NHD][OSTAGE]
  uint64_t* bars = reinterpret_cast<uint64_t*>(osm + NHD * OSTAGE);
  uint64_t* q_full = bars;        // [NHD]
  uint64_t* q_empty = bars + 2;   // [NHD]
  uint64_t* kv_full = bars + 4;   // [KV_STAGES]
  uint64_t* kv_empty = bars + 6;  // [KV_STAGES]
  uint64_t* s_full = bars + 8;    // [NHD]
  uint64_t* p_full = bars + 10;   // [NHD]
  uint64_t* o_done = bars + 12;   // [NHD]
  uint64_t* o_free = bars + 14;   // [NHD]
  uint64_t* p_half = bars + 16;   // [NHD]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NBARS);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    for (int i = 0; i < KV_STAGES; i++) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_done[i], 1);
      mbar_init(&o_free[i], 4);
      mbar_init(&p_half[i], 4);
    }
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
  // TMEM columns per head: S (P aliased into its first 64 columns), then O.
  auto s_col = [](int hd) { return (uint32_t)(hd * 256); };
  auto o_col = [](int hd) { return (uint32_t)(hd * 256 + 128); };

  if (warp < 4) {
  if (NHD == 2) warpgroup_reg_dealloc<REG_CTRL>();
  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_tensormap(&tmQ);
      prefetch_tensormap(&tmK);
      prefetch_tensormap(&tmV);
      int kt = 0;  // key tiles loaded, over all items
      bool ok = true;
      for (int k = 0; ok; k++) {
        const int idx = swa_item_index(k);
        if (idx >= a.n_items) break;
        const SwaItem it = swa_item<NHD>(a, idx);
        // Q of head hd loads once the previous item's last Q.K^T of that head
        // has read the buffer.
        auto load_q = [&](int hd) {
          if (k > 0 && !mbar_wait(&q_empty[hd], (k - 1) & 1, a.status)) return false;
          mbar_arrive_expect_tx(&q_full[hd], TILE);
          tma_load_4d(qsm + hd * TILE, &tmQ, &q_full[hd], 0, it.h0 + hd, it.m0, it.b);
          tma_load_4d(qsm + hd * TILE + BOX, &tmQ, &q_full[hd], 64, it.h0 + hd, it.m0, it.b);
          return true;
        };
        // Order of the buffers' release by the MMAs: head 0's Q, the stage of
        // the item's first K / V tile, then head 1's Q.
        if (!load_q(0)) break;
        for (int j = 0; ok && j < it.ntiles; j++, kt++) {
          if (j == 1)
            for (int hd = 1; ok && hd < NHD; hd++) ok = load_q(hd);
          if (!ok) break;
          const int s = kt % KV_STAGES;
          if (kt >= KV_STAGES && !mbar_wait(&kv_empty[s], ((kt - KV_STAGES) / KV_STAGES) & 1, a.status)) {
            ok = false;
            break;
          }
          uint8_t* st = kvsm + s * KV_STAGE;
          const int n0 = it.n_first + j * BN;
          mbar_arrive_expect_tx(&kv_full[s], KV_STAGE);
          tma_load_4d(st, &tmK, &kv_full[s], 0, it.g, n0, it.b);
          tma_load_4d(st + BOX, &tmK, &kv_full[s], 64, it.g, n0, it.b);
          tma_load_4d(st + TILE, &tmV, &kv_full[s], 0, it.g, n0, it.b);
          tma_load_4d(st + TILE + BOX, &tmV, &kv_full[s], 64, it.g, n0, it.b);
        }
        if (ok && it.ntiles == 1)
          for (int hd = 1; ok && hd < NHD; hd++) ok = load_q(hd);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    // The whole warp walks the loop (every value in it is warp-uniform); one
    // elected lane issues each tcgen05 instruction.
    {
      const bool leader = elect_one_sync();
      constexpr uint32_t idesc_qk = idesc_f16(BM, BN, true, false, false);
      constexpr uint32_t idesc_pv = idesc_f16(BM, HD, true, false, true);
      const uint32_t q0 = smem_u32(qsm), kv0 = smem_u32(kvsm);
      auto qk = [&](int hd, int s) {
#pragma unroll
        for (int ks = 0; ks < 8; ks++) {
          const uint64_t ad = smem_desc_sw128(q0 + hd * TILE + (ks >> 2) * BOX + (ks & 3) * 32, 16, 1024);
          const uint64_t bd = smem_desc_sw128(kv0 + s * KV_STAGE + (ks >> 2) * BOX + (ks & 3) * 32, 16, 1024);
          if (leader) mma_f16_ss(tmem + s_col(hd), ad, bd, idesc_qk, ks > 0);
        }
        if (leader) mma_commit(&s_full[hd]);
      };
      // P.V in two halves of 64 keys (k-steps 0-3, 4-7): the first runs
      // while the softmax still computes the second half of P.
      auto pv_half = [&](int hd, int s, int half, bool acc) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const int ks = 4 * half + i;
          const uint64_t bd = smem_desc_sw128(kv0 + s * KV_STAGE + TILE + ks * 2048, BOX, 1024);  // MN-major V
          if (leader) mma_f16_ts(tmem + o_col(hd), tmem + s_col(hd) + ks * 8, bd, idesc_pv, (acc || ks > 0) ? 1u : 0u);
        }
      };
      // The tiles of consecutive items form one stream: a head's next Q.K^T
      // (the item's next tile, or the next item's first) issues right behind
      // its P.V of the current tile, which has consumed the P it overwrites.
      int kt = 0;  // key tiles consumed (ring position and per-head tile count)
      bool ok = true;
      int idx = swa_item_index(0);
      int ntiles = idx < a.n_items ? swa_item<NHD>(a, idx).ntiles : 0;
      if (ntiles > 0) {
        for (int hd = 0; hd < NHD; hd++) {
          if (!__all_sync(0xffffffffu, mbar_wait(&q_full[hd], 0, a.status) &&
                                           (hd > 0 || mbar_wait(&kv_full[0], 0, a.status)))) {
            ok = false;
            break;
          }
          tc_fence_after();
          qk(hd, 0);
          if (ntiles == 1 && leader) mma_commit(&q_empty[hd]);  // the item's last Q.K^T of this head
        }
      }
      for (int k = 0; ok && ntiles > 0; k++) {
        idx = swa_item_index(k + 1);
        const int ntiles1 = idx < a.n_items ? swa_item<NHD>(a, idx).ntiles : 0;
        for (int j = 0; ok && j < ntiles; j++) {
          const int t = kt + j;
          const int s = t % KV_STAGES;
          const bool last = j + 1 == ntiles;
          for (int hd = 0; hd < NHD; hd++) {
            if (!__all_sync(0xffffffffu, mbar_wait(&p_half[hd], t & 1, a.status) &&
                                             (j > 0 || k == 0 || mbar_wait(&o_free[hd], (k - 1) & 1, a.status)))) {
              ok = false;
              break;
            }
            tc_fence_after();
            pv_half(hd, s, 0, j > 0);
            if (!__all_sync(0xffffffffu, mbar_wait(&p_full[hd], t & 1, a.status))) {
              ok = false;
              break;
            }
            tc_fence_after();
            pv_half(hd, s, 1, true);
            if (leader) {
              // o_done only after the CTA's last P.V of the head: any other
              // P.V is followed by a Q.K^T of the same head, whose s_full
              // arrive (a commit tracks every earlier MMA of this thread)
              // already tells the softmax that O is complete.
              if (last && ntiles1 == 0) mma_commit(&o_done[hd]);
              if (hd == NHD - 1) mma_commit(&kv_empty[s]);
            }
            if (!last || ntiles1 > 0) {
              const int s1 = (t + 1) % KV_STAGES;
              if (!__all_sync(0xffffffffu, (hd > 0 || mbar_wait(&kv_full[s1], ((t + 1) / KV_STAGES) & 1, a.status)) &&
                                               (!last || mbar_wait(&q_full[hd], (k + 1) & 1, a.status)))) {
                ok = false;
                break;
              }
              tc_fence_after();
              qk(hd, s1);  // overwrites S / P of this head: ordered after the P.V above
              if ((last ? ntiles1 == 1 : j + 2 == ntiles) && leader) mma_commit(&q_empty[hd]);
            }
          }
        }
        kt += ntiles;
        ntiles = ntiles1;
      }
    }
  }
  } else {
    // ---------------- softmax of head hd, one thread per query row ----------------
    if (NHD == 2) warpgroup_reg_alloc<REG_SOFTMAX>();
    const int hd = (warp - 4) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t sc = tmem + lane_off + s_col(hd), oc = tmem + lane_off + o_col(hd);
    // Epilogue of one item: O / l out of TMEM and into the output.  It runs
    // after the NEXT item's first P is in TMEM (O of the finished item has
    // long been complete by then), so the MMA round trip of that first tile
    // covers it; o_free then lets the next item's first P.V overwrite O.
    // bf16 output goes 64 columns at a time: each warp turns its 32 rows
    // around in its own 4 KB of the head's staging buffer (thread = row on
    // the way in, 8 threads per 128-byte row segment on the way out), so
    // every global store instruction writes four whole 128-byte segments.
    // fin_idx: the finished item, fin_l: this row's sum of P.  O is complete
    // once the next item's first S is in (its Q.K^T follows the last P.V);
    // after the CTA's last item, o_done says so.
    auto epilogue = [&](int fin_idx, float fin_l, bool last_item) -> bool {
      if (last_item && !__all_sync(0xffffffffu, mbar_wait(&o_done[hd], 0, a.status))) return false;
      tc_fence_after();
      uint32_t o[4][32];
#pragma unroll
      for (int c = 0; c < 4; c++) tmem_ld32(oc + 32 * c, o[c]);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_free[hd]);
      const SwaItem f = swa_item<NHD>(a, fin_idx);  // after o_free: the next P.V waits for it
      const float inv = 1.f / fin_l;
      if (a.out_bf16) {
        uint8_t* wst = osm + hd * OSTAGE + quarter * 4096;  // this warp's rows
        // Read-out: lane -> row 4i + (lane >> 3) of the warp, 16-byte piece lane & 7.
        const int rr = lane >> 3, seg = lane & 7;
        const size_t rstride = (size_t)a.H * HD;  // elements between consecutive tokens
        __nv_bfloat16* gp = static_cast<__nv_bfloat16*>(a.out) +
                            (((size_t)f.b * a.T + f.m0 + quarter * 32 + rr) * a.H + f.h0 + hd) * HD + 8 * seg;
        const int rows_left = a.T - (f.m0 + quarter * 32 + rr);  // rows 4i with 4i < rows_left exist
#pragma unroll
        for (int half = 0; half < 2; half++) {
#pragma unroll
          for (int c = 0; c < 8; c++) {
            const uint32_t* v = &o[2 * half + (c >> 2)][8 * (c & 3)];
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(v[0]) * inv, __uint_as_float(v[1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(v[2]) * inv, __uint_as_float(v[3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(v[4]) * inv, __uint_as_float(v[5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(v[6]) * inv, __uint_as_float(v[7]) * inv);
            *reinterpret_cast<uint4*>(wst + lane * 128 + ((c ^ (lane & 7)) << 4)) = w;
          }
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 8; i++) {
            const int r = 4 * i + rr;
            const uint4 w = *reinterpret_cast<const uint4*>(wst + r * 128 + ((seg ^ (r & 7)) << 4));
            if (4 * i < rows_left) *reinterpret_cast<uint4*>(gp + 4 * i * rstride + 64 * half) = w;
          }
          __syncwarp();
        }
      } else if (f.m0 + row < a.T) {
        float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.out) +
                                                (((size_t)f.b * a.T + f.m0 + row) * a.H + f.h0 + hd) * HD);
#pragma unroll
        for (int c = 0; c < 4; c++)
#pragma unroll
          for (int i = 0; i < 8; i++)
            dst[8 * c + i] = make_float4(__uint_as_float(o[c][4 * i]) * inv, __uint_as_float(o[c][4 * i + 1]) * inv,
                                         __uint_as_float(o[c][4 * i + 2]) * inv,
                                         __uint_as_float(o[c][4 * i + 3]) * inv);
      }
      return true;
    };
    int fin_idx = -1;
    float fin_l = 0.f;
    int kt = 0;  // key tiles processed, over all items
    bool ok = true;
    for (int k = 0; ok; k++) {
      const int idx = swa_item_index(k);
      if (idx >= a.n_items) break;
      const SwaItem it = swa_item<NHD>(a, idx);
      const int m0 = it.m0, query = m0 + row;
      float m_use = -INFINITY, l = 0.f;
      for (int j = 0; j < it.ntiles; j++) {
        const int t = kt + j;
        const int n0 = it.n_first + j * BN;
        if (!__all_sync(0xffffffffu, mbar_wait(&s_full[hd], t & 1, a.status))) {  // warp-uniform exit
          ok = false;
          break;
        }
        tc_fence_after();
        // The whole S row (128 columns) is loaded once, with one wait, and kept
        // in registers for both the row max and P.
        const bool full = (n0 + BN - 1 <= m0) && (a.W == 0 || n0 >= m0 + BM - a.W) && (n0 + BN <= a.T);
        const int lo = (a.W > 0 ? query - a.W + 1 : 0) - n0;  // valid column range of this row
        const int hi = min(query, a.T - 1) - n0;
        uint32_t s0[32], s1[32], s2[32], s3[32];
        tmem_ld32(sc, s0);
        tmem_ld32(sc + 32, s1);
        tmem_ld32(sc + 64, s2);
        tmem_ld32(sc + 96, s3);
        tmem_ld_wait();
        bool e0 = false, e1 = false, e2 = false, e3 = false;  // chunks no row of the warp keeps
        if (!full) {  // tile cut by the causal diagonal, the window edge or T
          e0 = mask_chunk<0>(s0, lo, hi);
          e1 = mask_chunk<32>(s1, lo, hi);
          e2 = mask_chunk<64>(s2, lo, hi);
          e3 = mask_chunk<96>(s3, lo, hi);
        }
        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        if (!e0) chunk_max<true>(s0, 0, lo, hi, mx4);
        if (!e1) chunk_max<true>(s1, 32, lo, hi, mx4);
        if (!e2) chunk_max<true>(s2, 64, lo, hi, mx4);
        if (!e3) chunk_max<true>(s3, 96, lo, hi, mx4);
        const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * a.scale_log2;
        // The running max grew by more than 2^8 (or this is the first finite
        // max): move to the new max.  Rows that already accumulated O rescale
        // it; tcgen05.ld / st are warp-collective, so the whole warp takes the
        // TMEM round trip when any of its rows needs it (factor 1 elsewhere).
        const bool move = mx > m_use + RESCALE_LOG2 || (j == 0 && mx > m_use);
        const bool rescale_o = move && j > 0 && m_use != -INFINITY;
        const float f = rescale_o ? exp2f(m_use - mx) : 1.f;
        if (__any_sync(0xffffffffu, rescale_o)) {  // P.V of tile j-1 has landed (s_full of tile j)
#pragma unroll
          for (int c = 0; c < 4; c++) {
            uint32_t r[32];
            tmem_ld32(oc + 32 * c, r);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; i++) r[i] = __float_as_uint(__uint_as_float(r[i]) * f);
            tmem_st32(oc + 32 * c, r);
          }
          tmem_st_wait();
        }
        if (move) {
          l *= f;
          m_use = mx;
        }
        // P = exp2(S*scale - m) as bf16, written over the S columns already
        // read (keys 64c..64c+63 land in columns 32c..32c+31).
        const float neg_m = m_use == -INFINITY ? 0.f : -m_use;
        const uint64_t scale2 = f2_pack(a.scale_log2, a.scale_log2), negm2 = f2_pack(neg_m, neg_m);
        uint64_t ls2[2] = {f2_pack(0.f, 0.f), f2_pack(0.f, 0.f)};
        {
          uint32_t pk[32];
          chunk_p<0>(s0, e0, scale2, negm2, ls2, pk);
          chunk_p<16>(s1, e1, scale2, negm2, ls2, pk);
          tmem_st32(sc, pk);
        }
        // Keys 0..63 of P are in TMEM: the first half of P.V may start.
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_half[hd]);
        {
          uint32_t pk[32];
          chunk_p<0>(s2, e2, scale2, negm2, ls2, pk);
          chunk_p<16>(s3, e3, scale2, negm2, ls2, pk);
          tmem_st32(sc + 32, pk);
        }
        {
          float a0, a1, b0, b1;
          f2_unpack(ls2[0], a0, a1);
          f2_unpack(ls2[1], b0, b1);
          l += (a0 + a1) + (b0 + b1);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[hd]);
        if (j == 0 && fin_idx >= 0) {
          if (!epilogue(fin_idx, fin_l, false)) {
            ok = false;
            break;
          }
          fin_idx = -1;
        }
      }
      if (!ok) break;  // warp-uniform
      fin_idx = idx;
      fin_l = l;
      kt += it.ntiles;
    }
    if (ok && fin_idx >= 0) epilogue(fin_idx, fin_l, true);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

template <int NHD>
int launch_swa(hcu_context* h, const SwaArgs& args, const CUtensorMap& tq, const CUtensorMap& tk,
               const CUtensorMap& tv) {
  constexpr size_t smem = 1024 + NHD * TILE + KV_STAGES * KV_STAGE + NHD * OSTAGE + NBARS * 8 + 16;
  static_assert(smem <= 227 * 1024, "shared memory of the SWA kernel");
  auto kern = swa_prefill_kernel<NHD>;
  static std::atomic<uint64_t> attr_done{0};  // per device
  HCU_TRY(once_per_device(attr_done, h->device, [&]() -> int {
    HCU_TRY(check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                       "hcu_swa_prefill: smem attribute"));
    return HCU_OK;
  }));
  // One CTA per SM (the shared memory admits no second), never more CTAs than
  // items.  HCU_OPT_SWA_CTAS caps the grid (tests use it to give every CTA a long
  // chain of items on small shapes).
  int grid = args.n_items < h->sm_count ? args.n_items : h->sm_count;
  if (h->opt_swa_ctas > 0 && h->opt_swa_ctas < grid) grid = (int)h->opt_swa_ctas;
  kern<<<grid, sw_threads(NHD), smem, h->stream>>>(tq, tk, tv, args);
  return after_launch("hcu_swa_prefill: launch");
}

}  // namespace
}  // namespace hcu

using hcu::fail;

extern "C" int hcu_swa_prefill(hcu_handle h, const hcu_swa_params* p, const void* q, const void* k, const void* v,
                               void* out) {
  HCU_TRY(hcu::begin_op(h, "hcu_swa_prefill"));
  if (!p || !q || !k || !v || !out) return fail(HCU_EINVAL, "hcu_swa_prefill: null argument");
  const int B = (int)p->B, T = (int)p->T, H = (int)p->H, KV = (int)p->KV, D = (int)p->D;
  if (B < 1 || T < 1 || H < 1 || KV < 1) return fail(HCU_EINVAL, "hcu_swa_prefill: B, T, H, KV must be positive");
  if (D != 128) return fail(HCU_EUNSUPPORTED, "hcu_swa_prefill: D=%d (built: 128)", D);
  if (H % KV) return fail(HCU_EINVAL, "hcu_swa_prefill: H (%d) is not a multiple of KV (%d)", H, KV);
  if (p->out_dtype != HCU_DT_BF16 && p->out_dtype != HCU_DT_F32)
    return fail(HCU_EINVAL, "hcu_swa_prefill: out_dtype must be HCU_DT_BF16 or HCU_DT_F32");
  if (B > 65535) return fail(HCU_EINVAL, "hcu_swa_prefill: B > 65535");
  if (reinterpret_cast<uintptr_t>(out) % 16) return fail(HCU_EINVAL, "hcu_swa_prefill: out must be 16-byte aligned");
  const int G = H / KV;
  const int nhd = (G % 2 == 0) ? 2 : 1;
  const int nqt = (T + hcu::BM - 1) / hcu::BM;
  CUtensorMap tq, tk, tv;
  {
    uint64_t dims[4] = {128, (uint64_t)H, (uint64_t)T, (uint64_t)B};
    uint64_t strides[3] = {256, (uint64_t)H * 256, (uint64_t)T * H * 256};
    uint32_t box[4] = {64, 1, 128, 1};
    HCU_TRY(hcu::make_tensor_map(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(q), dims, strides, box,
                                 CU_TENSOR_MAP_SWIZZLE_128B));
  }
  {
    uint64_t dims[4] = {128, (uint64_t)KV, (uint64_t)T, (uint64_t)B};
    uint64_t strides[3] = {256, (uint64_t)KV * 256, (uint64_t)T * KV * 256};
    uint32_t box[4] = {64, 1, 128, 1};
    HCU_TRY(hcu::make_tensor_map(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(k), dims, strides, box,
                                 CU_TENSOR_MAP_SWIZZLE_128B));
    HCU_TRY(hcu::make_tensor_map(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(v), dims, strides, box,
                                 CU_TENSOR_MAP_SWIZZLE_128B));
  }
  hcu::SwaArgs args{};
  args.B = B;
  args.T = T;
  args.H = H;
  args.KV = KV;
  args.W = (int)p->window;
  args.G = G;
  args.nqt = nqt;
  args.scale_log2 = hcu::kLog2e / sqrtf((float)D);
  args.out = out;
  args.out_bf16 = p->out_dtype == HCU_DT_BF16;
  args.status = h->dev_status;
  const long long n_items = (long long)B * KV * (G / nhd) * nqt;
  if (n_items > (1LL << 30)) return fail(HCU_EINVAL, "hcu_swa_prefill: B x H x T/128 too large");
  args.n_items = (int)n_items;
  if (nhd == 2) return hcu::launch_swa<2>(h, args, tq, tk, tv);
  return hcu::launch_swa<1>(h, args, tq, tk, tv);
}
