// attention_decode_tc.cu - tcgen05 (5th-gen tensor core) split-K decode
// attention for f16 / bf16 KV caches with head_dim 128.
//
// Same semantics and split-K / ticket-merge structure as the CUDA-core kernel
// (attention_decode.cu): replaces attention_q8 (src/kernels.ts:1341-1426) /
// runAttentionQ8 (src/wasm-backend.ts:826-895) for the f16 / bf16 cache formats.
//
// Per CTA: one (sequence, KV head, query block, key split).  Per 128-token tile:
//   S^T[128 tok x N] = K_tile[128 x 128] . Qcat^T   (tcgen05.mma, M=128, K=d)
//   O^T[128 d x N]   = V_tile^T . P^T               (tcgen05.mma, M=128, K=tokens)
// K_tile is the TMA-loaded, 128B-swizzled tile used directly as the K-major A
// operand; V_tile is the same tile read as an MN-major A operand, so nothing is
// transposed or copied.  The N columns are the CTA's R query rows (GQA group x
// queries), each split into 16-bit terms: q*2^8 = hi + lo (f16, ~22 bits) or
// hi + mid + lo (bf16, ~24 bits), and likewise p*2^8, so the tensor-core result
// keeps f32 accuracy (the fp32 tolerance of the decode path).  Accumulators
// live in TMEM: two S buffers and two O buffers, so the QK^T MMA of tile j+1
// and the P.V MMA of tile j-1 overlap the softmax of tile j.
//
// Warp roles (192 threads): warp 0 issues TMA (K tiles into a 2-slot ring,
// V tiles into a 1-slot ring, 32 KB per slot),
// warp 1 allocates TMEM and issues MMAs (one thread), warps 2-5 (128 threads,
// one TMEM lane each) run the online softmax and accumulate each tile's O^T
// into registers (thread = head-dim index), rescaled by the running max.
#include "attention.cuh"
#include "tcgen05.cuh"

namespace hcu {
namespace {

constexpr int TC_THREADS = 192;
constexpr int TC_TT = kTcTile;              // 128 tokens per tile
constexpr int TC_DH = 128;
constexpr int BOX_BYTES = TC_TT * 128;      // [128 tokens x 64 elements x 2 B]
constexpr int HALF_BYTES = 2 * BOX_BYTES;   // one K or V tile: lo and hi 64-element boxes
// K runs a tile ahead of V: a K slot frees as soon as Q.K^T has read it, the
// V slot only after P.V.  3 x 32 KB of ring (plus Q / P staging) lets two CTAs
// share an SM for NC = 16, so one CTA's start-up and split merge overlap the
// other's streaming.
constexpr int TC_KST = 2, TC_VST = 1;
constexpr int RING_BYTES = (TC_KST + TC_VST) * HALF_BYTES;
constexpr float PSCALE = 256.f;             // q and p are scaled by 2^8 before splitting

// x ~= sum of NT 16-bit terms, largest first.
template <bool BF16, int NT>
__device__ __forceinline__ void split_terms(float x, uint16_t (&t)[NT]) {
  float r = x;
#pragma unroll
  for (int i = 0; i < NT; i++) {
    if constexpr (BF16) {
      const __nv_bfloat16 h = __float2bfloat16_rn(r);
      t[i] = __bfloat16_as_ushort(h);
      r -= __bfloat162float(h);
    } else {
      const __half h = __float2half_rn(r);
      t[i] = __half_as_ushort(h);
      r -= __half2float(h);
    }
  }
}

// NC consecutive TMEM columns of this thread's lane, starting at `taddr`.
template <int NC>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&v)[NC]) {
  uint32_t c0[16];
  tmem_ld16(taddr, c0);
  if constexpr (NC == 32) {
    uint32_t c1[16];
    tmem_ld16(taddr + 16, c1);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 16; i++) v[16 + i] = c1[i];
  } else {
    tmem_ld_wait();
  }
#pragma unroll
  for (int i = 0; i < 16; i++) v[i] = c0[i];
}

__device__ __forceinline__ void st_u16(uint8_t* base, uint32_t off, uint16_t v) {
  *reinterpret_cast<uint16_t*>(base + off) = v;
}

template <bool BF16, int R, int NC>
__global__ void __launch_bounds__(TC_THREADS, NC == 16 ? 2 : 1)
    attn_decode_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                          const AttnArgs a) {
  constexpr int NT = BF16 ? 3 : 2;
  static_assert(NT * R <= NC && NC % 16 == 0 && NC <= 32, "bad column count");
  constexpr int QS_BLK = NC * 128;  // one 64-element K block of Qcat / P: NC rows x 128 B
  constexpr uint32_t TMEM_COLS = 4 * NC;
  constexpr uint32_t S_COL = 0, O_COL = 2 * NC;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;                       // K slots, then the V slot
  uint8_t* vslot = stages + TC_KST * HALF_BYTES;
  uint8_t* qs = stages + RING_BYTES;            // [2 blocks][NC rows x 128 B]
  uint8_t* ps = qs + 2 * QS_BLK;                // [2 buffers][2 blocks][NC rows x 128 B]
  uint64_t* bars = reinterpret_cast<uint64_t*>(ps + 4 * QS_BLK);
  uint64_t* k_full = bars;                      // [TC_KST]
  uint64_t* k_empty = bars + 2;                 // [TC_KST]
  uint64_t* v_full = bars + 4;
  uint64_t* v_empty = bars + 5;
  uint64_t* s_full = bars + 6;
  uint64_t* s_free = bars + 8;
  uint64_t* p_full = bars + 10;
  uint64_t* o_full = bars + 12;
  uint64_t* o_free = bars + 14;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  int* s_last = reinterpret_cast<int*>(tmem_slot + 1);
  float* red = reinterpret_cast<float*>(tmem_slot + 4);  // [2][4][R] tile maxima
  float* lred = red + 2 * 4 * R;                          // [4][R] row sums

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.x;
  const AttnUnit u = attn_unit(a, split);
  // In the cluster form every CTA of the unit's cluster reaches the two
  // cluster barriers; a CTA without work only contributes an empty partial.
  const bool clus = a.cluster != 0;
  const bool badarg = u.nsplit > (int)gridDim.x;
  if (badarg && split == 0 && tid == 0) atomicOr(a.status, HCU_DEVERR_BADARG);
  if (badarg || split >= u.nsplit) {
    if (!clus) return;
    float* cp = reinterpret_cast<float*>(stages);  // [R][Dh + 2]: acc, m, l
    for (int e = tid; e < R * (TC_DH + 2); e += TC_THREADS) cp[e] = e % (TC_DH + 2) == TC_DH ? -1e30f : 0.f;
    cluster_sync_all();
    if (warp >= 2)
      cluster_merge<R, TC_DH, 128>(a, u, badarg ? 0 : min(u.nsplit, (int)gridDim.x), cp, (warp & 3) * 32 + lane,
                                   !badarg);
    cluster_sync_all();
    return;
  }
  const int ntiles = (u.k_hi - u.k_lo + TC_TT - 1) / TC_TT;

  if (tid == 0) {
    for (int i = 0; i < TC_KST; i++) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    mbar_init(v_full, 1);
    mbar_init(v_empty, 1);
    for (int i = 0; i < 2; i++) {
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
  // Softmax threads: t = TMEM lane (token of a tile for S, head-dim for O).
  const int quarter = warp & 3;
  const int t = quarter * 32 + lane;
  int jlo[R], jhi[R];
  if (warp >= 2) {
    // Stage Qcat (rows term*R + r, columns d) scaled by log2(e)/sqrt(Dh) * 2^8.
#pragma unroll
    for (int r = 0; r < R; r++) {
      const int qi = u.q0 + r / a.G;
      const bool valid = (r < a.QB * a.G) && (r / a.G < u.qn);
      const int pos = u.pb + qi;
      jlo[r] = valid ? ((a.window > 0 && pos + 1 > a.window) ? pos + 1 - a.window : 0) : 1;
      jhi[r] = valid ? pos : 0;
      float x = 0.f;
      if (valid) x = __ldg(a.q + out_index(a, u, r, t, TC_DH)) * a.qscale * PSCALE;
      uint16_t tm[NT];
      split_terms<BF16, NT>(x, tm);
#pragma unroll
      for (int k = 0; k < NT; k++) st_u16(qs + (t >> 6) * QS_BLK, sw128_offset(k * R + r, (t & 63) * 2), tm[k]);
    }
    for (int n = NT * R; n < NC; n++) st_u16(qs + (t >> 6) * QS_BLK, sw128_offset(n, (t & 63) * 2), 0);
    for (int i = t; i < 4 * QS_BLK / 16; i += 128) reinterpret_cast<uint4*>(ps)[i] = make_uint4(0, 0, 0, 0);
    fence_proxy_async();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool aborted = false;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_tensormap(&tmK);
      prefetch_tensormap(&tmV);
      auto load_k = [&](int it) {  // K of tile it, after Q.K^T(it - TC_KST) read its slot
        const int s = it % TC_KST, rnd = it / TC_KST;
        if (rnd > 0 && !mbar_wait(&k_empty[s], (rnd - 1) & 1, a.status)) return false;
        uint8_t* st = stages + s * HALF_BYTES;
        const int row = (int)(u.roff + u.k_lo + it * TC_TT);
        mbar_arrive_expect_tx(&k_full[s], HALF_BYTES);
        tma_load_3d(st, &tmK, &k_full[s], 0, u.g, row);
        tma_load_3d(st + BOX_BYTES, &tmK, &k_full[s], 64, u.g, row);
        return true;
      };
      if (ntiles > 0 && load_k(0)) {
        for (int it = 0; it < ntiles; ++it) {
          if (it + 1 < ntiles && !load_k(it + 1)) break;
          // V of tile it, after P.V(it - 1) read the slot
          if (it > 0 && !mbar_wait(v_empty, (it - 1) & 1, a.status)) break;
          const int row = (int)(u.roff + u.k_lo + it * TC_TT);
          mbar_arrive_expect_tx(v_full, HALF_BYTES);
          tma_load_3d(vslot, &tmV, v_full, 0, u.g, row);
          tma_load_3d(vslot + BOX_BYTES, &tmV, v_full, 64, u.g, row);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    // The whole warp walks the loop (its values are warp-uniform); one
    // elected lane issues each tcgen05 instruction.
    {
      const bool leader = elect_one_sync();
      constexpr uint32_t idesc_qk = idesc_f16(128, NC, BF16, false, false);
      constexpr uint32_t idesc_pv = idesc_f16(128, NC, BF16, true, false);
      const uint32_t st0 = smem_u32(stages), qs0 = smem_u32(qs), ps0 = smem_u32(ps);
      for (int j = 0; j <= ntiles; ++j) {
        if (j < ntiles) {
          const int s = j % TC_KST, x = j & 1;
          if (!__all_sync(0xffffffffu, mbar_wait(&k_full[s], (j / TC_KST) & 1, a.status))) break;
          if (j >= 2 && !__all_sync(0xffffffffu, mbar_wait(&s_free[x], ((j - 2) >> 1) & 1, a.status))) break;
          tc_fence_after();
          const uint32_t kb = st0 + s * HALF_BYTES;
#pragma unroll
          for (int ks = 0; ks < 8; ks++) {
            const uint64_t ad = smem_desc_sw128(kb + (ks >> 2) * BOX_BYTES + (ks & 3) * 32, 16, 1024);
            const uint64_t bd = smem_desc_sw128(qs0 + (ks >> 2) * QS_BLK + (ks & 3) * 32, 16, 1024);
            if (leader) mma_f16_ss(tmem + S_COL + x * NC, ad, bd, idesc_qk, ks > 0);
          }
          if (leader) mma_commit(&s_full[x]);
          if (leader) mma_commit(&k_empty[s]);
        }
        if (j >= 1) {
          const int jp = j - 1, xp = jp & 1;
          // V(jp) landed (the softmax also waits for it before zeroing rows of a partial tile)
          if (!__all_sync(0xffffffffu, mbar_wait(v_full, jp & 1, a.status))) break;
          if (!__all_sync(0xffffffffu, mbar_wait(&p_full[xp], (jp >> 1) & 1, a.status))) break;
          if (jp >= 2 && !__all_sync(0xffffffffu, mbar_wait(&o_free[xp], ((jp - 2) >> 1) & 1, a.status))) break;
          tc_fence_after();
          const uint32_t vb = st0 + TC_KST * HALF_BYTES;
          const uint32_t pb = ps0 + xp * 2 * QS_BLK;
#pragma unroll
          for (int ks = 0; ks < 8; ks++) {
            const uint64_t ad = smem_desc_sw128(vb + ks * 2048, BOX_BYTES, 1024);  // MN-major V^T
            const uint64_t bd = smem_desc_sw128(pb + (ks >> 2) * QS_BLK + (ks & 3) * 32, 16, 1024);
            if (leader) mma_f16_ss(tmem + O_COL + xp * NC, ad, bd, idesc_pv, ks > 0);
          }
          if (leader) mma_commit(&o_full[xp]);
          if (leader) mma_commit(v_empty);
        }
      }
    }
  } else {
    // ---------------- softmax / accumulation (128 threads) ----------------
    const int sw = warp - 2;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    float m[R], lsum[R], acc[R], corr0[R], corr1[R];  // corr0/1: rescale of tiles with even / odd index
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
        if (!__all_sync(0xffffffffu, mbar_wait(&o_full[xo], (jo >> 1) & 1, a.status))) {  // warp-uniform exit
          aborted = true;
          break;
        }
        tc_fence_after();
        uint32_t o[NC];
        tmem_ld_cols<NC>(tmem + lane_off + O_COL + xo * NC, o);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&o_free[xo]);
#pragma unroll
        for (int r = 0; r < R; r++) {
          float v = 0.f;
#pragma unroll
          for (int k = NT - 1; k >= 0; k--) v += __uint_as_float(o[k * R + r]);
          acc[r] = fmaf(acc[r], xo ? corr1[r] : corr0[r], v);
        }
      }
      if (j < ntiles) {
        const int x = j & 1;
        if (!__all_sync(0xffffffffu, mbar_wait(&s_full[x], (j >> 1) & 1, a.status))) {
          aborted = true;
          break;
        }
        tc_fence_after();
        uint32_t sv[NC];
        tmem_ld_cols<NC>(tmem + lane_off + S_COL + x * NC, sv);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[x]);

        const int key = u.k_lo + j * TC_TT + t;
        float sc[R];
#pragma unroll
        for (int r = 0; r < R; r++) {
          float v = 0.f;
#pragma unroll
          for (int k = NT - 1; k >= 0; k--) v += __uint_as_float(sv[k * R + r]);
          const bool ok = key >= jlo[r] && key <= jhi[r] && key < u.k_hi;
          sc[r] = ok ? v * (1.f / PSCALE) : -INFINITY;
          const float mx = warp_max(sc[r]);
          if (lane == 0) red[(x * 4 + sw) * R + r] = mx;
        }
        named_bar(1, 128);
        uint8_t* pbuf = ps + x * 2 * QS_BLK + (t >> 6) * QS_BLK;
#pragma unroll
        for (int r = 0; r < R; r++) {
          float mt = red[(x * 4) * R + r];
#pragma unroll
          for (int w = 1; w < 4; w++) mt = fmaxf(mt, red[(x * 4 + w) * R + r]);
          const float mnew = fmaxf(m[r], mt);
          const float corr = exp2f(m[r] - mnew);
          if (x) corr1[r] = corr; else corr0[r] = corr;
          m[r] = mnew;
          const float p = exp2f(sc[r] - mnew);
          lsum[r] = fmaf(lsum[r], corr, p);
          uint16_t tm[NT];
          split_terms<BF16, NT>(p * PSCALE, tm);
#pragma unroll
          for (int k = 0; k < NT; k++) st_u16(pbuf, sw128_offset(k * R + r, (t & 63) * 2), tm[k]);
        }
        if (u.k_lo + j * TC_TT + TC_TT > u.k_hi) {  // partial tile (uniform for the CTA)
          // V(j) must have landed before its rows are overwritten.  P.V(j - 1)
          // completing first (its own O buffer, one phase in flight) means the
          // one V slot holds no earlier tile, so the wait for V(j) is exact.
          const int jm = j - 1;
          const bool okw = (jm < 0 || mbar_wait(&o_full[jm & 1], (jm >> 1) & 1, a.status)) &&
                           mbar_wait(v_full, j & 1, a.status);
          if (!__all_sync(0xffffffffu, okw)) {
            aborted = true;
            break;
          }
        }
        if (key >= u.k_hi) {
          // Rows past this split's keys may hold anything (another sequence,
          // unwritten cache): zero this token's V row so 0 * V stays 0.
          uint8_t* vrow = vslot + t * 128;
#pragma unroll
          for (int c = 0; c < 8; c++) {
            reinterpret_cast<uint4*>(vrow)[c] = make_uint4(0, 0, 0, 0);
            reinterpret_cast<uint4*>(vrow + BOX_BYTES)[c] = make_uint4(0, 0, 0, 0);
          }
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[x]);
      }
    }
    // row sums over the tile tokens
#pragma unroll
    for (int r = 0; r < R; r++) {
      const float v = warp_sum(lsum[r]);
      if (lane == 0) lred[sw * R + r] = v;
    }
    // One decision for the four softmax warps (a bounded wait may give up in
    // some of them only): the merge below synchronises them on named barriers.
    aborted = !named_bar_and(1, 128, !aborted);
#pragma unroll
    for (int r = 0; r < R; r++) {
      lsum[r] = lred[r] + lred[R + r] + lred[2 * R + r] + lred[3 * R + r];
      acc[r] *= (1.f / PSCALE);
    }
    // Hold the results until TMEM is released below.
    tc_fence_before();
    __syncthreads();
    if (clus) {
      // This CTA's partial into its own shared memory (the stages are free),
      // then the merge across the cluster.
      float* cp = reinterpret_cast<float*>(stages);
#pragma unroll
      for (int r = 0; r < R; r++) {
        cp[r * (TC_DH + 2) + t] = aborted ? 0.f : acc[r];
        if (t == 0) {
          cp[r * (TC_DH + 2) + TC_DH] = aborted ? -1e30f : m[r];
          cp[r * (TC_DH + 2) + TC_DH + 1] = aborted ? 0.f : lsum[r];
        }
      }
      cluster_sync_all();
      cluster_merge<R, TC_DH, 128>(a, u, u.nsplit, cp, t, true);
      cluster_sync_all();
      return;
    }
    if (aborted) {
      // The status word holds the timeout.  A multi-split unit still takes its
      // ticket so that the unit's last CTA re-arms it (its output is garbage,
      // which the status reports); tickets stay consistent for the next call.
      if (u.nsplit > 1) ticket_merge<R, TC_DH, 128>(a, u, t, 1, reinterpret_cast<float*>(stages), s_last);
      return;
    }
    if (u.nsplit == 1) {
#pragma unroll
      for (int r = 0; r < R; r++)
        if (r < u.rows_valid) store_out(a, out_index(a, u, r, t, TC_DH), acc[r] / lsum[r]);
      return;
    }
    float* part = a.part + ((size_t)u.unit * a.max_splits + split) * R * (TC_DH + 2);
#pragma unroll
    for (int r = 0; r < R; r++) {
      part[r * (TC_DH + 2) + t] = acc[r];
      if (t == 0) {
        part[r * (TC_DH + 2) + TC_DH] = m[r];
        part[r * (TC_DH + 2) + TC_DH + 1] = lsum[r];
      }
    }
    ticket_merge<R, TC_DH, 128>(a, u, t, 1, reinterpret_cast<float*>(stages), s_last);
    return;
  }
  // producer and MMA warps: wait for the softmax warps, then release TMEM
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

template <bool BF16, int R, int NC>
int launch(hcu_context* h, const AttnArgs& args, dim3 grid, const CUtensorMap& tk, const CUtensorMap& tv) {
  constexpr int QS_BLK = NC * 128;
  constexpr size_t smem = 1024 + RING_BYTES + 6 * QS_BLK + 16 * 8 + 16 + (2 * 4 * R + 4 * R) * 4;
  auto kern = attn_decode_tc_kernel<BF16, R, NC>;
  static std::atomic<uint64_t> attr_done{0};  // per device
  HCU_TRY(once_per_device(attr_done, h->device, [&]() -> int {
    HCU_TRY(check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                       "hcu_attention: tc smem attribute"));
    HCU_TRY(check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1),
                       "hcu_attention: tc cluster attribute"));
    return HCU_OK;
  }));
  launch_decode(kern, grid, TC_THREADS, smem, h->stream, args, tk, tv);
  return after_launch("hcu_attention: tc launch");
}

}  // namespace

bool attn_tc_supported(int fmt, int Dh, int R) {
  if (Dh != TC_DH) return false;
  if (fmt == HCU_KV_F16) return R <= 16;
  if (fmt == HCU_KV_BF16) return R <= 8;
  if (fmt == HCU_KV_Q8_0) return R <= 4;  // attention_decode_q8tc.cu
  return false;
}

int launch_attn_tc(hcu_context* h, int fmt, int R, const AttnArgs& args, dim3 grid, const CUtensorMap& tk,
                   const CUtensorMap& tv) {
  if (fmt == HCU_KV_F16) {
    switch (R) {
      case 1: return launch<false, 1, 16>(h, args, grid, tk, tv);
      case 2: return launch<false, 2, 16>(h, args, grid, tk, tv);
      case 4: return launch<false, 4, 16>(h, args, grid, tk, tv);
      case 8: return launch<false, 8, 16>(h, args, grid, tk, tv);
      case 16: return launch<false, 16, 32>(h, args, grid, tk, tv);
    }
  } else if (fmt == HCU_KV_BF16) {
    switch (R) {
      case 1: return launch<true, 1, 16>(h, args, grid, tk, tv);
      case 2: return launch<true, 2, 16>(h, args, grid, tk, tv);
      case 4: return launch<true, 4, 16>(h, args, grid, tk, tv);
      case 8: return launch<true, 8, 32>(h, args, grid, tk, tv);
    }
  }
  return fail(HCU_EUNSUPPORTED, "hcu_attention: no tensor-core variant for format %d with %d rows", fmt, R);
}

}  // namespace hcu
