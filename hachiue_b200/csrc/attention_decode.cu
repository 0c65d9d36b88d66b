// attention_decode.cu - split-K flash-decoding GQA attention over the KV cache.
//
// Replaces attention_q8 (src/kernels.ts:1341-1426) and runAttentionQ8
// (src/wasm-backend.ts:826-895).  Semantics kept from the reference: grouped
// head map kvh = h / (H / KV), key range [jStart, pos] with
// jStart = pos + 1 - windowSize when windowSize > 0 and pos + 1 > windowSize,
// score scale 1/sqrt(Dh), online softmax, output acc / l.
//
// B200 design (the reference runs one 32-thread workgroup per (query, head),
// serial over keys, and re-reads each KV head once per query head):
//  * One CTA per (sequence, KV head, query block, key split).  All G = H/KV
//    query heads of the KV head (and up to 16/G queries) are the CTA's R
//    "rows", so every K/V byte crosses HBM once per call.
//  * A producer warp streams [TT tokens x Dh] K and V tiles (16 KB each) with
//    3-D TMA tile loads (cp.async.bulk.tensor) into a 3-stage mbarrier
//    ring; four consumer warps each own a quarter of every tile.
//  * q.k: each lane owns Dh/32 dimensions; partial dots for 32 (token, row)
//    pairs are summed across the warp with a transpose-reduce (31 shuffles
//    for 32 values instead of 5 per value).
//  * Online softmax per row in the log2 domain (q pre-scaled by log2(e)/sqrt(Dh)).
//  * Splits write (m, l, acc) partials to the handle's workspace; the last CTA
//    of a unit (atomic ticket, no spinning) merges them and writes out.
#include "attention.cuh"

namespace {

using namespace hcu;

constexpr int NW = 4;                   // consumer warps
constexpr int NTHREADS = (NW + 1) * 32; // + 1 TMA producer warp
// Pipeline stages and CTAs per SM: with few rows per CTA, three CTAs of two
// stages share an SM (more warps to hide load and shared-memory latency);
// with more rows the registers allow two CTAs of three stages.
__host__ __device__ constexpr bool three_ctas(int R, int DH) { return R <= 2 || (R <= 4 && DH == 128); }
__host__ __device__ constexpr int ctas_per_sm(int R, int DH) { return three_ctas(R, DH) ? 3 : 2; }
__host__ __device__ constexpr int stages_for(int R, int DH) { return three_ctas(R, DH) ? 2 : 3; }

template <int FMT, int DH>
struct Cfg {
  static constexpr int ES = FMT == HCU_KV_F32 ? 4 : (FMT == HCU_KV_Q8_0 ? 1 : 2);
  static constexpr int TT = 16384 / (DH * ES);  // tokens per tile
  static constexpr int TPW = TT / NW;           // tokens per warp per tile
  static constexpr int DPL = DH / 32;           // dims per lane
  static constexpr int TILE_BYTES = TT * DH * ES;
  static constexpr int SC_BYTES = FMT == HCU_KV_Q8_0 ? TT * (DH / 32) * 4 : 0;
  static constexpr int STAGE_BYTES = 2 * (TILE_BYTES + SC_BYTES);
};



// Four int8 values packed in a word, as exact f32 values, without the
// int-to-float conversion instruction (a quarter-rate pipe): with its sign bit
// flipped, each byte b + 128 becomes the low mantissa byte of 2^23, and
// subtracting 2^23 + 128 leaves b.
__device__ __forceinline__ void s8x4_to_f32(uint32_t w, float* f) {
  const uint32_t u = w ^ 0x80808080u;
  f[0] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)) - 8388736.f;
  f[1] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541)) - 8388736.f;
  f[2] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)) - 8388736.f;
  f[3] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543)) - 8388736.f;
}

// Loads the lane's DPL elements of tile row `row` as f32 (Q8_0: times the
// block scale, like `kQ * kS` in wasm-backend.ts:861-866).
template <int FMT, int DH>
__device__ __forceinline__ void load_row(const uint8_t* tile, const float* scales, float smul, int row, int lane,
                                         float (&v)[DH / 32]) {
  constexpr int DPL = DH / 32;
  if constexpr (FMT == HCU_KV_F32) {
    const float4* p = reinterpret_cast<const float4*>(tile + (size_t)row * DH * 4) + lane * (DPL / 4);
#pragma unroll
    for (int i = 0; i < DPL / 4; i++) {
      float4 x = p[i];
      v[4 * i] = x.x;
      v[4 * i + 1] = x.y;
      v[4 * i + 2] = x.z;
      v[4 * i + 3] = x.w;
    }
  } else if constexpr (FMT == HCU_KV_F16 || FMT == HCU_KV_BF16) {
    const uint32_t* p = reinterpret_cast<const uint32_t*>(tile + (size_t)row * DH * 2) + lane * (DPL / 2);
    uint32_t w[DPL / 2];
    if constexpr (DPL == 4) {
      uint2 x = *reinterpret_cast<const uint2*>(p);
      w[0] = x.x;
      w[1] = x.y;
    } else {
      uint4 x = *reinterpret_cast<const uint4*>(p);
      w[0] = x.x;
      w[1] = x.y;
      w[2] = x.z;
      w[3] = x.w;
    }
#pragma unroll
    for (int i = 0; i < DPL / 2; i++) {
      if constexpr (FMT == HCU_KV_F16) {
        float2 f = f16x2_to_f2(w[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
      } else {
        v[2 * i] = bf16_lo(w[i]);
        v[2 * i + 1] = bf16_hi(w[i]);
      }
    }
  } else {  // Q8_0
    const int8_t* p = reinterpret_cast<const int8_t*>(tile + (size_t)row * DH) + lane * DPL;
    const float s = scales[row * (DH / 32) + (lane * DPL) / 32] * smul;
    if constexpr (DPL == 4) {
      s8x4_to_f32(*reinterpret_cast<const uint32_t*>(p), v);
    } else {
      const uint2 xx = *reinterpret_cast<const uint2*>(p);
      s8x4_to_f32(xx.x, v);
      s8x4_to_f32(xx.y, v + 4);
    }
#pragma unroll
    for (int i = 0; i < DPL; i++) v[i] *= s;
  }
}

// Transpose-reduce: sums N per-lane values across the warp.  Afterwards lane L
// holds the totals of entries (L*N)/32 + i, i < max(N/32, 1).
template <int N>
__device__ __forceinline__ void treduce(float (&v)[N], int lane) {
  int n = N;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    if (n >= 2) {
      const int half = n / 2;
      const bool up = (lane & off) != 0;
#pragma unroll
      for (int i = 0; i < N / 2; i++) {
        if (i < half) {
          float send = up ? v[i] : v[i + half];
          float keep = up ? v[i + half] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
      }
      n = half;
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
    }
  }
}

template <int FMT, int DH, int R>
__global__ void __launch_bounds__(NTHREADS, ctas_per_sm(R, DH))
    attn_decode_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                       const __grid_constant__ CUtensorMap tmKs, const __grid_constant__ CUtensorMap tmVs,
                       const AttnArgs a) {
  using C = Cfg<FMT, DH>;
  constexpr int TT = C::TT, TPW = C::TPW, DPL = C::DPL, NST = stages_for(R, DH);
  constexpr int TG = (32 / R) < TPW ? (32 / R > 0 ? 32 / R : 1) : TPW;  // tokens per reduce group
  constexpr int NV = TG * R;                                            // values per reduce
  constexpr int NPL = NV >= 32 ? NV / 32 : 1;                           // results per lane
  constexpr int TPL = (TPW + 31) / 32;                                  // softmax entries per lane

  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NST * C::STAGE_BYTES);
  uint64_t* empty = full + NST;
  float* sc_all = reinterpret_cast<float*>(empty + NST);
  int* s_last = reinterpret_cast<int*>(sc_all + NW * TPW * R);  // in the dynamic memory: no static padding

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.x;
  const AttnUnit u = attn_unit(a, split);
  // In the cluster form every CTA of the unit's cluster reaches the cluster
  // barriers, with or without work; otherwise a CTA without work leaves here,
  // uniformly and before any barrier.
  const bool clus = a.cluster != 0;
  const bool badarg = u.nsplit > (int)gridDim.x;
  if (badarg) {  // max_context under-stated by the caller: refuse, never half-merge
    if (split == 0 && threadIdx.x == 0) atomicOr(a.status, HCU_DEVERR_BADARG);
    if (!clus) return;
  }
  const bool has_work = !badarg && split < u.nsplit;
  if (!clus && !has_work) return;
  const int g = u.g, b = u.b, pb = u.pb, q0 = u.q0, qn = u.qn;
  const int k_lo = u.k_lo, k_hi = u.k_hi;
  const long long roff = u.roff;
  const int ntiles = has_work ? (k_hi - k_lo + TT - 1) / TT : 0;

  if (tid == 0) {
    for (int s = 0; s < NST; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NW);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == NW) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_tensormap(&tmK);
      prefetch_tensormap(&tmV);
      for (int it = 0; it < ntiles; ++it) {
        const int s = it % NST, rnd = it / NST;
        if (rnd > 0 && !mbar_wait(&empty[s], (rnd - 1) & 1, a.status)) break;
        uint8_t* st = stages + s * C::STAGE_BYTES;
        const int row = (int)(roff + k_lo + it * TT);
        mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
        tma_load_3d(st, &tmK, &full[s], 0, g, row);
        tma_load_3d(st + C::TILE_BYTES, &tmV, &full[s], 0, g, row);
        if constexpr (FMT == HCU_KV_Q8_0) {
          tma_load_3d(st + 2 * C::TILE_BYTES, &tmKs, &full[s], 0, g, row);
          tma_load_3d(st + 2 * C::TILE_BYTES + C::SC_BYTES, &tmVs, &full[s], 0, g, row);
        }
      }
    }
    // the producer takes no part in the epilogue (named barriers below); in the
    // cluster form it still joins the cluster barriers
    if (!clus) return;
    cluster_sync_all();
    cluster_sync_all();
    return;
  }

  // ---------------- consumers ----------------
  float qv[R][DPL];
  int jlo[R], jhi[R];
#pragma unroll
  for (int r = 0; r < R; r++) {
    const int qi = q0 + r / a.G;
    const bool valid = (r < a.QB * a.G) && (r / a.G < qn);
    const int h = g * a.G + (r % a.G);
    const int pos = pb + qi;
    jlo[r] = valid ? ((a.window > 0 && pos + 1 > a.window) ? pos + 1 - a.window : 0) : 1;
    jhi[r] = valid ? pos : 0;
    if (valid) {
      const float4* qp = reinterpret_cast<const float4*>(a.q + (((long long)b * a.S + qi) * a.H + h) * DH) +
                         lane * (DPL / 4);
#pragma unroll
      for (int i = 0; i < DPL / 4; i++) {
        float4 x = __ldg(qp + i);
        qv[r][4 * i] = x.x * a.qscale;
        qv[r][4 * i + 1] = x.y * a.qscale;
        qv[r][4 * i + 2] = x.z * a.qscale;
        qv[r][4 * i + 3] = x.w * a.qscale;
      }
    } else {
#pragma unroll
      for (int i = 0; i < DPL; i++) qv[r][i] = 0.f;
    }
  }

  float m[R], l[R], acc[R][DPL];
#pragma unroll
  for (int r = 0; r < R; r++) {
    m[r] = -1e30f;
    l[r] = 0.f;
#pragma unroll
    for (int i = 0; i < DPL; i++) acc[r][i] = 0.f;
  }
  float* sc = sc_all + warp * TPW * R;
  bool aborted = false;

  for (int it = 0; it < ntiles; ++it) {
    const int s = it % NST, rnd = it / NST;
    if (!mbar_wait(&full[s], rnd & 1, a.status)) {
      aborted = true;
      break;
    }
    const uint8_t* st = stages + s * C::STAGE_BYTES;
    const uint8_t* ktile = st;
    const uint8_t* vtile = st + C::TILE_BYTES;
    const float* kscale = reinterpret_cast<const float*>(st + 2 * C::TILE_BYTES);
    const float* vscale = reinterpret_cast<const float*>(st + 2 * C::TILE_BYTES + C::SC_BYTES);
    const int wk0 = k_lo + it * TT + warp * TPW;  // key index of this warp's first row
    const int wrow0 = warp * TPW;

    // ---- scores: sc[t * R + r] = q_r . k_t (log2 domain) ----
#pragma unroll
    for (int t0 = 0; t0 < TPW; t0 += TG) {
      float part[NV];
#pragma unroll
      for (int tt = 0; tt < TG; tt++) {
        float kvec[DPL];
        load_row<FMT, DH>(ktile, kscale, a.q8_smul, wrow0 + t0 + tt, lane, kvec);
#pragma unroll
        for (int r = 0; r < R; r++) {
          float d = 0.f;
#pragma unroll
          for (int i = 0; i < DPL; i++) d = fmaf(qv[r][i], kvec[i], d);
          part[tt * R + r] = d;
        }
      }
      treduce<NV>(part, lane);
      const int idx = (lane * NV) >> 5;
      if (NV >= 32 || (lane & ((32 / NV) - 1)) == 0) {
#pragma unroll
        for (int i = 0; i < NPL; i++) sc[t0 * R + idx + i] = part[i];
      }
    }
    __syncwarp();

    // ---- online softmax per row over this warp's TPW keys ----
    float corr[R];
#pragma unroll
    for (int r = 0; r < R; r++) {
      float sv[TPL];
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < TPL; i++) {
        const int t = lane + 32 * i;
        sv[i] = -INFINITY;
        if (t < TPW) {
          const int key = wk0 + t;
          if (key >= jlo[r] && key <= jhi[r] && key < k_hi) sv[i] = sc[t * R + r];
          mx = fmaxf(mx, sv[i]);
        }
      }
      mx = warp_max(mx);
      const float mnew = fmaxf(m[r], mx);
      corr[r] = exp2f(m[r] - mnew);
      float ps = 0.f;
#pragma unroll
      for (int i = 0; i < TPL; i++) {
        const int t = lane + 32 * i;
        if (t < TPW) {
          const float p = exp2f(sv[i] - mnew);
          sc[t * R + r] = p;
          ps += p;
        }
      }
      ps = warp_sum(ps);
      l[r] = l[r] * corr[r] + ps;
      m[r] = mnew;
    }
    __syncwarp();
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
      for (int i = 0; i < DPL; i++) acc[r][i] *= corr[r];

    // ---- acc += p . V over the warp's valid rows ----
    const int tcount = min(TPW, k_hi - wk0);
    constexpr int PV_UNROLL = R <= 4 ? 4 : 1;  // more rows leave no registers to unroll with
#pragma unroll PV_UNROLL
    for (int t = 0; t < tcount; t++) {
      float vvec[DPL];
      load_row<FMT, DH>(vtile, vscale, a.q8_smul, wrow0 + t, lane, vvec);
      float p[R];
      if constexpr (R % 4 == 0) {
#pragma unroll
        for (int r = 0; r < R; r += 4) {
          float4 x = *reinterpret_cast<const float4*>(sc + t * R + r);
          p[r] = x.x;
          p[r + 1] = x.y;
          p[r + 2] = x.z;
          p[r + 3] = x.w;
        }
      } else {
#pragma unroll
        for (int r = 0; r < R; r++) p[r] = sc[t * R + r];
      }
#pragma unroll
      for (int r = 0; r < R; r++)
#pragma unroll
        for (int i = 0; i < DPL; i++) acc[r][i] = fmaf(p[r], vvec[i], acc[r][i]);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  // ---------------- merge the four warps ----------------
  named_bar(1, NW * 32);  // every consumer is done with the stage buffers
  float* cb = reinterpret_cast<float*>(stages);  // [NW][R][DH]
  float* cm = cb + NW * R * DH;                  // [NW][R]
  float* cl = cm + NW * R;                       // [NW][R]
#pragma unroll
  for (int r = 0; r < R; r++) {
#pragma unroll
    for (int i = 0; i < DPL; i++) cb[(warp * R + r) * DH + lane * DPL + i] = acc[r][i];
    if (lane == 0) {
      cm[warp * R + r] = m[r];
      cl[warp * R + r] = l[r];
    }
  }
  // One decision for all consumer warps (a bounded wait may give up in some
  // warps only): the merge below synchronises them on named barriers.
  aborted = !named_bar_and(1, NW * 32, !aborted);
  if (clus) {
    // This CTA's partial into its own shared memory (an empty one without
    // work or after a timed-out wait), then the merge across the cluster.
    float* cp = cl + NW * R;  // [R][DH + 2], after the per-warp partials read below
    for (int e = tid; e < R * DH; e += NW * 32) {
      const int r = e / DH, d = e % DH;
      float M = -1e30f;
#pragma unroll
      for (int w = 0; w < NW; w++) M = fmaxf(M, cm[w * R + r]);
      float L = 0.f, A = 0.f;
#pragma unroll
      for (int w = 0; w < NW; w++) {
        const float f = exp2f(cm[w * R + r] - M);
        L += cl[w * R + r] * f;
        A += cb[(w * R + r) * DH + d] * f;
      }
      const bool keep = has_work && !aborted;
      cp[r * (DH + 2) + d] = keep ? A : 0.f;
      if (d == 0) {
        cp[r * (DH + 2) + DH] = keep ? M : -1e30f;
        cp[r * (DH + 2) + DH + 1] = keep ? L : 0.f;
      }
    }
    cluster_sync_all();
    cluster_merge<R, DH, NW * 32>(a, u, badarg ? 0 : min(u.nsplit, (int)gridDim.x), cp, tid, !badarg);
    cluster_sync_all();
    return;
  }
  if (aborted) {
    // The status word holds the timeout.  A multi-split unit still takes its
    // ticket so that the unit's last CTA re-arms it (its output is garbage,
    // which the status reports); tickets stay consistent for the next call.
    if (u.nsplit > 1) ticket_merge<R, DH, NW * 32>(a, u, tid, 1, reinterpret_cast<float*>(stages), s_last);
    return;
  }

  const int rows_valid = u.rows_valid;
  float* part = a.part + ((size_t)u.unit * a.max_splits + split) * R * (DH + 2);
  for (int e = tid; e < R * DH; e += NW * 32) {
    const int r = e / DH, d = e % DH;
    float M = -1e30f;
#pragma unroll
    for (int w = 0; w < NW; w++) M = fmaxf(M, cm[w * R + r]);
    float L = 0.f, A = 0.f;
#pragma unroll
    for (int w = 0; w < NW; w++) {
      const float f = exp2f(cm[w * R + r] - M);
      L += cl[w * R + r] * f;
      A += cb[(w * R + r) * DH + d] * f;
    }
    if (u.nsplit == 1) {
      if (r < rows_valid) store_out(a, out_index(a, u, r, d, DH), A / L);
    } else {
      part[r * (DH + 2) + d] = A;
      if (d == 0) {
        part[r * (DH + 2) + DH] = M;
        part[r * (DH + 2) + DH + 1] = L;
      }
    }
  }
  if (u.nsplit == 1) return;
  named_bar(1, NW * 32);  // cb / cm / cl are read above; the merge reuses the stage memory
  ticket_merge<R, DH, NW * 32>(a, u, tid, 1, reinterpret_cast<float*>(stages), s_last);
  (void)b;
  (void)pb;
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
template <int FMT, int DH, int R>
int launch_t(hcu_context* h, const AttnArgs& args, dim3 grid, const CUtensorMap& tk, const CUtensorMap& tv,
             const CUtensorMap& tks, const CUtensorMap& tvs) {
  using C = Cfg<FMT, DH>;
  auto kern = attn_decode_kernel<FMT, DH, R>;
  constexpr int NST = stages_for(R, DH);
  const size_t smem = NST * C::STAGE_BYTES + 2 * NST * sizeof(uint64_t) + NW * C::TPW * R * sizeof(float) + 16;
  // the per-warp partials and the split merge reuse the stage buffers
  static_assert((NW * R * DH + 2 * NW * R + R * (DH + 2)) * 4 <= NST * C::STAGE_BYTES &&
                    kMaxSplits * R * 4 <= NST * C::STAGE_BYTES,
                "merge buffers exceed the stage memory");
  static std::atomic<uint64_t> attr_done{0};  // per device
  HCU_TRY(once_per_device(attr_done, h->device, [&]() -> int {
    HCU_TRY(check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                       "hcu_attention: smem attribute"));
    // clusters of up to kMaxClusterSplits (16) CTAs: above the portable 8
    HCU_TRY(check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1),
                       "hcu_attention: cluster attribute"));
    return HCU_OK;
  }));
  launch_decode(kern, grid, NTHREADS, smem, h->stream, args, tk, tv, tks, tvs);
  return after_launch("hcu_attention: launch");
}

template <int FMT, int DH>
int launch_r(hcu_context* h, int R, const AttnArgs& args, dim3 grid, const CUtensorMap& tk, const CUtensorMap& tv,
             const CUtensorMap& tks, const CUtensorMap& tvs) {
  switch (R) {
    case 1: return launch_t<FMT, DH, 1>(h, args, grid, tk, tv, tks, tvs);
    case 2: return launch_t<FMT, DH, 2>(h, args, grid, tk, tv, tks, tvs);
    case 4: return launch_t<FMT, DH, 4>(h, args, grid, tk, tv, tks, tvs);
    case 8: return launch_t<FMT, DH, 8>(h, args, grid, tk, tv, tks, tvs);
    case 16:
      if constexpr (DH == 128) return launch_t<FMT, DH, 16>(h, args, grid, tk, tv, tks, tvs);
      break;
  }
  return fail(HCU_EUNSUPPORTED, "hcu_attention: %d rows per CTA not built for Dh=%d", R, DH);
}

template <int FMT>
int launch_d(hcu_context* h, int DH, int R, const AttnArgs& args, dim3 grid, const CUtensorMap& tk,
             const CUtensorMap& tv, const CUtensorMap& tks, const CUtensorMap& tvs) {
  if (DH == 128) return launch_r<FMT, 128>(h, R, args, grid, tk, tv, tks, tvs);
  return launch_r<FMT, 256>(h, R, args, grid, tk, tv, tks, tvs);
}

int tile_tokens(int fmt, int dh) {
  const int es = fmt == HCU_KV_F32 ? 4 : (fmt == HCU_KV_Q8_0 ? 1 : 2);
  return 16384 / (dh * es);
}

}  // namespace

extern "C" int hcu_attention(hcu_handle h, const hcu_attention_params* p, const float* q, const hcu_kv_cache* kv,
                             float* out) {
  HCU_TRY(hcu::begin_op(h, "hcu_attention"));
  if (!p || !q || !kv || !out || !kv->k || !kv->v) return fail(HCU_EINVAL, "hcu_attention: null argument");
  const int S = (int)p->S, H = (int)p->H, KV = (int)p->KV, Dh = (int)p->Dh;
  const int batch = p->batch ? (int)p->batch : 1;
  // The WGSL Q8_0 convention differs only in its scale (amax instead of
  // amax / 127): same kernels, with the scale multiplied by 1/127.
  const bool q8_wgsl = kv->format == HCU_KV_Q8_0_WGSL;
  const int fmt = q8_wgsl ? HCU_KV_Q8_0 : (int)kv->format;
  if (S < 1 || H < 1 || KV < 1) return fail(HCU_EINVAL, "hcu_attention: S, H and KV must be positive");
  if (H % KV) return fail(HCU_EINVAL, "hcu_attention: H (%d) is not a multiple of KV (%d)", H, KV);
  if (Dh != 128 && Dh != 256) return fail(HCU_EUNSUPPORTED, "hcu_attention: Dh=%d (built: 128, 256)", Dh);
  if (fmt < HCU_KV_F32 || fmt > HCU_KV_Q8_0)
    return fail(HCU_EINVAL, "hcu_attention: unknown KV format %u", kv->format);
  if (fmt == HCU_KV_Q8_0 && (!kv->k_scale || !kv->v_scale))
    return fail(HCU_EINVAL, "hcu_attention: Q8_0 cache needs k_scale and v_scale");
  if (batch > 1 && !p->pos_base && p->max_context == 0)
    ;  // every sequence uses posBase: max_context defaults below
  if (reinterpret_cast<uintptr_t>(q) % 16 || reinterpret_cast<uintptr_t>(out) % 16)
    return fail(HCU_EINVAL, "hcu_attention: q and out must be 16-byte aligned");
  const int G = H / KV;
  // The tcgen05 kernels serve f16 / bf16 (attention_decode_tc.cu) and Q8_0
  // (attention_decode_q8tc.cu) caches with Dh = 128; every other combination
  // (and HCU_OPT_ATTN_CUDA_CORES) uses the CUDA-core kernel.
  const bool force_cuda = h->opt_attn_cuda_cores != 0;
  const int rmax_cuda = Dh == 128 ? 16 : 8;
  const int rmax_tc = fmt == HCU_KV_F16 ? 16 : (fmt == HCU_KV_Q8_0 ? 4 : 8);
  bool use_tc = !force_cuda && hcu::attn_tc_supported(fmt, Dh, G);
  const int rmax = use_tc ? rmax_tc : rmax_cuda;
  if (G > rmax) return fail(HCU_EUNSUPPORTED, "hcu_attention: group size %d > %d", G, rmax);
  const int QB = S < rmax / G ? S : rmax / G;
  int R = 1;
  while (R < QB * G) R <<= 1;
  if (use_tc && !hcu::attn_tc_supported(fmt, Dh, R)) use_tc = false;
  const int nqb = (S + QB - 1) / QB;
  if ((long long)batch * nqb > 65535) return fail(HCU_EINVAL, "hcu_attention: batch x query blocks > 65535");
  if (KV > 65535) return fail(HCU_EINVAL, "hcu_attention: KV > 65535");
  const long long max_ctx = p->max_context ? (long long)p->max_context : (long long)p->posBase + S;
  if (max_ctx < S) return fail(HCU_EINVAL, "hcu_attention: max_context < S");
  const int W = (int)p->windowSize;
  long long max_range = max_ctx;
  if (W > 0 && (long long)W + QB - 1 < max_range) max_range = (long long)W + QB - 1;
  if (batch == 1 && !p->pos_base && (long long)p->posBase + S > (long long)kv->rows)
    return fail(HCU_EINVAL, "hcu_attention: cache holds %u rows, need posBase+S = %lld", kv->rows,
                (long long)p->posBase + S);
  if (kv->rows == 0 || kv->rows > 0x7fffffffu) return fail(HCU_EINVAL, "hcu_attention: bad cache row count");

  // Key splits: about 8 CTAs per SM over the whole call for the tensor-core
  // kernel, 24 for the CUDA-core one (three resident per SM, and shorter
  // splits balance its uneven sequences: cfg2's Q8_0 shapes 289 -> 259 us),
  // at most kMaxSplits per unit, each a whole number of tiles.
  const int TT = use_tc ? hcu::kTcTile : tile_tokens(fmt, Dh);
  const long long units = (long long)batch * KV * nqb;
  if (units > kMaxUnits)
    return fail(HCU_EINVAL, "hcu_attention: batch x KV x query blocks = %lld > %d", units, kMaxUnits);
  long long target = (use_tc ? 8LL : 24LL) * h->sm_count;
  long long want_splits = (target + units - 1) / units;
  if (want_splits < 1) want_splits = 1;
  long long chunk = (max_range + want_splits - 1) / want_splits;
  // Few units (a single sequence): CUDA-core splits of at least two tiles, so
  // each CTA's second load overlaps its first tile's work and the merge reads
  // half as many partials (cfg1's shapes: 10.2 -> 9.1 us per step).
  if (!use_tc && chunk < 2LL * TT) chunk = 2LL * TT;
  if (h->opt_attn_chunk > 0) chunk = h->opt_attn_chunk;
  const long long min_chunk = (max_range + kMaxSplits - 1) / kMaxSplits;
  if (chunk < min_chunk) chunk = min_chunk;
  chunk = ((chunk + TT - 1) / TT) * TT;
  if (chunk < TT) chunk = TT;
  // Split-merge tickets live in a fixed region at the start of the workspace so
  // that no call's partials ever overlap another call's tickets (each ticket is
  // re-armed to 0 by the CTA that consumes it).
  const size_t cnt_bytes = kTicketBytes;
  auto need = [&](long long c) {
    long long ms = (max_range + c - 1) / c;
    return cnt_bytes + (size_t)units * ms * R * (Dh + 2) * sizeof(float);
  };
  while (need(chunk) > h->workspace_bytes && chunk < max_range) chunk *= 2;
  if (need(chunk) > h->workspace_bytes)
    return fail(HCU_ENOMEM, "hcu_attention: workspace of %zu bytes too small (need %zu)", h->workspace_bytes,
                need(chunk));
  const long long max_splits = (max_range + chunk - 1) / chunk;
  if (max_splits > kMaxSplits || chunk > 0x7fffffff) return fail(HCU_EINVAL, "hcu_attention: too many splits");
  // A small launch merges its splits inside thread-block clusters
  // (one per unit, through distributed shared memory) instead of through
  // tickets and partials in L2: its merge is then a few hundred cycles rather
  // than a few microseconds of dependent L2 round trips.
  const bool cluster =
      max_splits >= 2 && max_splits <= hcu::kMaxClusterSplits && units * max_splits <= 2LL * h->sm_count;

  // TMA descriptors over the whole cache: dims (Dh, KV, rows).  The tensor-core
  // kernel loads 64-element (128-byte) boxes with the 128-byte swizzle its
  // MMA operand descriptors expect.
  const int es = fmt == HCU_KV_F32 ? 4 : (fmt == HCU_KV_Q8_0 ? 1 : 2);
  const CUtensorMapDataType dt = fmt == HCU_KV_F32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : fmt == HCU_KV_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                 : fmt == HCU_KV_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  CUtensorMap tk, tv, tks, tvs;
  {
    uint64_t dims[3] = {(uint64_t)Dh, (uint64_t)KV, (uint64_t)kv->rows};
    uint64_t strides[2] = {(uint64_t)Dh * es, (uint64_t)KV * Dh * es};
    // 128-byte boxes for the tensor cores: 64 16-bit or 128 8-bit elements
    uint32_t box[3] = {use_tc ? (fmt == HCU_KV_Q8_0 ? 128u : 64u) : (uint32_t)Dh, 1u, (uint32_t)TT};
    const CUtensorMapSwizzle sw = use_tc ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE;
    HCU_TRY(hcu::make_tensor_map(&tk, dt, 3, kv->k, dims, strides, box, sw));
    HCU_TRY(hcu::make_tensor_map(&tv, dt, 3, kv->v, dims, strides, box, sw));
  }
  if (fmt == HCU_KV_Q8_0) {
    uint64_t dims[3] = {(uint64_t)Dh / 32, (uint64_t)KV, (uint64_t)kv->rows};
    uint64_t strides[2] = {(uint64_t)Dh / 32 * 4, (uint64_t)KV * Dh / 32 * 4};
    uint32_t box[3] = {(uint32_t)Dh / 32, 1u, (uint32_t)TT};
    HCU_TRY(hcu::make_tensor_map(&tks, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, kv->k_scale, dims, strides, box,
                                 CU_TENSOR_MAP_SWIZZLE_NONE));
    HCU_TRY(hcu::make_tensor_map(&tvs, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, kv->v_scale, dims, strides, box,
                                 CU_TENSOR_MAP_SWIZZLE_NONE));
  } else {
    tks = tk;
    tvs = tv;
  }

  AttnArgs args{};
  args.q = q;
  args.out = out;
  args.pos_base = p->pos_base;
  args.row_off = p->kv_row_offset;
  args.seq_row_stride = p->seq_row_stride;
  args.S = S;
  args.H = H;
  args.KV = KV;
  args.G = G;
  args.QB = QB;
  args.nqb = nqb;
  args.window = W;
  args.pos_base_default = (int)p->posBase;
  args.chunk = (int)chunk;
  args.max_splits = (int)max_splits;
  args.qscale = kLog2e / sqrtf((float)Dh);
  args.counters = static_cast<int*>(h->workspace);
  args.cluster = cluster ? 1 : 0;
  args.part = reinterpret_cast<float*>(static_cast<char*>(h->workspace) + cnt_bytes);
  args.status = h->dev_status;
  args.gate = p->gate;
  args.q8_smul = q8_wgsl ? 1.f / 127.f : 1.f;
  dim3 grid((unsigned)max_splits, (unsigned)KV, (unsigned)(batch * nqb));
  if (use_tc && fmt == HCU_KV_Q8_0) return hcu::launch_attn_q8tc(h, R, args, grid, tk, tv, tks, tvs);
  if (use_tc) return hcu::launch_attn_tc(h, fmt, R, args, grid, tk, tv);
  switch (fmt) {
    case HCU_KV_F32: return launch_d<HCU_KV_F32>(h, Dh, R, args, grid, tk, tv, tks, tvs);
    case HCU_KV_F16: return launch_d<HCU_KV_F16>(h, Dh, R, args, grid, tk, tv, tks, tvs);
    case HCU_KV_BF16: return launch_d<HCU_KV_BF16>(h, Dh, R, args, grid, tk, tv, tks, tvs);
    default: return launch_d<HCU_KV_Q8_0>(h, Dh, R, args, grid, tk, tv, tks, tvs);
  }
}
