// deltanet.cu - Gated DeltaNet g/beta and the recurrent (decode / short
// segment) gated delta-rule scan.
//
// deltanet_gbeta (src/kernels.ts:1471-1491, JS src/wasm-backend.ts:1036-1045):
//   g = aNeg[h] * softplus(a + dtBias[h])  with the stable softplus
//   max(x,0) + log(1 + exp(-|x|)), beta = sigmoid(b).  Computed in f64 like
//   the JS, stored f32.
//
// deltanet_recur (src/kernels.ts:1496-1573, JS src/wasm-backend.ts:1047-1102),
// per V head h (QK head hk = h % HK, the tiled map) and token t:
//   k^ = k / sqrt(|k|^2 + 1e-6),  q^ = q / sqrt(|q|^2 + 1e-6) / sqrt(DK)
//   S *= exp(g);  kv = S^T k^;  delta = (v - kv) * beta;  S += k^ delta^T
//   o = S^T q^
// with the state S stored [dk][dv] as in the reference.
//
// B200 design: the reference runs ONE 128-thread workgroup per V head (NV = 32
// workgroups for the whole GPU) with a private 128-float array per thread.
// Here one 256-thread CTA owns one (sequence, V head) 128x128 f32 state held in
// registers: warp w owns dk rows [16w, 16w+16), lane l owns dv columns
// [4l, 4l+4), so every state row is one coalesced 512-byte access and the state
// crosses HBM exactly once in and once out per call, whatever S is.  Both
// column reductions (S^T k^ and S^T q^) come from the same pass over the
// decayed state; the output uses o = S_dec^T q^ + delta * (k^ . q^), which is
// S_new^T q^ without a second reduction.
#include "common.cuh"
#include "context.h"

namespace {

using namespace hcu;

constexpr int DN_D = 128;       // DK = DV
constexpr int DN_THREADS = 256; // 8 warps x 16 rows

struct DnArgs {
  const float* qkv;
  const float* gbeta;   // pre-computed [2, S, H] per sequence (or null when fused)
  const float* a;       // fused: [S, H] per sequence
  const float* b;
  const float* a_neg;
  const float* dt_bias;
  const float* state_in;
  float* state_out;
  float* core;
  int S, H, HK, load_state;
  long long qkv_stride, gbeta_stride, ab_stride, state_stride, core_stride;
  uint32_t* status;  // device status word (bounded waits of the step kernel)
  // Layer step only (conv1d_causal before, deltanet_norm_gate after the recurrence):
  // qkv holds the pre-conv mix [C]; conv state [K-1][C] in / out (ping-pong);
  // z [H*DV] gate; gamma [DV]; out [H*DV] the gated RMSNorm of the core row.
  const float* conv_w;
  const float* conv_in;
  float* conv_out;
  const float* z;
  const float* gamma;
  float* out;
  float eps;
  long long conv_stride, z_stride, out_stride;
};

constexpr int LAYER_K = 4;  // conv1d width of the fused layer step (qwen35 convKernel)

__device__ __forceinline__ void gbeta_f64(float a, float dtb, float aneg, float bb, float* g, float* beta) {
  const double x = (double)a + (double)dtb;
  const double sp = (x > 0 ? x : 0.0) + log(1.0 + exp(-fabs(x)));
  *g = (float)((double)aneg * sp);
  *beta = (float)(1.0 / (1.0 + exp(-(double)bb)));
}

__global__ void __launch_bounds__(256) gbeta_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                                    const float* __restrict__ a_neg,
                                                    const float* __restrict__ dt_bias, float* __restrict__ out,
                                                    int n, int H) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int h = i % H;
  float g, beta;
  gbeta_f64(a[i], dt_bias[h], a_neg[h], b[i], &g, &beta);
  out[i] = g;
  out[n + i] = beta;
}

template <bool FUSED>
__global__ void __launch_bounds__(DN_THREADS, 2) deltanet_recur_kernel(const DnArgs p) {
  __shared__ float qs[DN_D], ks[DN_D];
  __shared__ float red_k[8][DN_D], red_q[8][DN_D];
  __shared__ float sdelta[DN_D];
  __shared__ float scal[6];  // ik, iq, k.q (raw), g, beta

  const int h = blockIdx.x, bidx = blockIdx.y;
  const int hk = h % p.HK;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long key_dim = (long long)p.HK * DN_D;
  const long long conv_dim = 2 * key_dim + (long long)p.H * DN_D;
  const float* qkv = p.qkv + bidx * p.qkv_stride;
  const long long soff = bidx * p.state_stride + (long long)h * DN_D * DN_D;
  float* core = p.core + bidx * p.core_stride;

  // ---- state tile: rows [16w, 16w+16), cols [4l, 4l+4) ----
  float4 st[16];
  if (p.load_state) {
    const float4* src = reinterpret_cast<const float4*>(p.state_in + soff);
#pragma unroll
    for (int i = 0; i < 16; i++) st[i] = __ldcs(src + (warp * 16 + i) * (DN_D / 4) + lane);
  } else {
#pragma unroll
    for (int i = 0; i < 16; i++) st[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }

  const float inv_sqrt_dk = rsqrtf((float)DN_D);
  for (int t = 0; t < p.S; t++) {
    const float* row = qkv + (long long)t * conv_dim;
    if (tid < DN_D)
      qs[tid] = row[(long long)hk * DN_D + tid];
    else
      ks[tid - DN_D] = row[key_dim + (long long)hk * DN_D + (tid - DN_D)];
    if (tid == 0) {
      float g, beta;
      if constexpr (FUSED) {
        const long long i = bidx * p.ab_stride + (long long)t * p.H + h;
        gbeta_f64(p.a[i], p.dt_bias[h], p.a_neg[h], p.b[i], &g, &beta);
      } else {
        const float* gb = p.gbeta + bidx * p.gbeta_stride;
        g = gb[(long long)t * p.H + h];
        beta = gb[(long long)p.S * p.H + (long long)t * p.H + h];
      }
      scal[3] = expf(g);
      scal[4] = beta;
    }
    __syncthreads();
    if (warp < 3) {
      float v = 0.f;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const float x = warp == 0 ? qs[lane * 4 + i] : ks[lane * 4 + i];
        const float y = warp == 2 ? qs[lane * 4 + i] : x;
        v = fmaf(x, y, v);
      }
      v = warp_sum(v);
      if (lane == 0) {
        if (warp == 0) scal[1] = rsqrtf(v + 1e-6f) * inv_sqrt_dk;
        if (warp == 1) scal[0] = rsqrtf(v + 1e-6f);
        if (warp == 2) scal[2] = v;
      }
    }
    __syncthreads();
    const float ik = scal[0], iq = scal[1], gt = scal[3], bt = scal[4];
    const float kq = scal[2] * ik * iq;  // k^ . q^

    float4 pk = make_float4(0.f, 0.f, 0.f, 0.f), pq = pk;
#pragma unroll
    for (int i = 0; i < 16; i++) {
      const float kh = ks[warp * 16 + i] * ik;
      const float qh = qs[warp * 16 + i] * iq;
      st[i].x *= gt;
      st[i].y *= gt;
      st[i].z *= gt;
      st[i].w *= gt;
      pk.x = fmaf(st[i].x, kh, pk.x);
      pk.y = fmaf(st[i].y, kh, pk.y);
      pk.z = fmaf(st[i].z, kh, pk.z);
      pk.w = fmaf(st[i].w, kh, pk.w);
      pq.x = fmaf(st[i].x, qh, pq.x);
      pq.y = fmaf(st[i].y, qh, pq.y);
      pq.z = fmaf(st[i].z, qh, pq.z);
      pq.w = fmaf(st[i].w, qh, pq.w);
    }
    *reinterpret_cast<float4*>(&red_k[warp][lane * 4]) = pk;
    *reinterpret_cast<float4*>(&red_q[warp][lane * 4]) = pq;
    __syncthreads();
    if (tid < DN_D) {
      float kvd = 0.f, qd = 0.f;
#pragma unroll
      for (int w = 0; w < 8; w++) {
        kvd += red_k[w][tid];
        qd += red_q[w][tid];
      }
      const float v = row[2 * key_dim + (long long)h * DN_D + tid];
      const float delta = (v - kvd) * bt;
      sdelta[tid] = delta;
      core[((long long)t * p.H + h) * DN_D + tid] = fmaf(delta, kq, qd);
    }
    __syncthreads();
    const float4 d4 = *reinterpret_cast<const float4*>(&sdelta[lane * 4]);
#pragma unroll
    for (int i = 0; i < 16; i++) {
      const float kh = ks[warp * 16 + i] * ik;
      st[i].x = fmaf(kh, d4.x, st[i].x);
      st[i].y = fmaf(kh, d4.y, st[i].y);
      st[i].z = fmaf(kh, d4.z, st[i].z);
      st[i].w = fmaf(kh, d4.w, st[i].w);
    }
    __syncthreads();  // qs / ks / scal are rewritten by the next token
  }

  float4* dst = reinterpret_cast<float4*>(p.state_out + soff);
#pragma unroll
  for (int i = 0; i < 16; i++) __stcs(dst + (warp * 16 + i) * (DN_D / 4) + lane, st[i]);
}

// Single-token step (S = 1, the decode case) as a persistent kernel, two
// CTAs per SM: each walks (sequence, V head) items, and while it updates one
// state (in registers) the next item's state is already on its way into shared
// memory by bulk copy, with the next q / k / v and a / b in registers, so the
// SM's HBM stream does not pause for the reductions and barriers of an update.
// The arithmetic is the per-token body of deltanet_recur_kernel.
//
// LAYER adds the layer's neighbours of the recurrence (src/engine.ts:1358-1400)
// to the same pass: the causal conv1d + SiLU of the token's q / k / v channels
// from the pre-conv mix and the conv state (conv1d_causal, src/kernels.ts:
// 1431-1466), and the gated RMSNorm of the output row (deltanet_norm_gate,
// src/kernels.ts:1578-1611), so neither qkvConv nor core makes an HBM round
// trip.  Each item writes the new conv state of its V channels; the q / k
// channels of QK head hk are written by the item of V head hk.
template <bool FUSED, bool LAYER>
__global__ void __launch_bounds__(DN_THREADS, 2) deltanet_step_kernel(const DnArgs p, int n_items) {
  extern __shared__ __align__(16) float sstate[];  // [128][128] f32: the next item's state
  __shared__ float qs[DN_D], ks[DN_D];
  __shared__ float red_k[8][DN_D], red_q[8][DN_D];
  __shared__ float sdelta[DN_D];
  __shared__ float scal[6];  // ik, iq, k.q (raw), exp(g), beta
  __shared__ float nrm[4];   // LAYER: partial sums of squares of the output row
  __shared__ uint64_t full;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long key_dim = (long long)p.HK * DN_D;
  const float inv_sqrt_dk = rsqrtf((float)DN_D);
  constexpr uint32_t STATE_BYTES = DN_D * DN_D * 4;

  if (tid == 0) {
    mbar_init(&full, 1);
    fence_barrier_init();
  }
  __syncthreads();
  auto issue_state = [&](int it) {  // thread 0
    const int h = it % p.H, bidx = it / p.H;
    const float* src = p.state_in + bidx * p.state_stride + (long long)h * DN_D * DN_D;
    mbar_arrive_expect_tx(&full, STATE_BYTES);
#pragma unroll
    for (int c = 0; c < 4; c++) bulk_load(sstate + c * (DN_D * DN_D / 4), src + c * (DN_D * DN_D / 4), STATE_BYTES / 4, &full);
  };
  struct Small {
    float x;       // q (tid < 128) or k (tid >= 128) element (LAYER: pre-conv)
    float v;       // v element (tid < 128) (LAYER: pre-conv)
    float ga, gb;  // thread 0: a, b (fused) or g, beta
    // LAYER: conv taps and state of the two channels, and the gate element
    float wx[LAYER ? LAYER_K : 1], wv[LAYER ? LAYER_K : 1];
    float cx[LAYER ? LAYER_K - 1 : 1], cv[LAYER ? LAYER_K - 1 : 1];
    float z;
  };
  const long long conv_c = 2 * key_dim + (long long)p.H * DN_D;  // channels of the conv
  auto load_small = [&](int it, Small& I) {
    const int h = it % p.H, bidx = it / p.H, hk = h % p.HK;
    const float* row = p.qkv + bidx * p.qkv_stride;
    const long long chx = tid < DN_D ? (long long)hk * DN_D + tid : key_dim + (long long)hk * DN_D + (tid - DN_D);
    const long long chv = 2 * key_dim + (long long)h * DN_D + (tid & (DN_D - 1));
    I.x = __ldg(row + chx);
    I.v = tid < DN_D ? __ldg(row + chv) : 0.f;
    if constexpr (LAYER) {
#pragma unroll
      for (int j = 0; j < LAYER_K; j++) {
        I.wx[j] = __ldg(p.conv_w + chx * LAYER_K + j);
        I.wv[j] = tid < DN_D ? __ldg(p.conv_w + chv * LAYER_K + j) : 0.f;
      }
      const float* cs = p.conv_in + bidx * p.conv_stride;
#pragma unroll
      for (int j = 0; j < LAYER_K - 1; j++) {
        I.cx[j] = p.load_state ? __ldg(cs + j * conv_c + chx) : 0.f;
        I.cv[j] = p.load_state && tid < DN_D ? __ldg(cs + j * conv_c + chv) : 0.f;
      }
      I.z = tid < DN_D ? __ldg(p.z + bidx * p.z_stride + (long long)h * DN_D + tid) : 0.f;
    }
    I.ga = I.gb = 0.f;
    if (tid == 0) {
      if constexpr (FUSED) {
        const long long i = bidx * p.ab_stride + h;
        I.ga = __ldg(p.a + i);
        I.gb = __ldg(p.b + i);
      } else {
        const float* g = p.gbeta + bidx * p.gbeta_stride;
        I.ga = __ldg(g + h);
        I.gb = __ldg(g + p.H + h);
      }
    }
  };

  Small cur, nxt;
  int it = blockIdx.x;
  if (it < n_items) {
    if (tid == 0 && p.load_state) issue_state(it);
    load_small(it, cur);
  }
  for (int k = 0; it < n_items; it += gridDim.x, k++) {
    const int itn = it + gridDim.x;
    const int h = it % p.H, bidx = it / p.H;
    float4 st[16];  // rows [16w, 16w+16), cols [4l, 4l+4)
    if (p.load_state) {
      if (!mbar_wait(&full, k & 1, p.status)) {
        // a bulk copy that never landed (the status word now says so): go on
        // with a zero state rather than read a half-written buffer
#pragma unroll
        for (int i = 0; i < 16; i++) st[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      } else {
#pragma unroll
        for (int i = 0; i < 16; i++)
          st[i] = *reinterpret_cast<const float4*>(sstate + (warp * 16 + i) * DN_D + lane * 4);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 16; i++) st[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float xval = cur.x, vval = cur.v;
    if constexpr (LAYER) {
      // conv1d_causal for this token: ext rows 0..K-2 = conv state, row K-1 = x
      float ax = 0.f, av = 0.f;
#pragma unroll
      for (int j = 0; j < LAYER_K - 1; j++) {
        ax = fmaf(cur.wx[j], cur.cx[j], ax);
        av = fmaf(cur.wv[j], cur.cv[j], av);
      }
      ax = fmaf(cur.wx[LAYER_K - 1], cur.x, ax);
      av = fmaf(cur.wv[LAYER_K - 1], cur.v, av);
      xval = ax / (1.f + expf(-ax));
      vval = av / (1.f + expf(-av));
      // new conv state: rows shift up by one, the token's mix becomes row K-2
      const int hk = h % p.HK;
      float* cs = p.conv_out + bidx * p.conv_stride;
      const long long chx = tid < DN_D ? (long long)hk * DN_D + tid : key_dim + (long long)hk * DN_D + (tid - DN_D);
      const long long chv = 2 * key_dim + (long long)h * DN_D + tid;
      if (h == hk) {
#pragma unroll
        for (int j = 0; j < LAYER_K - 1; j++) cs[j * conv_c + chx] = j + 1 < LAYER_K - 1 ? cur.cx[j + 1] : cur.x;
      }
      if (tid < DN_D) {
#pragma unroll
        for (int j = 0; j < LAYER_K - 1; j++) cs[j * conv_c + chv] = j + 1 < LAYER_K - 1 ? cur.cv[j + 1] : cur.v;
      }
    }
    if (tid < DN_D) qs[tid] = xval; else ks[tid - DN_D] = xval;
    if (tid == 0) {
      float g = cur.ga, beta = cur.gb;
      if constexpr (FUSED) gbeta_f64(cur.ga, p.dt_bias[h], p.a_neg[h], cur.gb, &g, &beta);
      scal[3] = expf(g);
      scal[4] = beta;
    }
    __syncthreads();  // the state buffer is read: the next item's copy may start
    if (itn < n_items) {
      if (tid == 0 && p.load_state) issue_state(itn);
      load_small(itn, nxt);
    }
    if (warp < 3) {
      float v = 0.f;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const float x = warp == 0 ? qs[lane * 4 + i] : ks[lane * 4 + i];
        const float y = warp == 2 ? qs[lane * 4 + i] : x;
        v = fmaf(x, y, v);
      }
      v = warp_sum(v);
      if (lane == 0) {
        if (warp == 0) scal[1] = rsqrtf(v + 1e-6f) * inv_sqrt_dk;
        if (warp == 1) scal[0] = rsqrtf(v + 1e-6f);
        if (warp == 2) scal[2] = v;
      }
    }
    __syncthreads();
    const float ik = scal[0], iq = scal[1], gt = scal[3], bt = scal[4];
    const float kq = scal[2] * ik * iq;  // k^ . q^
    float orow = 0.f;                    // output element of thread tid < 128
    float4 pk = make_float4(0.f, 0.f, 0.f, 0.f), pq = pk;
#pragma unroll
    for (int i = 0; i < 16; i++) {
      const float kh = ks[warp * 16 + i] * ik;
      const float qh = qs[warp * 16 + i] * iq;
      st[i].x *= gt;
      st[i].y *= gt;
      st[i].z *= gt;
      st[i].w *= gt;
      pk.x = fmaf(st[i].x, kh, pk.x);
      pk.y = fmaf(st[i].y, kh, pk.y);
      pk.z = fmaf(st[i].z, kh, pk.z);
      pk.w = fmaf(st[i].w, kh, pk.w);
      pq.x = fmaf(st[i].x, qh, pq.x);
      pq.y = fmaf(st[i].y, qh, pq.y);
      pq.z = fmaf(st[i].z, qh, pq.z);
      pq.w = fmaf(st[i].w, qh, pq.w);
    }
    *reinterpret_cast<float4*>(&red_k[warp][lane * 4]) = pk;
    *reinterpret_cast<float4*>(&red_q[warp][lane * 4]) = pq;
    __syncthreads();
    if (tid < DN_D) {
      float kvd = 0.f, qd = 0.f;
#pragma unroll
      for (int w = 0; w < 8; w++) {
        kvd += red_k[w][tid];
        qd += red_q[w][tid];
      }
      const float delta = (vval - kvd) * bt;
      sdelta[tid] = delta;
      orow = fmaf(delta, kq, qd);
      if constexpr (LAYER) {
        const float sq = warp_sum(orow * orow);
        if (lane == 0) nrm[warp] = sq;
      } else {
        p.core[bidx * p.core_stride + (long long)h * DN_D + tid] = orow;
      }
    }
    __syncthreads();
    if constexpr (LAYER) {
      // deltanet_norm_gate: y = gamma * o / sqrt(mean(o^2) + eps) * silu(z)
      if (tid < DN_D) {
        const float inv = rsqrtf(((nrm[0] + nrm[1]) + (nrm[2] + nrm[3])) * (1.f / DN_D) + p.eps);
        const float zz = cur.z;
        p.out[bidx * p.out_stride + (long long)h * DN_D + tid] =
            __ldg(p.gamma + tid) * (orow * inv) * (zz / (1.f + expf(-zz)));
      }
    }
    const float4 d4 = *reinterpret_cast<const float4*>(&sdelta[lane * 4]);
    float4* dst = reinterpret_cast<float4*>(p.state_out + bidx * p.state_stride + (long long)h * DN_D * DN_D);
#pragma unroll
    for (int i = 0; i < 16; i++) {
      const float kh = ks[warp * 16 + i] * ik;
      st[i].x = fmaf(kh, d4.x, st[i].x);
      st[i].y = fmaf(kh, d4.y, st[i].y);
      st[i].z = fmaf(kh, d4.z, st[i].z);
      st[i].w = fmaf(kh, d4.w, st[i].w);
      __stcs(dst + (warp * 16 + i) * (DN_D / 4) + lane, st[i]);
    }
    __syncthreads();  // qs / ks / scal / sdelta are rewritten by the next item
    cur = nxt;
  }
}

int launch_dn(hcu_context* h, const hcu_deltanet_params* p, DnArgs a, bool fused) {
  const int batch = p->batch ? (int)p->batch : 1;
  a.status = h->dev_status;
  if (p->S == 1) {
    const long long n = (long long)batch * p->H;
    if (n > 0x7fffffffLL) return fail(HCU_EINVAL, "deltanet: batch x H too large");
    const int grid = (int)(n < 2LL * h->sm_count ? n : 2LL * h->sm_count);  // two CTAs per SM
    constexpr int smem = DN_D * DN_D * 4;
    static std::atomic<uint64_t> attr_done{0};  // per device
    HCU_TRY(once_per_device(attr_done, h->device, [&]() -> int {
      HCU_TRY(check_cuda(cudaFuncSetAttribute(deltanet_step_kernel<true, false>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                         "deltanet: smem attribute"));
      HCU_TRY(check_cuda(cudaFuncSetAttribute(deltanet_step_kernel<false, false>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                         "deltanet: smem attribute"));
      return HCU_OK;
    }));
    if (fused)
      deltanet_step_kernel<true, false><<<grid, DN_THREADS, smem, h->stream>>>(a, (int)n);
    else
      deltanet_step_kernel<false, false><<<grid, DN_THREADS, smem, h->stream>>>(a, (int)n);
  } else if (fused) {
    deltanet_recur_kernel<true><<<dim3(p->H, batch), DN_THREADS, 0, h->stream>>>(a);
  } else {
    deltanet_recur_kernel<false><<<dim3(p->H, batch), DN_THREADS, 0, h->stream>>>(a);
  }
  return HCU_OK;
}

// conv1d_causal (src/kernels.ts:1431-1466; JS src/wasm-backend.ts:1003-1031):
// y[t][c] = silu(sum_j w[c][j] * ext(t + j, c)) with ext rows 0..K-2 the conv
// state (zeros when !loadState) followed by the S input rows.  One thread per
// (sequence, token, channel); f32 arithmetic like the WGSL.
struct ConvArgs {
  const float* x;
  const float* w;
  const float* state_in;
  float* y;
  float* state_out;
  int S, C, K, load_state;
  long long x_stride, y_stride, state_stride;
};

__device__ __forceinline__ float conv_ext(const ConvArgs& a, int b, int m, int c) {
  if (m + 1 < a.K) return a.load_state ? a.state_in[b * a.state_stride + (long long)m * a.C + c] : 0.f;
  return a.x[b * a.x_stride + (long long)(m - (a.K - 1)) * a.C + c];
}

__global__ void __launch_bounds__(256) conv1d_kernel(const ConvArgs a) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long n = (long long)a.S * a.C;
  if (i >= n) return;
  const int b = blockIdx.y;
  const int c = (int)(i % a.C), t = (int)(i / a.C);
  float acc = 0.f;
  for (int j = 0; j < a.K; j++) acc = fmaf(__ldg(a.w + (long long)c * a.K + j), conv_ext(a, b, t + j, c), acc);
  a.y[b * a.y_stride + i] = acc / (1.f + expf(-acc));
}

// The new conv state: the last K-1 rows of the extended sequence.  One thread
// per (sequence, channel) reads all of them before writing any, so the state
// may be updated in place (the output kernel, launched first on the same
// stream, has finished reading the old rows).
constexpr int CONV_KMAX = 8;
__global__ void __launch_bounds__(256) conv1d_state_kernel(const ConvArgs a) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= a.C) return;
  const int b = blockIdx.y;
  float v[CONV_KMAX - 1];
#pragma unroll
  for (int sk = 0; sk < CONV_KMAX - 1; sk++)
    if (sk < a.K - 1) v[sk] = conv_ext(a, b, a.S + sk, c);
#pragma unroll
  for (int sk = 0; sk < CONV_KMAX - 1; sk++)
    if (sk < a.K - 1) a.state_out[b * a.state_stride + (long long)sk * a.C + c] = v[sk];
}

// deltanet_norm_gate (src/kernels.ts:1578-1611; JS src/wasm-backend.ts:
// 1104-1117): per row, y = gamma * core / sqrt(mean(core^2) + eps) * silu(z).
// One warp per row.
__global__ void __launch_bounds__(256) norm_gate_kernel(const float* __restrict__ core, const float* __restrict__ z,
                                                        const float* __restrict__ gamma, float* __restrict__ y,
                                                        int rows, int DV, float eps) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long r = (long long)blockIdx.x * 8 + warp;
  if (r >= rows) return;
  const float* c = core + r * DV;
  float s = 0.f;
  for (int i = lane; i < DV; i += 32) {
    const float v = c[i];
    s = fmaf(v, v, s);
  }
  s = warp_sum(s);
  const float inv = rsqrtf(s / (float)DV + eps);
  for (int i = lane; i < DV; i += 32) {
    const float zz = z[r * DV + i];
    y[r * DV + i] = __ldg(gamma + i) * (c[i] * inv) * (zz / (1.f + expf(-zz)));
  }
}

int check_dn(const hcu_deltanet_params* p, const char* op) {
  if (!p) return fail(HCU_EINVAL, "%s: null params", op);
  if (p->S < 1 || p->H < 1 || p->HK < 1) return fail(HCU_EINVAL, "%s: S, H and HK must be positive", op);
  if (p->DK != DN_D || p->DV != DN_D)
    return fail(HCU_EUNSUPPORTED, "%s: DK=%u DV=%u (built: %d)", op, p->DK, p->DV, DN_D);
  const int batch = p->batch ? (int)p->batch : 1;
  if (batch > 65535 || p->H > 0x7fffffffu) return fail(HCU_EINVAL, "%s: batch or H too large", op);
  return HCU_OK;
}

void fill_strides(const hcu_deltanet_params* p, DnArgs& a) {
  const long long conv_dim = 2LL * p->HK * DN_D + (long long)p->H * DN_D;
  a.qkv_stride = p->qkv_seq_stride ? (long long)p->qkv_seq_stride : (long long)p->S * conv_dim;
  a.gbeta_stride = p->gbeta_seq_stride ? (long long)p->gbeta_seq_stride : 2LL * p->S * p->H;
  a.ab_stride = (long long)p->S * p->H;
  a.state_stride = p->state_seq_stride ? (long long)p->state_seq_stride : (long long)p->H * DN_D * DN_D;
  a.core_stride = p->core_seq_stride ? (long long)p->core_seq_stride : (long long)p->S * p->H * DN_D;
  a.S = (int)p->S;
  a.H = (int)p->H;
  a.HK = (int)p->HK;
  a.load_state = p->loadState ? 1 : 0;
}

int check_align(const void* ptr, const char* what, const char* op) {
  if (reinterpret_cast<uintptr_t>(ptr) % 16) return fail(HCU_EINVAL, "%s: %s must be 16-byte aligned", op, what);
  return HCU_OK;
}

}  // namespace

extern "C" int hcu_deltanet_gbeta(hcu_handle h, uint32_t S, uint32_t H, const float* a, const float* b,
                                  const float* a_neg, const float* dt_bias, float* out) {
  HCU_TRY(hcu::begin_op(h, "hcu_deltanet_gbeta"));
  if (!a || !b || !a_neg || !dt_bias || !out) return fail(HCU_EINVAL, "hcu_deltanet_gbeta: null buffer");
  const long long n = (long long)S * H;
  if (n <= 0 || n > 0x3fffffffLL) return fail(HCU_EINVAL, "hcu_deltanet_gbeta: bad size S*H=%lld", n);
  gbeta_kernel<<<(unsigned)((n + 255) / 256), 256, 0, h->stream>>>(a, b, a_neg, dt_bias, out, (int)n, (int)H);
  return hcu::after_launch("hcu_deltanet_gbeta");
}

extern "C" int hcu_deltanet_recur(hcu_handle h, const hcu_deltanet_params* p, const float* qkv_conv,
                                  const float* gbeta, const float* state_in, float* core, float* state_out) {
  HCU_TRY(hcu::begin_op(h, "hcu_deltanet_recur"));
  HCU_TRY(check_dn(p, "hcu_deltanet_recur"));
  if (!qkv_conv || !gbeta || !core || !state_out || (p->loadState && !state_in))
    return fail(HCU_EINVAL, "hcu_deltanet_recur: null buffer");
  HCU_TRY(check_align(state_out, "stateOut", "hcu_deltanet_recur"));
  if (p->loadState) HCU_TRY(check_align(state_in, "stateIn", "hcu_deltanet_recur"));
  DnArgs a{};
  fill_strides(p, a);
  a.qkv = qkv_conv;
  a.gbeta = gbeta;
  a.state_in = state_in;
  a.state_out = state_out;
  a.core = core;
  HCU_TRY(launch_dn(h, p, a, false));
  return hcu::after_launch("hcu_deltanet_recur");
}

extern "C" int hcu_deltanet_decode(hcu_handle h, const hcu_deltanet_params* p, const float* qkv_conv, const float* a,
                                   const float* b, const float* a_neg, const float* dt_bias, const float* state_in,
                                   float* core, float* state_out) {
  HCU_TRY(hcu::begin_op(h, "hcu_deltanet_decode"));
  HCU_TRY(check_dn(p, "hcu_deltanet_decode"));
  if (!qkv_conv || !a || !b || !a_neg || !dt_bias || !core || !state_out || (p->loadState && !state_in))
    return fail(HCU_EINVAL, "hcu_deltanet_decode: null buffer");
  HCU_TRY(check_align(state_out, "stateOut", "hcu_deltanet_decode"));
  if (p->loadState) HCU_TRY(check_align(state_in, "stateIn", "hcu_deltanet_decode"));
  DnArgs args{};
  fill_strides(p, args);
  args.qkv = qkv_conv;
  args.a = a;
  args.b = b;
  args.a_neg = a_neg;
  args.dt_bias = dt_bias;
  args.state_in = state_in;
  args.state_out = state_out;
  args.core = core;
  HCU_TRY(launch_dn(h, p, args, true));
  return hcu::after_launch("hcu_deltanet_decode");
}

extern "C" int hcu_conv1d_causal(hcu_handle h, const hcu_conv1d_params* p, const float* x, const float* w,
                                 const float* state_in, float* y, float* state_out) {
  HCU_TRY(hcu::begin_op(h, "hcu_conv1d_causal"));
  if (!p || !x || !w || !y || !state_out || (p->loadState && !state_in))
    return fail(HCU_EINVAL, "hcu_conv1d_causal: null argument");
  if (p->S < 1 || p->C < 1 || p->K < 1 || p->K > (uint32_t)CONV_KMAX)
    return fail(HCU_EINVAL, "hcu_conv1d_causal: need S, C >= 1 and 1 <= K <= %d", CONV_KMAX);
  const int batch = p->batch ? (int)p->batch : 1;
  if (batch > 65535) return fail(HCU_EINVAL, "hcu_conv1d_causal: batch > 65535");
  const long long n = (long long)p->S * p->C;
  if (n > 0x3fffffffLL) return fail(HCU_EINVAL, "hcu_conv1d_causal: S x C too large");
  ConvArgs a{};
  a.x = x;
  a.w = w;
  a.state_in = state_in;
  a.y = y;
  a.state_out = state_out;
  a.S = (int)p->S;
  a.C = (int)p->C;
  a.K = (int)p->K;
  a.load_state = p->loadState ? 1 : 0;
  a.x_stride = p->x_seq_stride ? (long long)p->x_seq_stride : n;
  a.y_stride = p->y_seq_stride ? (long long)p->y_seq_stride : n;
  a.state_stride = p->state_seq_stride ? (long long)p->state_seq_stride : (long long)(p->K - 1) * p->C;
  conv1d_kernel<<<dim3((unsigned)((n + 255) / 256), (unsigned)batch), 256, 0, h->stream>>>(a);
  HCU_TRY(hcu::after_launch("hcu_conv1d_causal"));
  if (p->K > 1) {
    conv1d_state_kernel<<<dim3((unsigned)((p->C + 255) / 256), (unsigned)batch), 256, 0, h->stream>>>(a);
    HCU_TRY(hcu::after_launch("hcu_conv1d_causal: state"));
  }
  return HCU_OK;
}

extern "C" int hcu_deltanet_norm_gate(hcu_handle h, uint32_t rows, uint32_t DV, float eps, const float* core,
                                      const float* z, const float* gamma, float* y) {
  HCU_TRY(hcu::begin_op(h, "hcu_deltanet_norm_gate"));
  if (!core || !z || !gamma || !y) return fail(HCU_EINVAL, "hcu_deltanet_norm_gate: null buffer");
  if (rows < 1 || DV < 1 || rows > 0x3fffffffu) return fail(HCU_EINVAL, "hcu_deltanet_norm_gate: bad rows / DV");
  norm_gate_kernel<<<(rows + 7) / 8, 256, 0, h->stream>>>(core, z, gamma, y, (int)rows, (int)DV, eps);
  return hcu::after_launch("hcu_deltanet_norm_gate");
}

extern "C" int hcu_gdn_layer_step(hcu_handle h, const hcu_gdn_step_params* p, const float* qkv_mixed,
                                  const float* conv_w, const float* conv_state_in, float* conv_state_out,
                                  const float* a, const float* b, const float* a_neg, const float* dt_bias,
                                  const float* z, const float* gamma, const float* state_in, float* state_out,
                                  float* out) {
  HCU_TRY(hcu::begin_op(h, "hcu_gdn_layer_step"));
  if (!p || !qkv_mixed || !conv_w || !conv_state_out || !a || !b || !a_neg || !dt_bias || !z || !gamma ||
      !state_out || !out || (p->loadState && (!state_in || !conv_state_in)))
    return fail(HCU_EINVAL, "hcu_gdn_layer_step: null buffer");
  if (p->DK != DN_D || p->DV != DN_D)
    return fail(HCU_EUNSUPPORTED, "hcu_gdn_layer_step: DK=%u DV=%u (built: %d)", p->DK, p->DV, DN_D);
  if (p->K != (uint32_t)LAYER_K) return fail(HCU_EUNSUPPORTED, "hcu_gdn_layer_step: K=%u (built: %d)", p->K, LAYER_K);
  if (p->H < 1 || p->HK < 1 || p->H < p->HK)
    return fail(HCU_EINVAL, "hcu_gdn_layer_step: need H >= HK >= 1 (every QK head's conv state has a writer)");
  if (p->loadState && conv_state_in == conv_state_out)
    return fail(HCU_EINVAL, "hcu_gdn_layer_step: conv state in and out must be different buffers (ping-pong)");
  const int batch = p->batch ? (int)p->batch : 1;
  if (batch > 65535) return fail(HCU_EINVAL, "hcu_gdn_layer_step: batch > 65535");
  HCU_TRY(check_align(state_out, "stateOut", "hcu_gdn_layer_step"));
  if (p->loadState) HCU_TRY(check_align(state_in, "stateIn", "hcu_gdn_layer_step"));
  const long long C = 2LL * p->HK * DN_D + (long long)p->H * DN_D;
  DnArgs args{};
  args.qkv = qkv_mixed;
  args.a = a;
  args.b = b;
  args.a_neg = a_neg;
  args.dt_bias = dt_bias;
  args.state_in = state_in;
  args.state_out = state_out;
  args.S = 1;
  args.H = (int)p->H;
  args.HK = (int)p->HK;
  args.load_state = p->loadState ? 1 : 0;
  args.qkv_stride = p->qkv_seq_stride ? (long long)p->qkv_seq_stride : C;
  args.ab_stride = p->ab_seq_stride ? (long long)p->ab_seq_stride : p->H;
  args.state_stride = p->state_seq_stride ? (long long)p->state_seq_stride : (long long)p->H * DN_D * DN_D;
  args.conv_w = conv_w;
  args.conv_in = conv_state_in;
  args.conv_out = conv_state_out;
  args.conv_stride = p->conv_seq_stride ? (long long)p->conv_seq_stride : (LAYER_K - 1) * C;
  args.z = z;
  args.z_stride = p->z_seq_stride ? (long long)p->z_seq_stride : (long long)p->H * DN_D;
  args.gamma = gamma;
  args.out = out;
  args.out_stride = p->out_seq_stride ? (long long)p->out_seq_stride : (long long)p->H * DN_D;
  args.eps = p->eps;
  args.status = h->dev_status;
  const long long n = (long long)batch * p->H;
  const int grid = (int)(n < 2LL * h->sm_count ? n : 2LL * h->sm_count);
  constexpr int smem = DN_D * DN_D * 4;
  static std::atomic<uint64_t> attr_done{0};  // per device
  HCU_TRY(hcu::once_per_device(attr_done, h->device, [&]() -> int {
    HCU_TRY(hcu::check_cuda(cudaFuncSetAttribute(deltanet_step_kernel<true, true>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                            "hcu_gdn_layer_step: smem attribute"));
    return HCU_OK;
  }));
  deltanet_step_kernel<true, true><<<grid, DN_THREADS, smem, h->stream>>>(args, (int)n);
  return hcu::after_launch("hcu_gdn_layer_step");
}
