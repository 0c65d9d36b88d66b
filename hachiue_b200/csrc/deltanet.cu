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
};

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
template <bool FUSED>
__global__ void __launch_bounds__(DN_THREADS, 2) deltanet_step_kernel(const DnArgs p, int n_items) {
  extern __shared__ __align__(16) float sstate[];  // [128][128] f32: the next item's state
  __shared__ float qs[DN_D], ks[DN_D];
  __shared__ float red_k[8][DN_D], red_q[8][DN_D];
  __shared__ float sdelta[DN_D];
  __shared__ float scal[6];  // ik, iq, k.q (raw), exp(g), beta
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
    float x;       // q (tid < 128) or k (tid >= 128) element
    float v;       // v element (tid < 128)
    float ga, gb;  // thread 0: a, b (fused) or g, beta
  };
  auto load_small = [&](int it, Small& I) {
    const int h = it % p.H, bidx = it / p.H, hk = h % p.HK;
    const float* row = p.qkv + bidx * p.qkv_stride;
    I.x = tid < DN_D ? __ldg(row + (long long)hk * DN_D + tid)
                     : __ldg(row + key_dim + (long long)hk * DN_D + (tid - DN_D));
    I.v = tid < DN_D ? __ldg(row + 2 * key_dim + (long long)h * DN_D + tid) : 0.f;
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
    if (tid < DN_D) qs[tid] = cur.x; else ks[tid - DN_D] = cur.x;
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
      const float delta = (cur.v - kvd) * bt;
      sdelta[tid] = delta;
      p.core[bidx * p.core_stride + (long long)h * DN_D + tid] = fmaf(delta, kq, qd);
    }
    __syncthreads();
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
    static bool attr_done = false;
    if (!attr_done) {
      HCU_TRY(check_cuda(cudaFuncSetAttribute(deltanet_step_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              smem), "deltanet: smem attribute"));
      HCU_TRY(check_cuda(cudaFuncSetAttribute(deltanet_step_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              smem), "deltanet: smem attribute"));
      attr_done = true;
    }
    if (fused)
      deltanet_step_kernel<true><<<grid, DN_THREADS, smem, h->stream>>>(a, (int)n);
    else
      deltanet_step_kernel<false><<<grid, DN_THREADS, smem, h->stream>>>(a, (int)n);
  } else if (fused) {
    deltanet_recur_kernel<true><<<dim3(p->H, batch), DN_THREADS, 0, h->stream>>>(a);
  } else {
    deltanet_recur_kernel<false><<<dim3(p->H, batch), DN_THREADS, 0, h->stream>>>(a);
  }
  return HCU_OK;
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
