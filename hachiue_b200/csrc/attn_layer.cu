// attn_layer.cu - the full-attention layer's neighbours of the KV append and
// the attention kernel (qwen3 / qwen35 full-attention layers,
// src/engine.ts:1408-1458; JS src/wasm-backend.ts:1125-1157): split_q_gate,
// the per-head q / k RMSNorm, RoPE, and (in attention_decode*.cu) the qwen35
// sigmoid gate on the attention output.
//
// The standalone ops keep the reference's names and arithmetic: f64 like the
// JS backend, rounded to f32 where the JS stores into a Float32Array, with no
// fused multiply-adds where the JS has none.  hcu_attn_prologue fuses split +
// norms + RoPE + the K / V append for a batch of sequences: one warp per
// (token, head) row, lane l holding elements l, l + 32, ...  A Q8_0 block of 32
// is then one register across the warp, quantised exactly as
// kv_append_q8_kernel does, so the appended cache is bit-identical to the
// reference's appendKvQ8 of the same normed and rotated rows.
#include "common.cuh"
#include "context.h"

namespace {

using namespace hcu;

__device__ __forceinline__ double js_round_d(double x) {
  const double f = floor(x);
  return (x - f >= 0.5) ? f + 1.0 : f;
}

// ---- standalone ops -------------------------------------------------------
// rmsnorm (src/kernels.ts:324-355, JS src/wasm-backend.ts:427-444): one block per row.
__global__ void __launch_bounds__(256) rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                                                      float* __restrict__ y, int dim, double eps, int unit) {
  __shared__ double red[8];
  const long long base = (long long)blockIdx.x * dim;
  double s = 0.0;
  for (int i = threadIdx.x; i < dim; i += 256) {
    const double v = x[base + i];
    s = __dadd_rn(s, __dmul_rn(v, v));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  double t = 0.0;
#pragma unroll
  for (int w = 0; w < 8; w++) t += red[w];
  const double inv = 1.0 / sqrt(t / dim + eps);
  for (int i = threadIdx.x; i < dim; i += 256) {
    const double g = unit ? 1.0 + (double)gamma[i] : (double)gamma[i];
    y[base + i] = (float)__dmul_rn(__dmul_rn((double)x[base + i], inv), g);
  }
}

// rope (src/kernels.ts:1120-1150, JS src/wasm-backend.ts:767-791): one thread per pair.
__global__ void __launch_bounds__(256) rope_kernel(float* __restrict__ x, const float* __restrict__ cos_tab,
                                                   const float* __restrict__ sin_tab, long long pairs, int heads,
                                                   int head_dim, int half, int pos_base) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= pairs) return;
  const int pair = (int)(i % half);
  const long long sh = i / half;  // s * heads + h
  const int s = (int)(sh / heads);
  const long long cs = (long long)(pos_base + s) * half + pair;
  const double c = cos_tab[cs], sn = sin_tab[cs];
  const long long base = sh * head_dim;
  const double v0 = x[base + pair], v1 = x[base + pair + half];
  x[base + pair] = (float)__dsub_rn(__dmul_rn(v0, c), __dmul_rn(v1, sn));
  x[base + pair + half] = (float)__dadd_rn(__dmul_rn(v1, c), __dmul_rn(v0, sn));
}

// split_q_gate (src/kernels.ts:1155-1176): [S, H, 2 Dh] -> q, gate [S, H, Dh].
__global__ void __launch_bounds__(256) split_q_gate_kernel(const float* __restrict__ qg, float* __restrict__ q,
                                                           float* __restrict__ gate, long long n, int Dh) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const long long sh = i / Dh;
  const int d = (int)(i % Dh);
  q[i] = qg[sh * 2 * Dh + d];
  gate[i] = qg[sh * 2 * Dh + Dh + d];
}

// sigmoid_gate (src/kernels.ts:1249-1262, JS src/wasm-backend.ts:1152-1157): att *= 1 / (1 + exp(-gate)).
__global__ void __launch_bounds__(256) sigmoid_gate_kernel(const float* __restrict__ gate, float* __restrict__ att,
                                                           long long n) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  att[i] = (float)__dmul_rn((double)att[i], 1.0 / (1.0 + exp(-(double)gate[i])));
}

// ---- fused prologue ---------------------------------------------------------
struct ProArgs {
  const float* q;  // [B, S, H, Dh] or, with split, [B, S, H, 2 Dh]
  const float* k;  // [B, S, KV, Dh]
  const float* v;  // [B, S, KV, Dh]
  const float* qn_w;
  const float* kn_w;
  const float* cos_tab;
  const float* sin_tab;
  float* q_out;     // [B, S, H, Dh]
  float* gate_out;  // [B, S, H, Dh] (split only)
  void* kc;
  void* vc;
  float* ks;
  float* vs;
  const int32_t* pos_base;
  const int64_t* row_off;
  long long seq_row_stride;
  double eps;
  int S, H, KV, pos_default, split, fmt;
};

template <typename T>
__device__ __forceinline__ T to_cache(float x);
template <>
__device__ __forceinline__ float to_cache<float>(float x) { return x; }
template <>
__device__ __forceinline__ __half to_cache<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 to_cache<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

template <int NJ, int HJ>  // Dh / 32 elements per lane; rotaryDim / 64 = partner register distance
__global__ void __launch_bounds__(128) attn_prologue_kernel(const ProArgs a) {
  constexpr int Dh = NJ * 32;
  const int s = blockIdx.x, b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pos = (a.pos_base ? a.pos_base[b] : a.pos_default) + s;
  const long long row = (a.row_off ? a.row_off[b] : (long long)b * a.seq_row_stride) + pos;
  const long long tok = (long long)b * a.S + s;
  const int nrows = a.H + 2 * a.KV;
  // one warp per row: the rows' dependent chains (loads, f64 reductions) run side by side
  for (int r = blockIdx.z * 4 + warp; r < nrows; r += 4 * gridDim.z) {
    const int kind = r < a.H ? 0 : (r < a.H + a.KV ? 1 : 2);  // q, k, v
    const int head = kind == 0 ? r : (kind == 1 ? r - a.H : r - a.H - a.KV);
    const float* src = kind == 0 ? a.q + (tok * a.H + head) * (long long)(a.split ? 2 * Dh : Dh)
                                 : (kind == 1 ? a.k : a.v) + (tok * a.KV + head) * (long long)Dh;
    float x[NJ], wv[NJ], cv[HJ], sv[HJ];
#pragma unroll
    for (int j = 0; j < NJ; j++) x[j] = src[lane + 32 * j];
    if (kind < 2) {
      // the norm weights and this position's RoPE row are loaded with the row
      const float* w = kind == 0 ? a.qn_w : a.kn_w;
      const long long cs = (long long)pos * (32 * HJ);
#pragma unroll
      for (int j = 0; j < NJ; j++) wv[j] = w[lane + 32 * j];
#pragma unroll
      for (int j = 0; j < HJ; j++) {
        cv[j] = a.cos_tab[cs + lane + 32 * j];
        sv[j] = a.sin_tab[cs + lane + 32 * j];
      }
      // runRmsNorm: inv = 1 / sqrt(sum x^2 / Dh + eps), y = x * inv * gamma, stored f32
      double sq = 0.0;
#pragma unroll
      for (int j = 0; j < NJ; j++) sq = __dadd_rn(sq, __dmul_rn((double)x[j], (double)x[j]));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
      const double inv = 1.0 / sqrt(sq / Dh + a.eps);
#pragma unroll
      for (int j = 0; j < NJ; j++) x[j] = (float)__dmul_rn(__dmul_rn((double)x[j], inv), (double)wv[j]);
      // applyRope: pairs (e, e + half), half = 32 HJ, sit in one lane (registers j, j + HJ)
#pragma unroll
      for (int j = 0; j < HJ; j++) {
        const double c = cv[j], sn = sv[j];
        const double v0 = x[j], v1 = x[j + HJ];
        x[j] = (float)__dsub_rn(__dmul_rn(v0, c), __dmul_rn(v1, sn));
        x[j + HJ] = (float)__dadd_rn(__dmul_rn(v1, c), __dmul_rn(v0, sn));
      }
    }
    if (kind == 0) {
      float* dst = a.q_out + (tok * a.H + head) * Dh;
#pragma unroll
      for (int j = 0; j < NJ; j++) dst[lane + 32 * j] = x[j];
      if (a.split) {
        float* gd = a.gate_out + (tok * a.H + head) * Dh;
#pragma unroll
        for (int j = 0; j < NJ; j++) gd[lane + 32 * j] = src[Dh + lane + 32 * j];
      }
      continue;
    }
    // append the row to the cache at (row, head)
    const long long elem0 = (row * a.KV + head) * Dh;
    void* cache = kind == 1 ? a.kc : a.vc;
    if (a.fmt == HCU_KV_Q8_0_WGSL) {
      float* scl = kind == 1 ? a.ks : a.vs;
#pragma unroll
      for (int j = 0; j < NJ; j++) {
        float amax = fabsf(x[j]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        static_cast<int8_t*>(cache)[elem0 + lane + 32 * j] = (int8_t)q8_quant_wgsl(x[j], amax);
        if (lane == 0) scl[elem0 / 32 + j] = q8_scale_wgsl(amax);
      }
    } else if (a.fmt == HCU_KV_Q8_0) {
      float* scl = kind == 1 ? a.ks : a.vs;
#pragma unroll
      for (int j = 0; j < NJ; j++) {  // block j = elements 32j .. 32j + 31, element lane
        float amax = fabsf(x[j]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const double damax = (double)amax;
        const double qinv = damax > 0 ? 127.0 / damax : 0.0;
        double qd = js_round_d((double)x[j] * qinv);
        qd = qd < -127.0 ? -127.0 : (qd > 127.0 ? 127.0 : qd);
        static_cast<int8_t*>(cache)[elem0 + lane + 32 * j] = (int8_t)(int)qd;
        if (lane == 0) scl[elem0 / 32 + j] = (float)(damax / 127.0);
      }
    } else if (a.fmt == HCU_KV_F32) {
#pragma unroll
      for (int j = 0; j < NJ; j++) static_cast<float*>(cache)[elem0 + lane + 32 * j] = x[j];
    } else if (a.fmt == HCU_KV_F16) {
#pragma unroll
      for (int j = 0; j < NJ; j++) static_cast<__half*>(cache)[elem0 + lane + 32 * j] = to_cache<__half>(x[j]);
    } else {
#pragma unroll
      for (int j = 0; j < NJ; j++)
        static_cast<__nv_bfloat16*>(cache)[elem0 + lane + 32 * j] = to_cache<__nv_bfloat16>(x[j]);
    }
  }
}

unsigned blocks_for(long long n) { return (unsigned)((n + 255) / 256); }

}  // namespace

using hcu::fail;

extern "C" int hcu_rmsnorm(hcu_handle h, uint32_t rows, uint32_t dim, float eps, uint32_t add_unit_offset,
                           const float* x, const float* gamma, float* y) {
  HCU_TRY(hcu::begin_op(h, "hcu_rmsnorm"));
  if (!x || !gamma || !y) return fail(HCU_EINVAL, "hcu_rmsnorm: null buffer");
  if (rows < 1 || dim < 1 || rows > 0x7fffffffu) return fail(HCU_EINVAL, "hcu_rmsnorm: bad rows / dim");
  rmsnorm_kernel<<<rows, 256, 0, h->stream>>>(x, gamma, y, (int)dim, (double)eps, add_unit_offset ? 1 : 0);
  return hcu::after_launch("hcu_rmsnorm");
}

extern "C" int hcu_rope(hcu_handle h, uint32_t S, uint32_t heads, uint32_t head_dim, uint32_t rotary_dim,
                        uint32_t posBase, const float* cos_tab, const float* sin_tab, float* x) {
  HCU_TRY(hcu::begin_op(h, "hcu_rope"));
  if (!cos_tab || !sin_tab || !x) return fail(HCU_EINVAL, "hcu_rope: null buffer");
  if (rotary_dim < 2 || rotary_dim % 2 || rotary_dim > head_dim)
    return fail(HCU_EINVAL, "hcu_rope: rotary_dim %u must be even and <= head_dim %u", rotary_dim, head_dim);
  const long long pairs = (long long)S * heads * (rotary_dim / 2);
  if (pairs < 1 || pairs > 0x3fffffffLL) return fail(HCU_EINVAL, "hcu_rope: bad size");
  rope_kernel<<<blocks_for(pairs), 256, 0, h->stream>>>(x, cos_tab, sin_tab, pairs, (int)heads, (int)head_dim,
                                                         (int)(rotary_dim / 2), (int)posBase);
  return hcu::after_launch("hcu_rope");
}

extern "C" int hcu_split_q_gate(hcu_handle h, uint32_t S, uint32_t H, uint32_t Dh, const float* qg, float* q,
                                float* gate) {
  HCU_TRY(hcu::begin_op(h, "hcu_split_q_gate"));
  if (!qg || !q || !gate) return fail(HCU_EINVAL, "hcu_split_q_gate: null buffer");
  const long long n = (long long)S * H * Dh;
  if (n < 1 || n > 0x3fffffffLL) return fail(HCU_EINVAL, "hcu_split_q_gate: bad size");
  split_q_gate_kernel<<<blocks_for(n), 256, 0, h->stream>>>(qg, q, gate, n, (int)Dh);
  return hcu::after_launch("hcu_split_q_gate");
}

extern "C" int hcu_sigmoid_gate(hcu_handle h, uint64_t n, const float* gate, float* att) {
  HCU_TRY(hcu::begin_op(h, "hcu_sigmoid_gate"));
  if (!gate || !att) return fail(HCU_EINVAL, "hcu_sigmoid_gate: null buffer");
  if (n < 1 || n > 0x3fffffffULL) return fail(HCU_EINVAL, "hcu_sigmoid_gate: bad size");
  sigmoid_gate_kernel<<<blocks_for((long long)n), 256, 0, h->stream>>>(gate, att, (long long)n);
  return hcu::after_launch("hcu_sigmoid_gate");
}

extern "C" int hcu_attn_prologue(hcu_handle h, const hcu_attn_prologue_params* p, const float* q, const float* k,
                                 const float* v, const float* q_norm, const float* k_norm, const float* cos_tab,
                                 const float* sin_tab, float* q_out, float* gate_out, const hcu_kv_cache* kv) {
  HCU_TRY(hcu::begin_op(h, "hcu_attn_prologue"));
  if (!p || !q || !k || !v || !q_norm || !k_norm || !cos_tab || !sin_tab || !q_out || !kv || !kv->k || !kv->v ||
      (p->split_gate && !gate_out))
    return fail(HCU_EINVAL, "hcu_attn_prologue: null argument");
  const int Dh = (int)p->Dh;
  if (Dh != 128 && Dh != 256) return fail(HCU_EUNSUPPORTED, "hcu_attn_prologue: Dh=%d (built: 128, 256)", Dh);
  if (p->rotaryDim < 64 || p->rotaryDim % 64 || (int)p->rotaryDim > Dh)
    return fail(HCU_EUNSUPPORTED, "hcu_attn_prologue: rotaryDim %u (built: multiples of 64 up to Dh)", p->rotaryDim);
  const int fmt = (int)kv->format;
  if (fmt < HCU_KV_F32 || fmt > HCU_KV_Q8_0_WGSL)
    return fail(HCU_EINVAL, "hcu_attn_prologue: unknown KV format %d", fmt);
  if ((fmt == HCU_KV_Q8_0 || fmt == HCU_KV_Q8_0_WGSL) && (!kv->k_scale || !kv->v_scale))
    return fail(HCU_EINVAL, "hcu_attn_prologue: Q8_0 cache needs k_scale and v_scale");
  const int batch = p->batch ? (int)p->batch : 1;
  if (p->S < 1 || p->H < 1 || p->KV < 1 || p->S > 65535 || batch > 65535)
    return fail(HCU_EINVAL, "hcu_attn_prologue: bad S / H / KV / batch");
  if (batch == 1 && !p->pos_base && !p->kv_row_offset && (long long)p->posBase + p->S > (long long)kv->rows)
    return fail(HCU_EINVAL, "hcu_attn_prologue: cache holds %u rows, need posBase+S = %u", kv->rows,
                p->posBase + p->S);
  ProArgs a{};
  a.q = q;
  a.k = k;
  a.v = v;
  a.qn_w = q_norm;
  a.kn_w = k_norm;
  a.cos_tab = cos_tab;
  a.sin_tab = sin_tab;
  a.q_out = q_out;
  a.gate_out = gate_out;
  a.kc = kv->k;
  a.vc = kv->v;
  a.ks = kv->k_scale;
  a.vs = kv->v_scale;
  a.pos_base = p->pos_base;
  a.row_off = p->kv_row_offset;
  a.seq_row_stride = (long long)p->seq_row_stride;
  a.eps = (double)p->eps;
  a.S = (int)p->S;
  a.H = (int)p->H;
  a.KV = (int)p->KV;
  a.pos_default = (int)p->posBase;
  a.split = p->split_gate ? 1 : 0;
  a.fmt = fmt;
  // (token, sequence, group of four q / k / v rows)
  const long long nrows = (long long)p->H + 2ll * p->KV;
  if (nrows > 4ll * 65535) return fail(HCU_EINVAL, "hcu_attn_prologue: too many heads");
  const dim3 grid(p->S, (unsigned)batch, (unsigned)((nrows + 3) / 4));
  const int hj = (int)p->rotaryDim / 64;
  if (Dh == 128) {
    if (hj == 1) attn_prologue_kernel<4, 1><<<grid, 128, 0, h->stream>>>(a);
    else attn_prologue_kernel<4, 2><<<grid, 128, 0, h->stream>>>(a);
  } else {
    if (hj == 1) attn_prologue_kernel<8, 1><<<grid, 128, 0, h->stream>>>(a);
    else if (hj == 2) attn_prologue_kernel<8, 2><<<grid, 128, 0, h->stream>>>(a);
    else attn_prologue_kernel<8, 4><<<grid, 128, 0, h->stream>>>(a);
  }
  return hcu::after_launch("hcu_attn_prologue");
}
