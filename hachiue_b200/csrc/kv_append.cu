// kv_append.cu - append S rows of K or V into the KV cache.
//
// Q8_0 follows appendKvQ8 (src/wasm-backend.ts:793-824) bit for bit: per
// 32-element block amax = max|x|, scale = amax / 127 (f64) stored as f32,
// q = clamp(Math.round(x * (127 / amax)), -127, 127) with Math.round's
// ties-toward-+infinity rule, all in f64 like the JS "number" arithmetic.
// HCU_KV_Q8_0_WGSL follows the WGSL kv_append_q8 (src/kernels.ts:1287-1335)
// bit for bit instead: f32 arithmetic, round() ties-to-even, scale amax.
// One warp quantises one block (the WGSL twin, kernels.ts:1287-1335, uses one
// 32-thread workgroup per block as well).  F32 / F16 / BF16 rows are plain
// converting copies (round-to-nearest-even).
#include "common.cuh"
#include "context.h"

namespace {

using namespace hcu;

__device__ __forceinline__ double js_round(double x) {
  const double f = floor(x);
  return (x - f >= 0.5) ? f + 1.0 : f;
}

// Source block `blk` goes to destination block dst_block0 + blk, or, with a
// row map, to block dst_rows[blk / blocks_per_row] * blocks_per_row + blk % blocks_per_row.
// One append (a source, its cache tensor and scales); blockIdx.y selects one of
// two, so K and V rows of a decode step go out in one launch.
template <typename T>
struct AppendPair {
  const float* src[2];
  T* dst[2];
  float* scale[2];
};

template <bool WGSL>
__global__ void __launch_bounds__(256) kv_append_q8_kernel(const AppendPair<int8_t> pr, long long total_blocks,
                                                           long long dst_block0, const int64_t* __restrict__ dst_rows,
                                                           int blocks_per_row) {
  const float* __restrict__ src = pr.src[blockIdx.y];
  int8_t* __restrict__ cq = pr.dst[blockIdx.y];
  float* __restrict__ cs = pr.scale[blockIdx.y];
  const long long blk = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (blk >= total_blocks) return;
  const float x = src[blk * 32 + lane];
  float amax = fabsf(x);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const long long dst = dst_rows ? dst_rows[blk / blocks_per_row] * blocks_per_row + blk % blocks_per_row
                                 : dst_block0 + blk;
  if constexpr (WGSL) {
    cq[dst * 32 + lane] = (int8_t)q8_quant_wgsl(x, amax);
    if (lane == 0) cs[dst] = q8_scale_wgsl(amax);
  } else {
    const double damax = (double)amax;
    const double inv = damax > 0 ? 127.0 / damax : 0.0;
    double qd = js_round((double)x * inv);
    qd = qd < -127.0 ? -127.0 : (qd > 127.0 ? 127.0 : qd);
    cq[dst * 32 + lane] = (int8_t)(int)qd;
    if (lane == 0) cs[dst] = (float)(damax / 127.0);
  }
}

template <typename T>
__device__ __forceinline__ T cvt_from_f32(float x);
template <>
__device__ __forceinline__ float cvt_from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __half cvt_from_f32<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 cvt_from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

template <typename T>
__global__ void __launch_bounds__(256) kv_append_dense_kernel(const AppendPair<T> pr, long long n,
                                                              const int64_t* __restrict__ dst_rows,
                                                              long long row_elems) {
  const float* __restrict__ src = pr.src[blockIdx.y];
  T* __restrict__ dst = pr.dst[blockIdx.y];
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long o = dst_rows ? dst_rows[i / row_elems] * row_elems + i % row_elems : i;
    dst[o] = cvt_from_f32<T>(src[i]);
  }
}

template <typename T>
AppendPair<T> pair_of(int n, const float* const* src, void* const* data, float* const* scale, long long offset) {
  AppendPair<T> pr{};
  for (int i = 0; i < n; i++) {
    pr.src[i] = src[i];
    pr.dst[i] = static_cast<T*>(data[i]) + offset;
    pr.scale[i] = scale[i];
  }
  return pr;
}

// `n_pairs` (1 or 2) appends of the same shape in one launch.
int append_impl(hcu_context* h, const char* op, uint32_t S, uint32_t KV, uint32_t Dh, uint32_t posBase,
                const int64_t* dst_rows, uint32_t format, int n_pairs, const float* const* srcs, void* const* datas,
                float* const* scales) {
  HCU_TRY(hcu::begin_op(h, op));
  for (int i = 0; i < n_pairs; i++)
    if (!srcs[i] || !datas[i]) return fail(HCU_EINVAL, "%s: null buffer", op);
  if (S == 0 || KV == 0 || Dh == 0) return fail(HCU_EINVAL, "%s: S, KV and Dh must be positive", op);
  const long long row_elems = (long long)KV * Dh;
  const long long n = (long long)S * row_elems;
  const long long dst0 = dst_rows ? 0 : (long long)posBase * row_elems;
  if (format == HCU_KV_Q8_0 || format == HCU_KV_Q8_0_WGSL) {
    for (int i = 0; i < n_pairs; i++)
      if (!scales[i]) return fail(HCU_EINVAL, "%s: Q8_0 needs a scale buffer", op);
    if (Dh % 32) return fail(HCU_EINVAL, "%s: Dh (%u) must be a multiple of 32 for Q8_0", op, Dh);
    const long long blocks = n / 32;
    const long long grid = (blocks + 7) / 8;
    if (grid > 0x7fffffffLL) return fail(HCU_EINVAL, "%s: too many blocks", op);
    auto kern = format == HCU_KV_Q8_0_WGSL ? kv_append_q8_kernel<true> : kv_append_q8_kernel<false>;
    kern<<<dim3((unsigned)grid, (unsigned)n_pairs), 256, 0, h->stream>>>(
        pair_of<int8_t>(n_pairs, srcs, datas, scales, 0), blocks, dst0 / 32, dst_rows, (int)(row_elems / 32));
    return hcu::after_launch(op);
  }
  long long grid = (n + 255) / 256;
  if (grid > 16LL * h->sm_count * 8) grid = 16LL * h->sm_count * 8;
  const dim3 g((unsigned)grid, (unsigned)n_pairs);
  switch (format) {
    case HCU_KV_F32:
      kv_append_dense_kernel<float>
          <<<g, 256, 0, h->stream>>>(pair_of<float>(n_pairs, srcs, datas, scales, dst0), n, dst_rows, row_elems);
      break;
    case HCU_KV_F16:
      kv_append_dense_kernel<__half>
          <<<g, 256, 0, h->stream>>>(pair_of<__half>(n_pairs, srcs, datas, scales, dst0), n, dst_rows, row_elems);
      break;
    case HCU_KV_BF16:
      kv_append_dense_kernel<__nv_bfloat16><<<g, 256, 0, h->stream>>>(
          pair_of<__nv_bfloat16>(n_pairs, srcs, datas, scales, dst0), n, dst_rows, row_elems);
      break;
    default: return fail(HCU_EINVAL, "%s: unknown format %u", op, format);
  }
  return hcu::after_launch(op);
}

}  // namespace

extern "C" int hcu_kv_append(hcu_handle h, uint32_t S, uint32_t KV, uint32_t Dh, uint32_t posBase, uint32_t format,
                             const float* src, void* data, float* scale) {
  return append_impl(h, "hcu_kv_append", S, KV, Dh, posBase, nullptr, format, 1, &src, &data, &scale);
}

extern "C" int hcu_kv_append_rows(hcu_handle h, uint32_t n, uint32_t KV, uint32_t Dh, uint32_t format,
                                  const float* src, const int64_t* dst_rows, void* data, float* scale) {
  if (!dst_rows) return fail(HCU_EINVAL, "hcu_kv_append_rows: null row list");
  return append_impl(h, "hcu_kv_append_rows", n, KV, Dh, 0, dst_rows, format, 1, &src, &data, &scale);
}

extern "C" int hcu_kv_append_rows_kv(hcu_handle h, uint32_t n, uint32_t KV, uint32_t Dh, const float* k_src,
                                     const float* v_src, const int64_t* dst_rows, const hcu_kv_cache* kv) {
  if (!dst_rows || !kv) return fail(HCU_EINVAL, "hcu_kv_append_rows_kv: null row list or cache");
  const float* srcs[2] = {k_src, v_src};
  void* datas[2] = {kv->k, kv->v};
  float* scales[2] = {kv->k_scale, kv->v_scale};
  return append_impl(h, "hcu_kv_append_rows_kv", n, KV, Dh, 0, dst_rows, kv->format, 2, srcs, datas, scales);
}
