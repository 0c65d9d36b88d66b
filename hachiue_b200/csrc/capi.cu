// capi.cu - handle lifecycle, housekeeping entry points, error plumbing and the
// reference-shaped hcu_dispatch() seam of libhachiue_cuda.
#include <cudaTypedefs.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "context.h"

namespace {
thread_local std::string g_last_error;
constexpr size_t kDefaultWorkspace = 64ull << 20;

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
}  // namespace

namespace hcu {

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = std::string("hachiue: ") + buf;
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return HCU_OK;
  return fail(HCU_ECUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

int begin_op(hcu_context* h, const char* op) {
  if (!h) return fail(HCU_EINVAL, "%s: null handle", op);
  if (h->inject_count > 0) {
    h->inject_count--;
    return fail(h->inject_status, "%s: injected failure (status %d)", op, h->inject_status);
  }
  return check_cuda(cudaSetDevice(h->device), op);
}

int after_launch(const char* what) { return check_cuda(cudaGetLastError(), what); }

int ensure_scratch(hcu_context* h, size_t bytes, const char* what) {
  if (h->scratch_bytes >= bytes) return HCU_OK;
  HCU_TRY(check_cuda(cudaStreamSynchronize(h->stream), what));
  if (h->scratch) {
    cudaFree(h->scratch);
    h->scratch = nullptr;
    h->scratch_bytes = 0;
  }
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) {
    cudaGetLastError();
    return fail(HCU_ENOMEM, "%s: cannot allocate %zu bytes of scratch", what, bytes);
  }
  h->scratch = p;
  h->scratch_bytes = bytes;
  return HCU_OK;
}

int make_tensor_map(CUtensorMap* map, CUtensorMapDataType dtype, int rank, void* base,
                    const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                    CUtensorMapSwizzle swizzle) {
  std::call_once(g_encode_once, [] {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) return fail(HCU_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    return fail(HCU_EINVAL, "TMA base address %p is not 16-byte aligned", base);
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5];
  cuuint32_t e[5];
  for (int i = 0; i < rank; i++) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i + 1 < rank) {
      s[i] = strides_bytes[i];
      if (s[i] % 16 != 0) return fail(HCU_EINVAL, "TMA stride %llu is not a multiple of 16 bytes",
                                      (unsigned long long)s[i]);
    }
  }
  CUresult r = g_encode(map, dtype, rank, base, d, s, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(HCU_ECUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
  return HCU_OK;
}

}  // namespace hcu

using hcu::check_cuda;
using hcu::fail;

extern "C" {

int hcu_version(void) { return HCU_ABI_VERSION; }

const char* hcu_last_error(void) { return g_last_error.c_str(); }

int hcu_create(int device, size_t workspace_bytes, hcu_handle* out) {
  if (!out) return fail(HCU_EINVAL, "hcu_create: null output pointer");
  *out = nullptr;
  int n = 0;
  HCU_TRY(check_cuda(cudaGetDeviceCount(&n), "hcu_create: cudaGetDeviceCount"));
  if (device < 0 || device >= n) return fail(HCU_EINVAL, "hcu_create: device %d out of range (%d)", device, n);
  HCU_TRY(check_cuda(cudaSetDevice(device), "hcu_create: cudaSetDevice"));
  cudaDeviceProp prop;
  HCU_TRY(check_cuda(cudaGetDeviceProperties(&prop, device), "hcu_create: properties"));
  if (prop.major < 10)
    return fail(HCU_EUNSUPPORTED, "hcu_create: device %d is sm_%d%d; this library is built for sm_100a",
                device, prop.major, prop.minor);
  hcu_context* h = new hcu_context();
  h->device = device;
  h->sm_count = prop.multiProcessorCount;
  h->workspace_bytes = workspace_bytes ? workspace_bytes : kDefaultWorkspace;
  int st = check_cuda(cudaStreamCreateWithFlags(&h->own_stream, cudaStreamNonBlocking), "hcu_create: stream");
  if (st == HCU_OK) st = check_cuda(cudaMalloc(&h->workspace, h->workspace_bytes), "hcu_create: workspace");
  if (st == HCU_OK) st = check_cuda(cudaMemset(h->workspace, 0, h->workspace_bytes), "hcu_create: memset");
  if (st == HCU_OK) st = check_cuda(cudaMalloc(&h->dev_status, sizeof(uint32_t)), "hcu_create: status");
  if (st == HCU_OK) st = check_cuda(cudaMemset(h->dev_status, 0, sizeof(uint32_t)), "hcu_create: status");
  if (st == HCU_OK) st = check_cuda(cudaDeviceSynchronize(), "hcu_create: sync");
  if (st != HCU_OK) {
    if (h->workspace) cudaFree(h->workspace);
    if (h->dev_status) cudaFree(h->dev_status);
    if (h->own_stream) cudaStreamDestroy(h->own_stream);
    delete h;
    return st;
  }
  h->stream = h->own_stream;
  *out = h;
  return HCU_OK;
}

int hcu_destroy(hcu_handle h) {
  if (!h) return HCU_OK;
  cudaSetDevice(h->device);
  cudaStreamSynchronize(h->stream);
  if (h->workspace) cudaFree(h->workspace);
  if (h->dev_status) cudaFree(h->dev_status);
  if (h->scratch) cudaFree(h->scratch);
  if (h->own_stream) cudaStreamDestroy(h->own_stream);
  delete h;
  return HCU_OK;
}

int hcu_set_stream(hcu_handle h, void* stream) {
  if (!h) return fail(HCU_EINVAL, "hcu_set_stream: null handle");
  // NULL is the CUDA legacy default stream (what torch's default stream is),
  // not "the handle's own stream": ops must stay ordered with the caller's work.
  h->stream = reinterpret_cast<cudaStream_t>(stream);
  return HCU_OK;
}

void* hcu_get_stream(hcu_handle h) { return h ? reinterpret_cast<void*>(h->stream) : nullptr; }

int hcu_stream_sync(hcu_handle h) {
  if (!h) return fail(HCU_EINVAL, "hcu_stream_sync: null handle");
  HCU_TRY(check_cuda(cudaSetDevice(h->device), "hcu_stream_sync"));
  return check_cuda(cudaStreamSynchronize(h->stream), "hcu_stream_sync");
}

int hcu_alloc(hcu_handle h, size_t bytes, void** ptr) {
  if (!h || !ptr) return fail(HCU_EINVAL, "hcu_alloc: null argument");
  HCU_TRY(check_cuda(cudaSetDevice(h->device), "hcu_alloc"));
  cudaError_t e = cudaMalloc(ptr, bytes ? bytes : 16);
  if (e == cudaErrorMemoryAllocation) {
    cudaGetLastError();
    return fail(HCU_ENOMEM, "hcu_alloc: out of device memory (%zu bytes)", bytes);
  }
  return check_cuda(e, "hcu_alloc");
}

int hcu_free(hcu_handle h, void* ptr) {
  if (!h) return fail(HCU_EINVAL, "hcu_free: null handle");
  if (!ptr) return HCU_OK;
  HCU_TRY(check_cuda(cudaSetDevice(h->device), "hcu_free"));
  return check_cuda(cudaFree(ptr), "hcu_free");
}

int hcu_memset(hcu_handle h, void* ptr, int value, size_t bytes) {
  if (!h || (!ptr && bytes)) return fail(HCU_EINVAL, "hcu_memset: null argument");
  HCU_TRY(check_cuda(cudaSetDevice(h->device), "hcu_memset"));
  return check_cuda(cudaMemsetAsync(ptr, value, bytes, h->stream), "hcu_memset");
}

int hcu_copy_to_device(hcu_handle h, void* dst, const void* src, size_t bytes) {
  if (!h || ((!dst || !src) && bytes)) return fail(HCU_EINVAL, "hcu_copy_to_device: null argument");
  HCU_TRY(check_cuda(cudaSetDevice(h->device), "hcu_copy_to_device"));
  return check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, h->stream), "hcu_copy_to_device");
}

int hcu_copy_to_host(hcu_handle h, void* dst, const void* src, size_t bytes) {
  if (!h || ((!dst || !src) && bytes)) return fail(HCU_EINVAL, "hcu_copy_to_host: null argument");
  HCU_TRY(check_cuda(cudaSetDevice(h->device), "hcu_copy_to_host"));
  HCU_TRY(check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, h->stream), "hcu_copy_to_host"));
  return check_cuda(cudaStreamSynchronize(h->stream), "hcu_copy_to_host");
}

int hcu_device_status(hcu_handle h, uint32_t* status, int clear) {
  if (!h || !status) return fail(HCU_EINVAL, "hcu_device_status: null argument");
  HCU_TRY(check_cuda(cudaSetDevice(h->device), "hcu_device_status"));
  HCU_TRY(check_cuda(cudaMemcpyAsync(status, h->dev_status, sizeof(uint32_t), cudaMemcpyDeviceToHost, h->stream),
                     "hcu_device_status"));
  HCU_TRY(check_cuda(cudaStreamSynchronize(h->stream), "hcu_device_status"));
  if (clear) {
    HCU_TRY(check_cuda(cudaMemsetAsync(h->dev_status, 0, sizeof(uint32_t), h->stream), "hcu_device_status"));
    // A decode-attention call whose bounded wait gave up may have left split
    // tickets partly counted; re-arm them all so the next call merges correctly.
    HCU_TRY(check_cuda(cudaMemsetAsync(h->workspace, 0, hcu::kTicketBytes, h->stream), "hcu_device_status"));
  }
  return HCU_OK;
}

int hcu_selftest_dirty_tickets(hcu_handle h) {
  if (!h) return fail(HCU_EINVAL, "hcu_selftest_dirty_tickets: null handle");
  HCU_TRY(check_cuda(cudaSetDevice(h->device), "hcu_selftest_dirty_tickets"));
  return check_cuda(cudaMemsetAsync(h->workspace, 0x01, hcu::kTicketBytes, h->stream), "hcu_selftest_dirty_tickets");
}

int hcu_set_option(hcu_handle h, int option, int64_t value) {
  if (!h) return fail(HCU_EINVAL, "hcu_set_option: null handle");
  if (value < 0) return fail(HCU_EINVAL, "hcu_set_option: negative value %lld", (long long)value);
  switch (option) {
    case HCU_OPT_ATTN_CUDA_CORES: h->opt_attn_cuda_cores = value; return HCU_OK;
    case HCU_OPT_ATTN_CHUNK: h->opt_attn_chunk = value; return HCU_OK;
    case HCU_OPT_GDN_SCRATCH_MB: h->opt_gdn_scratch_mb = value; return HCU_OK;
    case HCU_OPT_SWA_CTAS: h->opt_swa_ctas = value; return HCU_OK;
    case HCU_OPT_GDN_CHAIN_COLS:
      if (value != 0 && value != 64 && value != 128)
        return fail(HCU_EINVAL, "hcu_set_option: HCU_OPT_GDN_CHAIN_COLS must be 0, 64 or 128 (got %lld)",
                    (long long)value);
      h->opt_gdn_chain_cols = value;
      return HCU_OK;
  }
  return fail(HCU_EINVAL, "hcu_set_option: unknown option %d", option);
}

int hcu_set_q8_convention(hcu_handle h, uint32_t format) {
  if (!h) return fail(HCU_EINVAL, "hcu_set_q8_convention: null handle");
  if (format != HCU_KV_Q8_0 && format != HCU_KV_Q8_0_WGSL)
    return fail(HCU_EINVAL, "hcu_set_q8_convention: format %u is not a Q8_0 convention", format);
  h->q8_format = format;
  return HCU_OK;
}

int hcu_inject_failure(hcu_handle h, int status, int n) {
  if (!h) return fail(HCU_EINVAL, "hcu_inject_failure: null handle");
  h->inject_status = status;
  h->inject_count = status ? n : 0;
  return HCU_OK;
}

int hcu_dispatch(hcu_handle h, const char* shader, const uint32_t words[8], void* const* buffers,
                 int n_buffers) {
  if (!shader || !words) return fail(HCU_EINVAL, "hcu_dispatch: null shader name or uniform words");
  auto need = [&](int n) -> int {
    if (n_buffers < n || !buffers) return fail(HCU_EINVAL, "%s: expected %d storage buffers, got %d", shader, n, n_buffers);
    for (int i = 0; i < n; i++)
      if (!buffers[i]) return fail(HCU_EINVAL, "%s: storage buffer %d is null", shader, i + 1);
    return HCU_OK;
  };
  if (!strcmp(shader, "kv_append_q8")) {
    HCU_TRY(need(3));
    if (!h) return fail(HCU_EINVAL, "kv_append_q8: null handle");
    return hcu_kv_append(h, words[0], words[1], words[2], words[3], h->q8_format,
                         static_cast<const float*>(buffers[0]), buffers[1], static_cast<float*>(buffers[2]));
  }
  if (!strcmp(shader, "attention_q8")) {
    HCU_TRY(need(6));
    hcu_attention_params p{};
    p.S = words[0];
    p.H = words[1];
    p.KV = words[2];
    p.Dh = words[3];
    p.posBase = words[4];
    p.windowSize = words[5];
    p.batch = 1;
    if (!h) return fail(HCU_EINVAL, "attention_q8: null handle");
    hcu_kv_cache kv{};
    kv.format = h->q8_format;
    kv.rows = p.posBase + p.S;
    kv.k = buffers[1];
    kv.k_scale = static_cast<float*>(buffers[2]);
    kv.v = buffers[3];
    kv.v_scale = static_cast<float*>(buffers[4]);
    return hcu_attention(h, &p, static_cast<const float*>(buffers[0]), &kv, static_cast<float*>(buffers[5]));
  }
  if (!strcmp(shader, "deltanet_gbeta")) {
    HCU_TRY(need(5));
    return hcu_deltanet_gbeta(h, words[0], words[1], static_cast<const float*>(buffers[0]),
                              static_cast<const float*>(buffers[1]), static_cast<const float*>(buffers[2]),
                              static_cast<const float*>(buffers[3]), static_cast<float*>(buffers[4]));
  }
  if (!strcmp(shader, "deltanet_recur")) {
    HCU_TRY(need(5));
    hcu_deltanet_params p{};
    p.S = words[0];
    p.H = words[1];
    p.DK = words[2];
    p.DV = words[3];
    p.HK = words[4];
    p.loadState = words[5];
    p.batch = 1;
    return hcu_deltanet_recur(h, &p, static_cast<const float*>(buffers[0]), static_cast<const float*>(buffers[1]),
                              static_cast<const float*>(buffers[2]), static_cast<float*>(buffers[3]),
                              static_cast<float*>(buffers[4]));
  }
  if (!strcmp(shader, "conv1d_causal")) {
    HCU_TRY(need(5));
    hcu_conv1d_params p{};
    p.S = words[0];
    p.C = words[1];
    p.K = words[2];
    p.loadState = words[3];
    p.batch = 1;
    return hcu_conv1d_causal(h, &p, static_cast<const float*>(buffers[0]), static_cast<const float*>(buffers[1]),
                             static_cast<const float*>(buffers[2]), static_cast<float*>(buffers[3]),
                             static_cast<float*>(buffers[4]));
  }
  if (!strcmp(shader, "deltanet_norm_gate")) {
    HCU_TRY(need(4));
    float eps;
    memcpy(&eps, &words[2], sizeof(float));  // mkUniform writes rmsEps as an f32 word (src/engine.ts:1399)
    return hcu_deltanet_norm_gate(h, words[0], words[1], eps, static_cast<const float*>(buffers[0]),
                                  static_cast<const float*>(buffers[1]), static_cast<const float*>(buffers[2]),
                                  static_cast<float*>(buffers[3]));
  }
  if (!strcmp(shader, "rmsnorm")) {
    HCU_TRY(need(3));
    float eps;
    memcpy(&eps, &words[2], sizeof(float));  // f32 uniform word (src/engine.ts:1104)
    return hcu_rmsnorm(h, words[0], words[1], eps, words[3], static_cast<const float*>(buffers[0]),
                       static_cast<const float*>(buffers[1]), static_cast<float*>(buffers[2]));
  }
  if (!strcmp(shader, "rope")) {
    HCU_TRY(need(3));
    return hcu_rope(h, words[0], words[1], words[2], words[3], words[4], static_cast<const float*>(buffers[0]),
                    static_cast<const float*>(buffers[1]), static_cast<float*>(buffers[2]));
  }
  if (!strcmp(shader, "split_q_gate")) {
    HCU_TRY(need(3));
    return hcu_split_q_gate(h, words[0], words[1], words[2], static_cast<const float*>(buffers[0]),
                            static_cast<float*>(buffers[1]), static_cast<float*>(buffers[2]));
  }
  if (!strcmp(shader, "sigmoid_gate")) {
    HCU_TRY(need(2));
    return hcu_sigmoid_gate(h, words[0], static_cast<const float*>(buffers[0]), static_cast<float*>(buffers[1]));
  }
  return fail(HCU_EINVAL, "missing pipeline %s", shader);
}

}  // extern "C"
