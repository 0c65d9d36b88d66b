// attention_noalloc.cu - hcu_attention_noalloc: the decode-attention entry point
// for callers that must not allocate device memory.
//
// Some callers cannot let a library call cudaMalloc: a serving process that
// reserves its whole HBM budget up front in its own pool (a stray cudaMalloc
// either fails or fragments memory the pool owns), or a plugin reached through
// a stateless FFI call that has nowhere to keep an hcu_handle (creating one
// allocates its workspace, status word and stream).  This entry point takes no
// handle and allocates nothing: the split-K scratch that hcu_attention keeps in
// the handle's workspace comes from the fixed-size __device__ array below
// instead, which every GPU that loads this library holds until the process
// exits.
//
// The kernels are the ones hcu_attention launches; only the scratch differs.
#include <mutex>

#include "context.h"

// [tickets: 65536 x int32][split partials ...][status word (last 256 B)]
static __device__ __align__(256) unsigned char g_noalloc_scratch[HCU_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr size_t kStatusBytes = 256;
constexpr int kMaxDevices = 64;

struct NoallocDevice {
  bool ready = false;
  void* scratch = nullptr;  // device address of g_noalloc_scratch on this device
  int sm_count = 0;
  int device = -1;
};

std::mutex g_mu;
NoallocDevice g_devices[kMaxDevices];

// Once per device, with that device current: look up the device address of
// the scratch array (in host code the array's name is only a host-side
// stand-in, never a usable device address) and the SM count.
int setup_device(int dev, NoallocDevice* out) {
  std::lock_guard<std::mutex> lock(g_mu);
  NoallocDevice& d = g_devices[dev];
  if (!d.ready) {
    void* ptr = nullptr;
    HCU_TRY(hcu::check_cuda(cudaGetSymbolAddress(&ptr, g_noalloc_scratch),
                            "hcu_attention_noalloc: cudaGetSymbolAddress(scratch)"));
    int sms = 0, major = 0;
    HCU_TRY(hcu::check_cuda(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev),
                            "hcu_attention_noalloc: SM count"));
    HCU_TRY(hcu::check_cuda(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev),
                            "hcu_attention_noalloc: compute capability"));
    if (major < 10)
      return hcu::fail(HCU_EUNSUPPORTED, "hcu_attention_noalloc: device %d is not sm_100a", dev);
    d.scratch = ptr;
    d.sm_count = sms;
    d.device = dev;
    d.ready = true;
  }
  *out = d;
  return HCU_OK;
}

uint32_t* status_word(void* scratch) {
  return reinterpret_cast<uint32_t*>(static_cast<unsigned char*>(scratch) + HCU_NOALLOC_SCRATCH_BYTES - kStatusBytes);
}

int current_device(const char* op, NoallocDevice* d) {
  int dev = -1;
  HCU_TRY(hcu::check_cuda(cudaGetDevice(&dev), op));
  if (dev < 0 || dev >= kMaxDevices) return hcu::fail(HCU_EINVAL, "%s: device %d", op, dev);
  return setup_device(dev, d);
}

}  // namespace

// For callers without a handle, the failure report of hcu_attention_noalloc:
// a kernel whose bounded wait gave up records it in the status word at the end
// of the static scratch (the only device memory these callers have), and this
// copies it out (into the caller's host word; no allocation) and optionally
// clears it.
extern "C" int hcu_attention_noalloc_status(uint32_t* status, int clear, void* cuda_stream) {
  if (!status) return hcu::fail(HCU_EINVAL, "hcu_attention_noalloc_status: null argument");
  NoallocDevice d;
  HCU_TRY(current_device("hcu_attention_noalloc_status", &d));
  const cudaStream_t stream = reinterpret_cast<cudaStream_t>(cuda_stream);
  HCU_TRY(hcu::check_cuda(cudaMemcpyAsync(status, status_word(d.scratch), sizeof(uint32_t), cudaMemcpyDeviceToHost,
                                          stream),
                          "hcu_attention_noalloc_status: read"));
  HCU_TRY(hcu::check_cuda(cudaStreamSynchronize(stream), "hcu_attention_noalloc_status: sync"));
  if (clear)
    HCU_TRY(hcu::check_cuda(cudaMemsetAsync(status_word(d.scratch), 0, sizeof(uint32_t), stream),
                            "hcu_attention_noalloc_status: clear"));
  return HCU_OK;
}

extern "C" int hcu_attention_noalloc(const hcu_attention_params* p, const float* q, const hcu_kv_cache* kv,
                                     float* out, void* cuda_stream) {
  if (!p || !q || !kv || !out) return hcu::fail(HCU_EINVAL, "hcu_attention_noalloc: null argument");
  NoallocDevice d;
  HCU_TRY(current_device("hcu_attention_noalloc", &d));
  const int dev = d.device;

  const cudaStream_t stream = reinterpret_cast<cudaStream_t>(cuda_stream);
  // Tickets must read 0 when a call starts.  A completed call leaves them at 0,
  // but a call that gave up part-way may not, so clear the slots this call can
  // use (at most batch x KV x S units).  This enqueues a memset on `stream`;
  // it allocates nothing.
  const unsigned long long batch = p->batch ? p->batch : 1;
  unsigned long long units = batch * (unsigned long long)p->KV * (unsigned long long)(p->S ? p->S : 1);
  if (units > (1ull << 16)) units = 1ull << 16;
  HCU_TRY(hcu::check_cuda(cudaMemsetAsync(d.scratch, 0, units * sizeof(int), stream),
                          "hcu_attention_noalloc: clear tickets"));

  // A handle-shaped view of the static scratch, on the stack; it owns nothing.
  hcu_context view;
  view.device = dev;
  view.sm_count = d.sm_count;
  view.own_stream = nullptr;
  view.stream = stream;
  view.workspace = d.scratch;
  view.workspace_bytes = HCU_NOALLOC_SCRATCH_BYTES - kStatusBytes;
  view.dev_status = status_word(d.scratch);
  static_assert(HCU_NOALLOC_SCRATCH_BYTES > hcu::kTicketBytes + kStatusBytes, "scratch smaller than the ticket region");

  const int st = hcu_attention(&view, p, q, kv, out);
  if (st == HCU_ENOMEM)
    return hcu::fail(HCU_ENOMEM,
                     "hcu_attention_noalloc: this call needs more split-K scratch than the %u-byte static array "
                     "holds (HCU_NOALLOC_SCRATCH_BYTES); use hcu_attention with a larger workspace",
                     (unsigned)HCU_NOALLOC_SCRATCH_BYTES);
  return st;
}
