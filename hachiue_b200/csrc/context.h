// context.h - host-side handle state and error plumbing of libhachiue_cuda.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <atomic>
#include <string>

#include "hachiue_cuda.h"

struct hcu_context {
  int device = 0;
  int sm_count = 148;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  void* workspace = nullptr;  // split-K partials + counters (zeroed at create)
  size_t workspace_bytes = 0;
  uint32_t* dev_status = nullptr;  // device status word (HCU_DEVERR_*)
  void* scratch = nullptr;         // large temporaries of the prefill ops, grown on demand
  size_t scratch_bytes = 0;
  int inject_status = 0;
  int inject_count = 0;
  uint32_t q8_format = HCU_KV_Q8_0;  // Q8_0 convention of hcu_dispatch (hcu_set_q8_convention)
  // hcu_set_option values (0 = the tuned default)
  int64_t opt_attn_cuda_cores = 0;
  int64_t opt_attn_chunk = 0;
  int64_t opt_gdn_scratch_mb = 0;
  int64_t opt_swa_ctas = 0;
  int64_t opt_gdn_chain_cols = 0;
};

namespace hcu {

// Split-merge tickets of the decode-attention kernels: one int per (sequence,
// KV head, query block) unit at the head of the handle's workspace.  Every
// ticket reads 0 between calls (the CTA that draws a unit's last ticket re-arms
// it); hcu_device_status(clear) also zeroes them.
constexpr int kMaxUnits = 1 << 16;
constexpr size_t kTicketBytes = (size_t)kMaxUnits * sizeof(int);

// Records `msg` as this thread's last error and returns `code`.
int fail(int code, const char* fmt, ...);
// Maps a CUDA error to HCU_ECUDA with context; HCU_OK for cudaSuccess.
int check_cuda(cudaError_t e, const char* what);
// Validates the handle and consumes one injected failure, if armed.
int begin_op(hcu_context* h, const char* op);
// Launch-status check after a kernel launch.
int after_launch(const char* what);
// Kernel attributes such as the dynamic shared-memory limit belong to a
// device: a call site sets them once per device, recorded in `done` (one bit
// per device id; ids of 64 and above set them on every call).
template <typename F>
int once_per_device(std::atomic<uint64_t>& done, int device, F&& set) {
  const uint64_t bit = (device >= 0 && device < 64) ? (1ull << device) : 0ull;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return HCU_OK;
  const int rc = set();
  if (rc == HCU_OK && bit) done.fetch_or(bit, std::memory_order_acq_rel);
  return rc;
}
// Makes h->scratch at least `bytes` long.  Growing synchronises the handle's
// stream (queued work may still read the old buffer) and reallocates.
int ensure_scratch(hcu_context* h, size_t bytes, const char* what);

// Encodes a tiled TMA descriptor (row-major tensor, dims innermost first).
int make_tensor_map(CUtensorMap* map, CUtensorMapDataType dtype, int rank, void* base,
                    const uint64_t* dims, const uint64_t* strides_bytes /* rank-1 */,
                    const uint32_t* box, CUtensorMapSwizzle swizzle);

}  // namespace hcu

#define HCU_TRY(expr)            \
  do {                           \
    int _st = (expr);            \
    if (_st != HCU_OK) return _st; \
  } while (0)
