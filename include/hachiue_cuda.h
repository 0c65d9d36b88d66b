/*
 * hachiue_cuda.h - C ABI of libhachiue_cuda.so, the sm_100a (B200) backend for
 * hachiue's attention hot path: GQA decode attention over the KV cache
 * (qwen3 / qwen35 full-attention layers), causal sliding-window attention
 * (plamo3) and the gated delta-rule recurrence of qwen35's Gated DeltaNet
 * layers.
 *
 * The reference drives these ops through one seam,
 *     HachiueEngine.dispatch(pass, shaderName, uniformBuf, storageBufs, gx)
 * (src/engine.ts:1056-1075), with at most eight u32/f32 uniform words packed by
 * mkUniform (src/engine.ts:1040-1054) and storage buffers bound in order at
 * bindings 1..n.  hcu_dispatch() below is that seam; the typed entry points
 * after it are the same ops with named arguments and the batched / tensor-core
 * extensions the B200 build adds.
 *
 * Conventions
 *  - Every function returns HCU_OK (0) or a negative-free status code; the
 *    message of the last failure on the calling thread is hcu_last_error().
 *    No C++ exception crosses this ABI.
 *  - Pointers named "device" are CUDA device pointers on the handle's device.
 *  - Op calls only enqueue work on the handle's stream (asynchronous, like a
 *    WebGPU dispatch); hcu_stream_sync() is the flushDeviceQueue analogue
 *    (src/engine.ts:927-933).  Calls on one handle are not thread-safe, as in
 *    the reference.
 *  - Op calls never allocate device memory.  Split-K partials and counters use
 *    the workspace reserved at hcu_create() time (the reference likewise
 *    pre-allocates every scratch buffer, src/engine.ts:445-474).
 */
#ifndef HACHIUE_CUDA_H
#define HACHIUE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HCU_ABI_VERSION 3  /* 2: hcu_attention_params.gate; 3: HCU_KV_Q8_0_WGSL */

/* Status codes. */
#define HCU_OK 0
#define HCU_EINVAL 1        /* bad argument (size, shape, null pointer, alignment) */
#define HCU_ECUDA 2         /* CUDA runtime / driver error */
#define HCU_ENCCL 3         /* collective error (multi-GPU helpers) */
#define HCU_ETIMEDOUT 4     /* a bounded device-side wait gave up (see hcu_device_status) */
#define HCU_ENOMEM 5        /* allocation or workspace too small */
#define HCU_EUNSUPPORTED 6  /* shape / format combination not built */

/* KV-cache element formats.  The reference always stores Q8_0
 * (src/engine.ts:483-492, src/wasm-backend.ts:358-374): int8 values plus one
 * f32 scale per 32 elements.  F32 / F16 / BF16 are the formats
 * EngineOptions.kvCache (src/types.ts:177) declares. */
#define HCU_KV_F32 0
#define HCU_KV_F16 1
#define HCU_KV_BF16 2
#define HCU_KV_Q8_0 3
/* Q8_0 as the reference's WGSL ops store it: the scale array holds amax
 * (kv_append_q8 writes (amax/127)*127 in f32, src/kernels.ts:1333) and an
 * element dequantises as max(q/127, -1) * amax (unpack4x8snorm,
 * src/kernels.ts:1386-1411).  HCU_KV_Q8_0 is the JS backend's convention
 * (scale = amax/127, element = q * scale, src/wasm-backend.ts:815,861).  Both
 * hold the same int8 values up to the rounding rule (WGSL round() is
 * half-to-even in f32, the JS Math.round half-up in f64). */
#define HCU_KV_Q8_0_WGSL 4

/* Element types of the tensor-core prefill inputs and outputs. */
#define HCU_DT_F32 0
#define HCU_DT_BF16 2

typedef struct hcu_context *hcu_handle;

/* ------------------------------------------------------------------------ */
/* Housekeeping                                                              */
/* ------------------------------------------------------------------------ */

/* ABI version (HCU_ABI_VERSION). */
int hcu_version(void);

/* Message of the last failed call on this thread ("" if none).  Messages start
 * with "hachiue: " like the reference's thrown Errors (src/engine.ts:1066). */
const char *hcu_last_error(void);

/* Create a handle on CUDA device `device` with its own non-blocking stream and
 * `workspace_bytes` of device workspace (0 = default, 64 MiB).  The workspace
 * bounds how many split-K partials one attention call may use. */
int hcu_create(int device, size_t workspace_bytes, hcu_handle *out);
int hcu_destroy(hcu_handle h);

/* Enqueue subsequent ops on `cuda_stream` (e.g. torch.cuda.current_stream()
 * .cuda_stream) instead of the handle's own stream.  NULL is the CUDA legacy
 * default stream.  hcu_get_stream() returns the stream in use (save it to
 * switch back to the handle's own stream). */
int hcu_set_stream(hcu_handle h, void *cuda_stream);
void *hcu_get_stream(hcu_handle h);
int hcu_stream_sync(hcu_handle h);

/* Tuning options of one handle, for tests and profiling; every default is the
 * tuned choice, and 0 restores it.  Options are read when an op is called
 * (never from the environment).
 *   HCU_OPT_ATTN_CUDA_CORES  1: decode attention always on the CUDA-core
 *                            kernel (otherwise f16 / bf16 / Q8_0 caches with
 *                            Dh 128 use the tcgen05 kernels)
 *   HCU_OPT_ATTN_CHUNK       keys per split-K split (rounded up to a tile)
 *   HCU_OPT_GDN_SCRATCH_MB   scratch budget of the chunked GDN prefill, in MiB
 *                            (default 1024); smaller budgets process the
 *                            prompt in slabs of chunks
 *   HCU_OPT_SWA_CTAS         cap on the SWA prefill's persistent grid
 *   HCU_OPT_GDN_CHAIN_COLS   value columns per CTA of the chunked GDN
 *                            prefill's state recurrence: 128 (one CTA per
 *                            sequence and V head) or 64 (two); by default
 *                            64 when that still fits one wave, else 128 */
#define HCU_OPT_ATTN_CUDA_CORES 1
#define HCU_OPT_ATTN_CHUNK 2
#define HCU_OPT_GDN_SCRATCH_MB 3
#define HCU_OPT_SWA_CTAS 4
#define HCU_OPT_GDN_CHAIN_COLS 5
int hcu_set_option(hcu_handle h, int option, int64_t value);

int hcu_alloc(hcu_handle h, size_t bytes, void **device_ptr);
int hcu_free(hcu_handle h, void *device_ptr);
int hcu_memset(hcu_handle h, void *device_ptr, int value, size_t bytes);
int hcu_copy_to_device(hcu_handle h, void *device_dst, const void *host_src, size_t bytes);
int hcu_copy_to_host(hcu_handle h, void *host_dst, const void *device_src, size_t bytes);

/* Device-side status word of the handle: 0, or a bit set by a kernel whose
 * bounded wait gave up (1 = pipeline barrier timeout) or that found its
 * arguments inconsistent and skipped its work (2, e.g. a sequence longer than
 * hcu_attention_params.max_context).  Reading it synchronises the stream.
 * `clear` resets it and re-arms the decode-attention split tickets that a
 * call which gave up may have left partly counted. */
int hcu_device_status(hcu_handle h, uint32_t *status, int clear);

/* Test hook for failure detection: marks every split-merge ticket of the
 * handle's workspace as partly counted, the state a decode-attention call whose
 * bounded wait gave up can leave behind.  hcu_device_status(h, .., clear = 1)
 * re-arms them; until then decode attention on this handle may not merge its
 * splits (outputs unwritten).  No kernel runs and nothing can hang. */
int hcu_selftest_dirty_tickets(hcu_handle h);

/* Single-process multi-GPU: the reference drives one GPUDevice from one Node
 * process (src/engine.ts:320), so a multi-GPU host of this library drives
 * every GPU from one process.  A communicator over
 * `n` of this process's devices (ncclCommInitAll; NCCL is opened with dlopen
 * at the first call, fails with HCU_ENCCL if absent).  Rank i is devices[i]. */
#define HCU_COMM_MAX_DEVICES 16
typedef struct hcu_comm_s *hcu_comm;
int hcu_comm_create(int n, const int *devices, hcu_comm *comm);
/* Destroy once every all-gather enqueued on the communicator has completed
 * (synchronise its streams first). */
int hcu_comm_destroy(hcu_comm comm);

/* Multi-process form (one process per GPU, as under torchrun): rank 0 makes
 * an id with hcu_comm_unique_id and passes its HCU_COMM_ID_BYTES bytes to
 * every rank over any host channel; each rank then joins with its own device
 * (ncclCommInitRank, which returns once all `nranks` ranks have joined).
 * max_ctas > 0 caps the SMs its collectives occupy (ncclConfig_t.maxCTAs),
 * for small gathers that overlap the next step's kernels; 0 leaves NCCL's
 * choice.  The communicator drives one local rank: hcu_allgather takes one
 * send, receive and stream entry. */
#define HCU_COMM_ID_BYTES 128
int hcu_comm_unique_id(uint8_t *id);
int hcu_comm_init_rank(int nranks, int rank, const uint8_t *id, int device, int max_ctas, hcu_comm *comm);

/* All-gather of the sharded path's per-rank outputs, the one collective of
 * the multi-GPU layout: each rank this process drives (entry i: devices[i])
 * sends `bytes` from send[i] and receives every rank's block, rank-major,
 * into recv[i] (nranks * bytes).  streams[i] is a CUDA stream of that
 * device (NULL: its default stream); the call enqueues and returns.  Every
 * argument is checked before any rank's collective is enqueued. */
int hcu_allgather(hcu_comm comm, void *const *send, void *const *recv, size_t bytes, void *const *streams);

/* Test hook for failure detection: the next `n` op calls on this handle fail
 * with `status` on the host before launching anything (0 disables). */
int hcu_inject_failure(hcu_handle h, int status, int n);

/* Failure-detection self-test (no counterpart in the reference, whose device
 * failures surface as onDeviceLost, src/engine.ts:641-643): launches one warp
 * that waits on a pipeline barrier nothing ever signals, through the bounded
 * wait every kernel here uses.  After about 2 s the wait gives up, sets bit 1
 * (timeout) in the handle's device status word and the kernel returns: no
 * fault, and the context stays usable.  Read it with hcu_device_status. */
int hcu_selftest_wait_timeout(hcu_handle h);

/* ------------------------------------------------------------------------ */
/* The reference's dispatch seam                                              */
/* ------------------------------------------------------------------------ */

/* Q8_0 convention of the dispatch seam's "kv_append_q8" / "attention_q8":
 * HCU_KV_Q8_0 (the default: the JS backend's scales, amax/127) or
 * HCU_KV_Q8_0_WGSL (the WGSL ops' scales, amax), so that a cache written by
 * the reference's own WebGPU kv_append_q8 reads correctly here and the
 * reverse.  Per handle. */
int hcu_set_q8_convention(hcu_handle h, uint32_t format);

/* Run the op the reference names `shader` with its uniform words and storage
 * buffers in binding order (src/engine.ts:1056-1075).  Supported names and the
 * buffer lists (all device pointers) are exactly the reference's:
 *
 *   "kv_append_q8"   words [S, KV, Dh, posBase]                 (kernels.ts:1287)
 *                    buffers [src f32, cacheQ int8, cacheS f32]
 *   "attention_q8"   words [S, H, KV, Dh, posBase, windowSize]  (kernels.ts:1341)
 *                    buffers [q f32, Kq int8, Ks f32, Vq int8, Vs f32, out f32]
 *                    The Q8 cache must hold at least posBase+S rows.
 *   "deltanet_gbeta" words [S, H]                               (kernels.ts:1471)
 *                    buffers [a f32, b f32, aNeg f32, dtBias f32, out f32]
 *   "deltanet_recur" words [S, H, DK, DV, HK, loadState]        (kernels.ts:1496)
 *                    buffers [qkvConv f32, gbeta f32, stateIn f32, core f32,
 *                             stateOut f32]   (stateIn == stateOut allowed)
 *   "conv1d_causal"  words [S, C, K, loadState]                 (kernels.ts:1431)
 *                    buffers [x f32, w f32, stateIn f32, y f32, stateOut f32]
 *                    (stateIn == stateOut allowed)
 *   "deltanet_norm_gate" words [rows, DV, eps (f32 bits), 0]   (kernels.ts:1578)
 *                    buffers [core f32, z f32, gamma f32, y f32]
 *   "rmsnorm"        words [rows, D, eps (f32 bits), addUnitOffset] (kernels.ts:324)
 *                    buffers [x f32, gamma f32, y f32]
 *   "rope"           words [S, H, Dh, rotaryDim, posBase]       (kernels.ts:1120)
 *                    buffers [cos f32, sin f32, x f32 (rotated in place)]
 *   "split_q_gate"   words [S, H, Dh]                           (kernels.ts:1155)
 *                    buffers [qg f32, q f32, gate f32]
 *   "sigmoid_gate"   words [N]                                  (kernels.ts:1249)
 *                    buffers [gate f32, att f32 (gated in place)]
 *
 * Q8 scales follow the handle's convention (hcu_set_q8_convention): by
 * default the JS backend's amax/127 (wasm-backend.ts:815), or the WGSL ops'
 * amax (kernels.ts:1333).  Unknown names fail with
 * "hachiue: missing pipeline <name>" (src/engine.ts:1066). */
int hcu_dispatch(hcu_handle h, const char *shader, const uint32_t words[8],
                 void *const *buffers, int n_buffers);

/* ------------------------------------------------------------------------ */
/* Typed ops                                                                 */
/* ------------------------------------------------------------------------ */

/* KV cache of one attention layer: K and V as [rows, KV, Dh] elements of
 * `format` (int8 for Q8_0), row-major; Q8_0 adds f32 scales [rows, KV, Dh/32].
 * Mirrors kCacheQ/kCacheS/vCacheQ/vCacheS (src/engine.ts:339-343). */
typedef struct {
  uint32_t format;     /* HCU_KV_* */
  uint32_t rows;       /* capacity in token rows (all sequences of a packed batch) */
  void *k;             /* device */
  void *v;             /* device */
  float *k_scale;      /* device, Q8_0 only */
  float *v_scale;      /* device, Q8_0 only */
} hcu_kv_cache;

/* Uniform words of attention_q8 (src/kernels.ts:1342) plus a batch extension.
 * Sequence b (0 <= b < batch) has queries q[b, 0..S) at positions
 * pos_base[b] + qi, and its keys / values at cache rows
 * kv_row_offset[b] + j, j in [jStart, pos], jStart = pos+1-windowSize when
 * windowSize > 0 and pos+1 > windowSize, else 0 (kernels.ts:1373-1377,
 * wasm-backend.ts:847).  batch <= 1 with NULL arrays is exactly the
 * reference's single-sequence call. */
typedef struct {
  uint32_t S, H, KV, Dh, posBase, windowSize;
  uint32_t batch;               /* 0 or 1: single sequence */
  uint32_t max_context;         /* >= max_b(pos_base[b] + S); 0 = posBase + S */
  const int32_t *pos_base;      /* device [batch] or NULL: posBase for every sequence */
  const int64_t *kv_row_offset; /* device [batch] or NULL: b * seq_row_stride */
  uint64_t seq_row_stride;      /* rows per sequence when kv_row_offset is NULL */
  const float *gate;            /* device [batch, S, H, Dh] or NULL: out *= sigmoid(gate), the qwen35
                                   attention output gate (sigmoid_gate, src/kernels.ts:1249-1262) */
} hcu_attention_params;

/* out[b, qi, h, :] = softmax_j(q . k_j / sqrt(Dh)) . v_j with the grouped head
 * map kvh = h / (H / KV) (kernels.ts:1361, wasm-backend.ts:851).
 * q and out are f32 [batch, S, H, Dh].  Replaces runAttentionQ8
 * (src/wasm-backend.ts:826-895) and attention_q8 (src/kernels.ts:1341-1426).
 * Split-K flash-decoding over the key range; Dh in {128, 256}. */
int hcu_attention(hcu_handle h, const hcu_attention_params *p, const float *q,
                  const hcu_kv_cache *kv, float *out);

/* hcu_attention for callers that cannot allocate device memory.  This entry
 * point has no counterpart in the reference.
 *
 * Who needs it: a process that reserves its whole HBM budget up front in its
 * own pool (a library cudaMalloc would fail or fragment memory the pool owns),
 * or a plugin reached through a stateless FFI call with nowhere to keep an
 * hcu_handle (creating a handle allocates its workspace, status word and
 * stream).
 *
 * How it works: same arguments and results as hcu_attention, on the caller's
 * `cuda_stream` (NULL = default stream) of the current device, with no handle.
 * The split-K scratch is a file-scope __device__ array of
 * HCU_NOALLOC_SCRATCH_BYTES, which every GPU that loads this library holds
 * until the process exits; the call makes no cudaMalloc / cudaFree or other
 * allocating call.
 *
 * Limits and rules:
 *  - A call whose partials do not fit fails with HCU_ENOMEM and a message
 *    naming the limit (about batch x KV heads x query blocks <= 3800 at
 *    Dh = 128 with 4 rows per KV head).
 *  - The first call on a device looks up the array's device address and the
 *    SM count; make it before any stream capture.
 *  - All calls share the one array (its tickets are cleared at the start of
 *    each call), so calls that overlap on the GPU race: issue them on one
 *    stream or otherwise serialise them.
 *  - A device-side wait that gives up (the output is then invalid) sets a
 *    status word inside the array; read it with hcu_attention_noalloc_status. */
#define HCU_NOALLOC_SCRATCH_BYTES (8u << 20)
int hcu_attention_noalloc(const hcu_attention_params *p, const float *q, const hcu_kv_cache *kv,
                          float *out, void *cuda_stream);

/* The device status word of hcu_attention_noalloc on the current device (the
 * bits of hcu_device_status), for callers without a handle: copies it to
 * *status after the work queued on `cuda_stream` (NULL = default stream)
 * completes, and with `clear` resets it.  Allocates nothing; like the entry
 * point, it has no counterpart in the reference. */
int hcu_attention_noalloc_status(uint32_t *status, int clear, void *cuda_stream);

/* Append S rows of K or V (f32 [S, KV, Dh]) at cache row posBase in `format`.
 * For Q8_0 this is appendKvQ8 (src/wasm-backend.ts:793-824) bit for bit:
 * scale = amax/127 stored as f32, q = clamp(Math.round(x*127/amax), +-127).
 * `data` is K or V of an hcu_kv_cache, `scale` its scale array (Q8_0 only).
 * The call does not know the cache's length: the caller keeps posBase + S
 * within it, as the engine does by allocating maxSeqLen rows up front
 * (src/engine.ts:483-492).  (The Python host checks it against KVCache.rows.) */
int hcu_kv_append(hcu_handle h, uint32_t S, uint32_t KV, uint32_t Dh, uint32_t posBase,
                  uint32_t format, const float *src, void *data, float *scale);

/* Batched decode form of hcu_kv_append: source row i (f32 [n, KV, Dh]) goes to
 * cache row dst_rows[i] (device int64 array), e.g. one new token per sequence
 * of a packed batch.  Same per-row arithmetic as hcu_kv_append; every
 * dst_rows[i] must be a row of the cache. */
int hcu_kv_append_rows(hcu_handle h, uint32_t n, uint32_t KV, uint32_t Dh, uint32_t format,
                       const float *src, const int64_t *dst_rows, void *data, float *scale);

/* The K and V rows of a decode step in one launch: row i of k_src and of
 * v_src (f32 [n, KV, Dh]) goes to cache row dst_rows[i] of kv->k and kv->v,
 * in kv->format, with hcu_kv_append's per-row arithmetic.  The engine issues
 * the two appends as two kv_append_q8 dispatches (src/engine.ts:1448-1449). */
int hcu_kv_append_rows_kv(hcu_handle h, uint32_t n, uint32_t KV, uint32_t Dh, const float *k_src,
                          const float *v_src, const int64_t *dst_rows, const hcu_kv_cache *kv);

/* g = aNeg[h]*softplus(a + dtBias[h]), beta = sigmoid(b); a, b f32 [S, H];
 * out f32 [2, S, H] (g block, then beta block).  deltanet_gbeta
 * (src/kernels.ts:1471-1491, src/wasm-backend.ts:1036-1045). */
int hcu_deltanet_gbeta(hcu_handle h, uint32_t S, uint32_t H, const float *a, const float *b,
                       const float *a_neg, const float *dt_bias, float *out);

/* Uniform words of deltanet_recur (src/kernels.ts:1497) plus a batch
 * extension: sequence b's tensors start at the given per-sequence strides
 * (elements).  H = number of V heads (NV), HK = number of QK heads (NK); V head
 * h reads QK head h % HK (tiled map, kernels.ts:1511). */
typedef struct {
  uint32_t S, H, DK, DV, HK, loadState;
  uint32_t batch;                 /* 0 or 1: single sequence */
  uint64_t qkv_seq_stride;        /* default S * (2*HK*DK + H*DV) */
  uint64_t gbeta_seq_stride;      /* default 2 * S * H */
  uint64_t state_seq_stride;      /* default H * DK * DV */
  uint64_t core_seq_stride;       /* default S * H * DV */
} hcu_deltanet_params;

/* Gated delta-rule scan over S tokens (deltanet_recur, src/kernels.ts:1496-1573;
 * JS src/wasm-backend.ts:1047-1102).  qkvConv f32 [batch, S, 2*HK*DK + H*DV];
 * gbeta f32 [batch, 2, S, H]; state f32 [batch, H, DK, DV] ([dk][dv] order);
 * core f32 [batch, S, H, DV].  loadState = 0 starts from a zero state.
 * state_in == state_out updates in place.  DK = DV = 128. */
int hcu_deltanet_recur(hcu_handle h, const hcu_deltanet_params *p, const float *qkv_conv,
                       const float *gbeta, const float *state_in, float *core, float *state_out);

/* deltanet_gbeta fused into deltanet_recur: one kernel reads a, b
 * ([batch, S, H] f32), aNeg[H], dtBias[H] instead of a precomputed gbeta
 * buffer.  Same results as the two calls in sequence. */
int hcu_deltanet_decode(hcu_handle h, const hcu_deltanet_params *p, const float *qkv_conv,
                        const float *a, const float *b, const float *a_neg,
                        const float *dt_bias, const float *state_in, float *core,
                        float *state_out);

/* The full-attention layer's neighbours of the KV append and the attention
 * (src/engine.ts:1408-1458; JS src/wasm-backend.ts:1125-1157), with the
 * reference's arithmetic (f64, rounded to f32 where the JS stores):
 *   hcu_rmsnorm:      y = x / sqrt(mean(x^2) + eps) * (gamma or 1 + gamma) per
 *                     row of dim (rmsnorm, kernels.ts:324-355);
 *   hcu_rope:         x [S, heads, head_dim] rotated in place at positions
 *                     posBase + s, pairs (i, i + rotary_dim/2), tables
 *                     [pos][rotary_dim/2] (rope, kernels.ts:1120-1150);
 *   hcu_split_q_gate: qg [S, H, 2*Dh] -> q, gate [S, H, Dh] (kernels.ts:1155);
 *   hcu_sigmoid_gate: att[i] *= 1 / (1 + exp(-gate[i])) (kernels.ts:1249). */
int hcu_rmsnorm(hcu_handle h, uint32_t rows, uint32_t dim, float eps, uint32_t add_unit_offset,
                const float *x, const float *gamma, float *y);
int hcu_rope(hcu_handle h, uint32_t S, uint32_t heads, uint32_t head_dim, uint32_t rotary_dim,
             uint32_t posBase, const float *cos_tab, const float *sin_tab, float *x);
int hcu_split_q_gate(hcu_handle h, uint32_t S, uint32_t H, uint32_t Dh, const float *qg, float *q,
                     float *gate);
int hcu_sigmoid_gate(hcu_handle h, uint64_t n, const float *gate, float *att);

/* The attention prologue of a full-attention layer, fused: split_q_gate
 * (qwen35), the per-head q / k RMSNorm, RoPE, and the append of K (normed and
 * rotated) and V to the cache, for S tokens of each of `batch` sequences.
 * Sequence b's tokens sit at positions pos_base[b] + s (or posBase) and cache
 * rows kv_row_offset[b] + pos (or b * seq_row_stride + pos), as in
 * hcu_attention.  q f32 [batch, S, H, Dh] (split_gate: [batch, S, H, 2*Dh],
 * the attn_q GEMV output with the gate in the second half); k, v f32
 * [batch, S, KV, Dh]; q_norm, k_norm f32 [Dh]; cos / sin f32
 * [positions, rotaryDim / 2]; q_out f32 [batch, S, H, Dh]; gate_out f32
 * [batch, S, H, Dh] (split_gate only).  A Q8_0 cache receives exactly what
 * appendKvQ8 of the same rows would write.  Dh 128 or 256; rotaryDim a
 * multiple of 64, at most Dh. */
typedef struct {
  uint32_t S, H, KV, Dh, rotaryDim, posBase;
  uint32_t batch;               /* 0 or 1: single sequence */
  uint32_t split_gate;          /* 1: qwen35 doubled q projection */
  float eps;                    /* rmsEps */
  const int32_t *pos_base;      /* device [batch] or NULL */
  const int64_t *kv_row_offset; /* device [batch] or NULL */
  uint64_t seq_row_stride;
} hcu_attn_prologue_params;

int hcu_attn_prologue(hcu_handle h, const hcu_attn_prologue_params *p, const float *q, const float *k,
                      const float *v, const float *q_norm, const float *k_norm, const float *cos_tab,
                      const float *sin_tab, float *q_out, float *gate_out, const hcu_kv_cache *kv);

/* Causal depthwise conv1d of width K plus SiLU, with its conv state:
 * conv1d_causal (src/kernels.ts:1431-1466; JS src/wasm-backend.ts:1003-1031).
 * x f32 [batch, S, C]; w f32 [C, K]; state f32 [batch, K-1, C], read when
 * loadState and then replaced by the last K-1 rows of the extended sequence
 * (state_in == state_out updates in place); y f32 [batch, S, C] with
 * y[t][c] = silu(sum_j w[c][j] * ext(t + j, c)).  Strides are per sequence, in
 * elements (0 = dense).  1 <= K <= 8. */
typedef struct {
  uint32_t S, C, K, loadState;
  uint32_t batch;                 /* 0 or 1: single sequence */
  uint64_t x_seq_stride;          /* default S * C */
  uint64_t y_seq_stride;          /* default S * C */
  uint64_t state_seq_stride;      /* default (K - 1) * C */
} hcu_conv1d_params;

int hcu_conv1d_causal(hcu_handle h, const hcu_conv1d_params *p, const float *x, const float *w,
                      const float *state_in, float *y, float *state_out);

/* Gated RMSNorm of the recurrence output: y = gamma * core /
 * sqrt(mean(core^2) + eps) * silu(z) per row of DV (deltanet_norm_gate,
 * src/kernels.ts:1578-1611; JS src/wasm-backend.ts:1104-1117).  core, z, y
 * f32 [rows, DV]; gamma f32 [DV]. */
int hcu_deltanet_norm_gate(hcu_handle h, uint32_t rows, uint32_t DV, float eps, const float *core,
                           const float *z, const float *gamma, float *y);

/* One Gated DeltaNet layer step for one token per sequence (decode), fused:
 * conv1d_causal on the pre-conv mix, g / beta, the delta-rule update and the
 * gated RMSNorm, i.e. the dispatches at src/engine.ts:1366-1400 between the
 * qkv / gate GEMVs and the ssm_out GEMV, with neither qkvConv nor core
 * leaving the chip.
 * qkv_mixed f32 [batch, C] (C = 2*HK*DK + H*DV, the attn_qkv GEMV output);
 * conv_w f32 [C, K]; conv state f32 [batch, K-1, C], in and out different
 * buffers (the engine's ping-pong, src/engine.ts:1359-1372); a, b f32
 * [batch, H]; aNeg, dtBias f32 [H]; z f32 [batch, H*DV] (the attn_gate GEMV
 * output); gamma f32 [DV] (ssm_norm); state f32 [batch, H, DK, DV], in place
 * allowed; out f32 [batch, H*DV] (the input of ssm_out).  K = 4,
 * DK = DV = 128, H >= HK. */
typedef struct {
  uint32_t H, HK, DK, DV, K, loadState;
  uint32_t batch;                 /* 0 or 1: single sequence */
  float eps;                      /* rmsEps */
  uint64_t qkv_seq_stride;        /* default C */
  uint64_t conv_seq_stride;       /* default (K - 1) * C */
  uint64_t ab_seq_stride;         /* default H */
  uint64_t z_seq_stride;          /* default H * DV */
  uint64_t state_seq_stride;      /* default H * DK * DV */
  uint64_t out_seq_stride;        /* default H * DV */
} hcu_gdn_step_params;

int hcu_gdn_layer_step(hcu_handle h, const hcu_gdn_step_params *p, const float *qkv_mixed,
                       const float *conv_w, const float *conv_state_in, float *conv_state_out,
                       const float *a, const float *b, const float *a_neg, const float *dt_bias,
                       const float *z, const float *gamma, const float *state_in, float *state_out,
                       float *out);

/* Causal sliding-window attention over whole prompts (plamo3 SWA layers):
 * query i of each sequence attends keys max(0, i - window + 1) .. i
 * (window = 0: full causal), scale 1/sqrt(D), kvh = h / (H / KV).  These are
 * the semantics of attention_q8 / runAttentionQ8 with S = T, posBase = 0
 * (src/kernels.ts:1341-1426, src/wasm-backend.ts:826-895); the reference
 * feeds prompts through them 8 tokens at a time (src/engine.ts:29).
 * q bf16 [B, T, H, D]; k, v bf16 [B, T, KV, D] (RoPE applied); out
 * [B, T, H, D] bf16 or f32.  D = 128.  tcgen05 tensor cores, f32 accumulate. */
typedef struct {
  uint32_t B, T, H, KV, D, window;
  uint32_t out_dtype; /* HCU_DT_BF16 or HCU_DT_F32 */
} hcu_swa_params;

int hcu_swa_prefill(hcu_handle h, const hcu_swa_params *p, const void *q, const void *k, const void *v,
                    void *out);

/* Chunked Gated DeltaNet prefill (qwen35 linear-attention layers over whole
 * prompts): the recurrence of hcu_deltanet_recur / deltanet_recur
 * (src/kernels.ts:1496-1573, src/wasm-backend.ts:1047-1102) evaluated 64
 * tokens at a time in WY form on the tensor cores (bf16 operands, f32
 * accumulation, f32 state carried between chunks).  The reference instead
 * runs the token-serial scan 8 tokens per call (src/engine.ts:29, :1388).
 * q, k: bf16 [B, T, NK, D] (token t of sequence b at element
 * b*q_seq_stride + t*q_row_stride + hk*D); v: bf16 [B, T, NV, D]; V head h
 * reads QK head h % NK.  g (log decay, <= 0) and beta: f32 at
 * b*gb_seq_stride + t*gb_row_stride + h (the reference's gbeta buffer
 * [2, S, NV] is g = gbeta, beta = gbeta + S*NV).  core: f32 [B, T, NV, D];
 * state_in / state_out: f32 [B, NV, D, D] in [dk][dv] order (may alias).
 * D = 128.  Strides of 0 select the dense defaults. */
typedef struct {
  uint32_t B, T, NK, NV, D, load_state;
  uint64_t q_row_stride, k_row_stride, v_row_stride;   /* elements between tokens */
  uint64_t q_seq_stride, k_seq_stride, v_seq_stride;   /* elements between sequences */
  uint64_t gb_row_stride, gb_seq_stride;
} hcu_gdn_prefill_params;

int hcu_deltanet_chunked_prefill(hcu_handle h, const hcu_gdn_prefill_params *p, const void *q,
                                 const void *k, const void *v, const float *g, const float *beta,
                                 const float *state_in, float *core, float *state_out);

/* The same prefill, also writing state snapshots for prefix reuse.  The engine
 * resets a hybrid (GDN) model's cache whenever a new prompt diverges from the
 * token history, because it keeps no GDN state but the latest
 * (src/engine.ts:1580-1584); with snapshots taken every snap_every chunks it can
 * instead restore the last snapshot at or before the common prefix (as
 * state_in of the next call) and prefill only from there.
 * Snapshot j (0 <= j < T / (64 * snap_every)) is the state after token
 * 64 * snap_every * (j + 1): f32 [B, n_snap, NV, D, D], [dk][dv] order, 16-byte
 * aligned.  The snapshots and state_out equal, bit for bit, the state_out of a
 * call over that prefix; a call that resumes from a snapshot reproduces the
 * remaining outputs bit for bit. */
int hcu_deltanet_chunked_prefill_snap(hcu_handle h, const hcu_gdn_prefill_params *p, const void *q,
                                      const void *k, const void *v, const float *g, const float *beta,
                                      const float *state_in, float *core, float *state_out,
                                      uint32_t snap_every, float *snapshots);

#ifdef __cplusplus
}
#endif

#endif /* HACHIUE_CUDA_H */
