/*
 * hachiue_oracle.c - CPU restatement of hachiue's attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the CPU
 * baseline legs of bench.py load this library, as the checker.  The product
 * path (libhachiue_cuda.so) never calls it.
 *
 * Parity status: UNPINNED by the reference.  hachiue is TypeScript; no JS
 * runtime exists in this build environment or on the GPU box, the WGSL twin
 * needs a WebGPU browser, and the reference's tests hold no golden vectors for
 * this path.  Each function below restates one reference function line by
 * line, keeping its JS number semantics: f64 ("number") arithmetic, rounding
 * to f32 exactly where the JS stores into a Float32Array, and Math.round for
 * the Q8 quantiser.  WGSL-semantics variants (f32 arithmetic) are included to
 * cross-check the two reference implementations against each other.
 *
 * Citations are paths within the hachiue project (v0.3.1).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <pthread.h>

/* Minimal parallel-for over [0, n) on `threads` pthreads (dynamic chunks of 1).
 * Used for independent sequences / heads only. */
typedef void (*par_body_fn)(void *ctx, int i);
typedef struct {
  par_body_fn fn;
  void *ctx;
  int n;
  int next;
  pthread_mutex_t mu;
} par_state;

static void *par_worker(void *arg) {
  par_state *st = (par_state *)arg;
  for (;;) {
    pthread_mutex_lock(&st->mu);
    int i = st->next++;
    pthread_mutex_unlock(&st->mu);
    if (i >= st->n) break;
    st->fn(st->ctx, i);
  }
  return NULL;
}

static void parallel_for(int n, int threads, par_body_fn fn, void *ctx) {
  if (threads <= 1 || n <= 1) {
    for (int i = 0; i < n; i++) fn(ctx, i);
    return;
  }
  if (threads > n) threads = n;
  if (threads > 256) threads = 256;
  par_state st = {fn, ctx, n, 0, PTHREAD_MUTEX_INITIALIZER};
  pthread_t tid[256];
  int started = 0;
  for (int t = 0; t < threads; t++)
    if (pthread_create(&tid[t], NULL, par_worker, &st) == 0) started++;
  if (started == 0) par_worker(&st);
  for (int t = 0; t < started; t++) pthread_join(tid[t], NULL);
}

static inline float fround(double x) { return (float)x; }

/* JS Math.round: nearest integer, ties toward +infinity. */
static inline double js_round(double x) {
  double f = floor(x);
  return (x - f >= 0.5) ? f + 1.0 : f;
}

/* IEEE binary16 -> value, as fp16ToFp32 (src/gguf.ts:81-87). */
double oracle_f16_to_f64(uint16_t h) {
  double s = (h & 0x8000) ? -1.0 : 1.0;
  int e = (h >> 10) & 0x1f;
  int m = h & 0x03ff;
  if (e == 0) return s * m * ldexp(1.0, -24);
  if (e == 31) return m ? NAN : s * INFINITY;
  return s * (1024 + m) * ldexp(1.0, e - 25);
}

/* 65536-entry decode table, as the JS backend's fp16Table
 * (src/wasm-backend.ts:26,71,291). */
static double g_f16_table[65536];
static pthread_once_t g_f16_once = PTHREAD_ONCE_INIT;
static void f16_table_init(void) {
  for (int i = 0; i < 65536; i++) g_f16_table[i] = oracle_f16_to_f64((uint16_t)i);
}

static inline double bf16_to_f64(uint16_t h) {
  uint32_t u = ((uint32_t)h) << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* ------------------------------------------------------------------------ */
/* appendKvQ8 (src/wasm-backend.ts:793-824)                                   */
/* ------------------------------------------------------------------------ */
void oracle_append_kv_q8(const float *src, int8_t *cacheQ, float *cacheS, int S, int kvHeads,
                         int headDim, int posBase) {
  const int blocksPerToken = kvHeads * (headDim >> 5);
  const int totalBlocks = S * blocksPerToken;
  for (int blk = 0; blk < totalBlocks; blk++) {
    const int s = blk / blocksPerToken;
    const int rem = blk % blocksPerToken;
    const long srcBase = ((long)s * blocksPerToken + rem) * 32;
    const long dstBlk = ((long)(posBase + s)) * blocksPerToken + rem;
    const long dstBase = dstBlk * 32;
    double amax = 0;
    for (int i = 0; i < 32; i++) {
      double av = fabs((double)src[srcBase + i]);
      if (av > amax) amax = av;
    }
    double scale = amax / 127.0;
    double inv = amax > 0 ? 127.0 / amax : 0;
    cacheS[dstBlk] = fround(scale);
    for (int i = 0; i < 32; i++) {
      double q = js_round((double)src[srcBase + i] * inv);
      cacheQ[dstBase + i] = (int8_t)(q < -127 ? -127 : q > 127 ? 127 : q);
    }
  }
}

/* kv_append_q8 WGSL semantics (src/kernels.ts:1287-1335): f32 arithmetic,
 * amax over the 32-element block, inv = 127/amax (0 when amax is 0), q =
 * clamp(i32(round(v * inv)), -127, 127) with WGSL round()'s ties-to-even
 * (rintf in the default rounding mode), and the stored scale (amax/127)*127. */
void oracle_append_kv_q8_wgsl(const float *src, int8_t *cacheQ, float *cacheAmax, int S, int kvHeads,
                              int headDim, int posBase) {
  const int blocksPerToken = kvHeads * (headDim >> 5);
  const int totalBlocks = S * blocksPerToken;
  for (int blk = 0; blk < totalBlocks; blk++) {
    const int s = blk / blocksPerToken;
    const int rem = blk % blocksPerToken;
    const long srcBase = ((long)s * blocksPerToken + rem) * 32;
    const long dstBlk = ((long)(posBase + s)) * blocksPerToken + rem;
    float amax = 0.0f;
    for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(src[srcBase + i]));
    const volatile float scale = amax / 127.0f;
    const volatile float inv = amax > 0.0f ? 127.0f / amax : 0.0f;
    for (int i = 0; i < 32; i++) {
      const volatile float prod = src[srcBase + i] * inv;
      float q = rintf(prod);
      q = q < -127.0f ? -127.0f : (q > 127.0f ? 127.0f : q);
      cacheQ[dstBlk * 32 + i] = (int8_t)q;
    }
    cacheAmax[dstBlk] = scale * 127.0f;
  }
}

/* ------------------------------------------------------------------------ */
/* runAttentionQ8 (src/wasm-backend.ts:826-895)                               */
/*                                                                          */
/* kv_format 3 (Q8_0) is the JS function itself.  Formats 0/1/2 (f32, f16,   */
/* bf16 caches, which EngineOptions.kvCache declares) keep the same loop with */
/* the dequantisation `kQ * kS` replaced by the stored element's value.      */
/* `kRowOff` shifts the cache rows (packed batches).                         */
/* ------------------------------------------------------------------------ */
static inline double kv_elem(const void *base, int fmt, long idx) {
  switch (fmt) {
    case 0: return ((const float *)base)[idx];
    case 1: return g_f16_table[((const uint16_t *)base)[idx]];
    case 2: return bf16_to_f64(((const uint16_t *)base)[idx]);
    default: return ((const int8_t *)base)[idx];
  }
}

void oracle_attention(const float *q, const void *kQ, const float *kS, const void *vQ,
                      const float *vS, float *out, int S, int heads, int kvHeads, int headDim,
                      int posBase, int windowSize, int kvFormat, long kRowOff) {
  const int groupSize = heads / kvHeads;
  const int b32 = headDim >> 5;
  const double scale = 1.0 / sqrt((double)headDim);
  pthread_once(&g_f16_once, f16_table_init);
  float *acc = (float *)malloc(sizeof(float) * headDim);
  const int q8 = kvFormat == 3;

  for (int qi = 0; qi < S; qi++) {
    const int pos = posBase + qi;
    const int jStart = windowSize > 0 && pos + 1 > windowSize ? pos + 1 - windowSize : 0;
    for (int h = 0; h < heads; h++) {
      const int kvh = h / groupSize;
      const long qBase = ((long)qi * heads + h) * headDim;
      for (int d = 0; d < headDim; d++) acc[d] = 0.0f;
      double m = -1e30;
      double l = 0.0;
      for (int j = jStart; j <= pos; j++) {
        const long kvRow = (kRowOff + j) * kvHeads + kvh;
        const long sBase = kvRow * b32;
        const long qOffBase = kvRow * headDim;
        double dot = 0.0;
        for (int b = 0; b < b32; b++) {
          double subDot = 0.0;
          const long qb = qBase + (b << 5);
          const long kb = qOffBase + (b << 5);
          for (int d = 0; d < 32; d++) subDot += (double)q[qb + d] * kv_elem(kQ, kvFormat, kb + d);
          dot += q8 ? subDot * (double)kS[sBase + b] : subDot;
        }
        const double score = dot * scale;
        const double mNew = score > m ? score : m;
        const double corr = exp(m - mNew);
        const double wgt = exp(score - mNew);
        l = l * corr + wgt;
        for (int b = 0; b < b32; b++) {
          const double vs = q8 ? wgt * (double)vS[sBase + b] : wgt;
          const long vb = qOffBase + (b << 5);
          const int ab = b << 5;
          for (int d = 0; d < 32; d++)
            acc[ab + d] = fround((double)acc[ab + d] * corr + vs * kv_elem(vQ, kvFormat, vb + d));
        }
        m = mNew;
      }
      const double invL = 1.0 / l;
      for (int d = 0; d < headDim; d++) out[qBase + d] = fround((double)acc[d] * invL);
    }
  }
  free(acc);
}

/* Batched driver: sequence b has S queries at q + b*S*heads*headDim, positions
 * posBase[b]+qi, cache rows starting at rowOff[b].  Independent sequences run
 * on `threads` pthreads (the JS runs one sequence per call, single-threaded). */
typedef struct {
  const float *q;
  const void *kQ, *vQ;
  const float *kS, *vS;
  float *out;
  int S, heads, kvHeads, headDim, windowSize, kvFormat;
  const int32_t *posBase;
  const int64_t *rowOff;
} attn_batch_ctx;

static void attn_batch_body(void *p, int b) {
  const attn_batch_ctx *c = (const attn_batch_ctx *)p;
  const long qStride = (long)c->S * c->heads * c->headDim;
  oracle_attention(c->q + b * qStride, c->kQ, c->kS, c->vQ, c->vS, c->out + b * qStride, c->S,
                   c->heads, c->kvHeads, c->headDim, c->posBase[b], c->windowSize, c->kvFormat,
                   c->rowOff[b]);
}

void oracle_attention_batch(const float *q, const void *kQ, const float *kS, const void *vQ,
                            const float *vS, float *out, int batch, int S, int heads,
                            int kvHeads, int headDim, const int32_t *posBase,
                            const int64_t *rowOff, int windowSize, int kvFormat, int threads) {
  attn_batch_ctx c = {q, kQ, vQ, kS, vS, out, S, heads, kvHeads, headDim, windowSize, kvFormat,
                      posBase, rowOff};
  parallel_for(batch, threads, attn_batch_body, &c);
}

/* attention_q8 WGSL semantics (src/kernels.ts:1341-1426): f32 arithmetic, the
 * scale array holds amax (= JS scale * 127) and unpack4x8snorm divides by 127. */
void oracle_attention_q8_wgsl(const float *q, const int8_t *kQ, const float *kAmax,
                              const int8_t *vQ, const float *vAmax, float *out, int S, int H,
                              int KV, int Dh, int posBase, int windowSize) {
  const float scale = 1.0f / sqrtf((float)Dh);
  float *acc = (float *)malloc(sizeof(float) * Dh);
  for (int qi = 0; qi < S; qi++)
    for (int h = 0; h < H; h++) {
      const int pos = posBase + qi;
      const int kvh = h / (H / KV);
      const long qBase = ((long)qi * H + h) * Dh;
      int jStart = 0;
      if (windowSize > 0 && pos + 1 > windowSize) jStart = pos + 1 - windowSize;
      for (int d = 0; d < Dh; d++) acc[d] = 0.0f;
      float m = -1e30f, l = 0.0f;
      for (int j = jStart; j <= pos; j++) {
        const long kvRow = (long)j * KV + kvh;
        float part = 0.0f;
        for (int d = 0; d < Dh; d++) {
          float kn = fmaxf((float)kQ[kvRow * Dh + d] / 127.0f, -1.0f);
          part += q[qBase + d] * (kn * kAmax[kvRow * (Dh >> 5) + (d >> 5)]);
        }
        float score = part * scale;
        float mNew = fmaxf(m, score);
        float corr = expf(m - mNew);
        float wgt = expf(score - mNew);
        l = l * corr + wgt;
        for (int d = 0; d < Dh; d++) {
          float vn = fmaxf((float)vQ[kvRow * Dh + d] / 127.0f, -1.0f);
          acc[d] = acc[d] * corr + wgt * (vn * vAmax[kvRow * (Dh >> 5) + (d >> 5)]);
        }
        m = mNew;
      }
      const float invL = 1.0f / l;
      for (int d = 0; d < Dh; d++) out[qBase + d] = acc[d] * invL;
    }
  free(acc);
}

/* ------------------------------------------------------------------------ */
/* Gated DeltaNet g / beta (src/wasm-backend.ts:1036-1045)                    */
/* ------------------------------------------------------------------------ */
void oracle_deltanet_gbeta(const float *aProj, const float *bProj, const float *aNeg,
                           const float *dtBias, float *gbeta, int S, int NV) {
  const int nGb = S * NV;
  for (int i = 0; i < nGb; i++) {
    const int h = i % NV;
    const double xVal = (double)aProj[i] + (double)dtBias[h];
    const double sp = (xVal > 0 ? xVal : 0) + log(1.0 + exp(-fabs(xVal)));
    gbeta[i] = fround((double)aNeg[h] * sp);
    gbeta[nGb + i] = fround(1.0 / (1.0 + exp(-(double)bProj[i])));
  }
}

/* ------------------------------------------------------------------------ */
/* Gated DeltaNet recurrence (src/wasm-backend.ts:1047-1102)                  */
/*                                                                          */
/* qkvConv f32 [S, 2*NK*DKV + NV*DKV]; gbeta f32 [2, S, NV]; recState f32    */
/* [NV, DKV, DKV] updated in place ([dk][dv] order); core f32 [S, NV, DKV].  */
/* Heads run on `threads` pthreads when > 1 (they are independent).         */
/* ------------------------------------------------------------------------ */
typedef struct {
  const float *qkvConv, *gbeta;
  float *recState, *core;
  int S, NK, NV, DKV;
} recur_ctx;

static void recur_head(void *p, int h) {
  const recur_ctx *c = (const recur_ctx *)p;
  const int S = c->S, NK = c->NK, NV = c->NV, DKV = c->DKV;
  const float *qkvConv = c->qkvConv, *gbeta = c->gbeta;
  float *recState = c->recState, *core = c->core;
  const long keyDim = (long)NK * DKV;
  const long convDim = keyDim * 2 + (long)NV * DKV;
  const long nGb = (long)S * NV;
  const double scale = 1.0 / sqrt((double)DKV);
  float *kNorm = (float *)malloc(sizeof(float) * DKV);
  float *qNorm = (float *)malloc(sizeof(float) * DKV);
  const int hk = h % NK;
  const long sBase = (long)h * DKV * DKV;
  for (int t = 0; t < S; t++) {
    const long rowConv = (long)t * convDim;
    const long qOff = rowConv + (long)hk * DKV;
    const long kOff = rowConv + keyDim + (long)hk * DKV;
    const long vOff = rowConv + keyDim * 2 + (long)h * DKV;
    const long gbIdx = (long)t * NV + h;
    double sk = 0.0, sq = 0.0;
    for (int dk = 0; dk < DKV; dk++) {
      const double qv = qkvConv[qOff + dk];
      const double kv = qkvConv[kOff + dk];
      sq += qv * qv;
      sk += kv * kv;
    }
    const double ik = 1.0 / sqrt(sk + 1e-6);
    const double iq = (1.0 / sqrt(sq + 1e-6)) * scale;
    for (int dk = 0; dk < DKV; dk++) {
      qNorm[dk] = fround((double)qkvConv[qOff + dk] * iq);
      kNorm[dk] = fround((double)qkvConv[kOff + dk] * ik);
    }
    const double gt = exp((double)gbeta[gbIdx]);
    const double bt = gbeta[nGb + gbIdx];
    const long coreBase = ((long)t * NV + h) * DKV;
    for (int dv = 0; dv < DKV; dv++) {
      double kvDot = 0.0;
      for (int dk = 0; dk < DKV; dk++) {
        const long sIdx = sBase + (long)dk * DKV + dv;
        const float sVal = fround((double)recState[sIdx] * gt);
        recState[sIdx] = sVal;
        kvDot += (double)sVal * kNorm[dk];
      }
      const double delta = ((double)qkvConv[vOff + dv] - kvDot) * bt;
      double o = 0.0;
      for (int dk = 0; dk < DKV; dk++) {
        const long sIdx = sBase + (long)dk * DKV + dv;
        const float sVal = fround((double)recState[sIdx] + (double)kNorm[dk] * delta);
        recState[sIdx] = sVal;
        o += (double)sVal * qNorm[dk];
      }
      core[coreBase + dv] = fround(o);
    }
  }
  free(kNorm);
  free(qNorm);
}

void oracle_deltanet_recur(const float *qkvConv, const float *gbeta, float *recState,
                           float *core, int S, int NK, int NV, int DKV, int loadState,
                           int threads) {
  if (!loadState) memset(recState, 0, sizeof(float) * (size_t)NV * DKV * DKV);
  recur_ctx c = {qkvConv, gbeta, recState, core, S, NK, NV, DKV};
  parallel_for(NV, threads, recur_head, &c);
}

/* deltanet_recur WGSL semantics (src/kernels.ts:1496-1573): f32 arithmetic,
 * ping-pong state (stateIn read, stateOut written). */
void oracle_deltanet_recur_wgsl(const float *qkvConv, const float *gbeta, const float *stateIn,
                                float *core, float *stateOut, int S, int H, int DK, int DV,
                                int HK, int loadState) {
  const int keyDim = HK * DK;
  const int valDim = H * DV;
  const int convDim = keyDim * 2 + valDim;
  const float scale = 1.0f / sqrtf((float)DK);
  const int betaOff = S * H;
  float *s = (float *)malloc(sizeof(float) * DK);
  for (int h = 0; h < H; h++) {
    const int hk = h % HK;
    for (int dv = 0; dv < DV; dv++) {
      const long sbase = (long)h * DK * DV + dv;
      for (int dk = 0; dk < DK; dk++) s[dk] = loadState ? stateIn[sbase + (long)dk * DV] : 0.0f;
      for (int t = 0; t < S; t++) {
        const long rowConv = (long)t * convDim;
        const long qOff = rowConv + hk * DK, kOff = rowConv + keyDim + hk * DK;
        const long vOff = rowConv + keyDim * 2 + h * DV;
        const int gbIdx = t * H + h;
        float sk = 0.0f, sq = 0.0f;
        for (int dk = 0; dk < DK; dk++) {
          sk += qkvConv[kOff + dk] * qkvConv[kOff + dk];
          sq += qkvConv[qOff + dk] * qkvConv[qOff + dk];
        }
        const float ik = 1.0f / sqrtf(sk + 1e-6f);
        const float iq = 1.0f / sqrtf(sq + 1e-6f) * scale;
        const float gt = expf(gbeta[gbIdx]);
        const float bt = gbeta[betaOff + gbIdx];
        float kv = 0.0f;
        for (int dk = 0; dk < DK; dk++) {
          s[dk] = s[dk] * gt;
          kv += s[dk] * qkvConv[kOff + dk] * ik;
        }
        const float delta = (qkvConv[vOff + dv] - kv) * bt;
        float o = 0.0f;
        for (int dk = 0; dk < DK; dk++) {
          s[dk] += qkvConv[kOff + dk] * ik * delta;
          o += s[dk] * qkvConv[qOff + dk] * iq;
        }
        core[((long)t * H + h) * DV + dv] = o;
      }
      for (int dk = 0; dk < DK; dk++) stateOut[sbase + (long)dk * DV] = s[dk];
    }
  }
  free(s);
}

/* Batched recurrence driver: sequence b's qkvConv / gbeta / state / core start
 * at the given strides (elements); sequences run on `threads` pthreads. */
typedef struct {
  const float *qkvConv, *gbeta;
  float *recState, *core;
  int S, NK, NV, DKV, loadState;
  long qkvStride, gbStride, stStride, coreStride;
} recur_batch_ctx;

static void recur_batch_body(void *p, int b) {
  const recur_batch_ctx *c = (const recur_batch_ctx *)p;
  oracle_deltanet_recur(c->qkvConv + b * c->qkvStride, c->gbeta + b * c->gbStride,
                        c->recState + b * c->stStride, c->core + b * c->coreStride, c->S, c->NK,
                        c->NV, c->DKV, c->loadState, 1);
}

void oracle_deltanet_recur_batch(const float *qkvConv, const float *gbeta, float *recState,
                                 float *core, int batch, int S, int NK, int NV, int DKV,
                                 int loadState, long qkvStride, long gbStride, long stStride,
                                 long coreStride, int threads) {
  recur_batch_ctx c = {qkvConv, gbeta, recState, core, S, NK, NV, DKV, loadState,
                       qkvStride, gbStride, stStride, coreStride};
  parallel_for(batch, threads, recur_batch_body, &c);
}

/* ------------------------------------------------------------------------ */
/* Causal depthwise conv1d + SiLU with its conv state                        */
/* (src/wasm-backend.ts:1003-1031; WGSL twin conv1d_causal,                  */
/* src/kernels.ts:1431-1466).                                               */
/*                                                                          */
/* qkvMixed f32 [S, C]; convW f32 [C, K]; convState f32 [K-1, C], read when  */
/* loadState and replaced in place by the last K-1 rows of the extended      */
/* sequence; qkvConv f32 [S, C] = silu(sum_j w[c][j] * ext(t + j, c)).        */
/* ------------------------------------------------------------------------ */
static inline double conv_ext(const float *qkvMixed, const float *convState, int m, int c, int C, int K,
                              int loadState) {
  if (m + 1 < K) return loadState ? (double)convState[(long)m * C + c] : 0.0;
  return (double)qkvMixed[(long)(m - (K - 1)) * C + c];
}

void oracle_conv1d_causal(const float *qkvMixed, const float *convW, float *convState, float *qkvConv, int S,
                          int C, int K, int loadState) {
  for (int t = 0; t < S; t++) {
    for (int c = 0; c < C; c++) {
      double acc = 0.0;
      for (int j = 0; j < K; j++)
        acc += (double)convW[(long)c * K + j] * conv_ext(qkvMixed, convState, t + j, c, C, K, loadState);
      qkvConv[(long)t * C + c] = fround(acc / (1.0 + exp(-acc)));
    }
  }
  float *next = (float *)malloc(sizeof(float) * (size_t)(K - 1) * (size_t)C);
  for (int sk = 0; sk < K - 1; sk++)
    for (int c = 0; c < C; c++)
      next[(long)sk * C + c] = fround(conv_ext(qkvMixed, convState, S + sk, c, C, K, loadState));
  memcpy(convState, next, sizeof(float) * (size_t)(K - 1) * (size_t)C);
  free(next);
}

/* ------------------------------------------------------------------------ */
/* Gated RMSNorm y = gamma * rmsnorm(core) * silu(z)                         */
/* (src/wasm-backend.ts:1104-1117; WGSL twin deltanet_norm_gate,             */
/* src/kernels.ts:1578-1611).  core, z, y f32 [rows, DV]; gamma f32 [DV].    */
/* ------------------------------------------------------------------------ */
void oracle_deltanet_norm_gate(const float *core, const float *z, const float *gamma, float *y, int rows, int DV,
                               double eps) {
  for (int r = 0; r < rows; r++) {
    const long base = (long)r * DV;
    double sumSq = 0.0;
    for (int i = 0; i < DV; i++) {
      const double c = core[base + i];
      sumSq += c * c;
    }
    const double inv = 1.0 / sqrt(sumSq / DV + eps);
    for (int i = 0; i < DV; i++) {
      const double zz = z[base + i];
      y[base + i] = fround((double)gamma[i] * ((double)core[base + i] * inv) * (zz / (1.0 + exp(-zz))));
    }
  }
}

/* ------------------------------------------------------------------------ */
/* RMSNorm y = x / sqrt(mean(x^2) + eps) * gamma per row of `dim`            */
/* (runRmsNorm, src/wasm-backend.ts:427-444; WGSL twin rmsnorm,              */
/* src/kernels.ts:324-355, whose addUnitOffset adds 1 to gamma).             */
/* ------------------------------------------------------------------------ */
void oracle_rmsnorm(const float *x, const float *gamma, float *y, int rows, int dim, double eps, int addUnitOffset) {
  for (int r = 0; r < rows; r++) {
    const long base = (long)r * dim;
    double sumSq = 0.0;
    for (int i = 0; i < dim; i++) {
      const double v = x[base + i];
      sumSq += v * v;
    }
    const double inv = 1.0 / sqrt(sumSq / dim + eps);
    for (int i = 0; i < dim; i++) {
      const double g = addUnitOffset ? 1.0 + (double)gamma[i] : (double)gamma[i];
      y[base + i] = fround((double)x[base + i] * inv * g);
    }
  }
}

/* ------------------------------------------------------------------------ */
/* RoPE in place on x [S, nHeads, headDim] at positions posBase + s, rotating */
/* the pairs (i, i + rotaryDim/2) with cos / sin tables [pos][rotaryDim/2]    */
/* (applyRope, src/wasm-backend.ts:767-791; WGSL twin rope,                  */
/* src/kernels.ts:1120-1150).                                               */
/* ------------------------------------------------------------------------ */
void oracle_rope(float *x, int S, int nHeads, int headDim, int rotaryDim, int posBase, const float *cosTab,
                 const float *sinTab) {
  const int halfRot = rotaryDim >> 1;
  for (int s = 0; s < S; s++) {
    const long csBase = (long)(posBase + s) * halfRot;
    for (int h = 0; h < nHeads; h++) {
      const long base = ((long)s * nHeads + h) * headDim;
      for (int pair = 0; pair < halfRot; pair++) {
        const double c = cosTab[csBase + pair], sn = sinTab[csBase + pair];
        const double v0 = x[base + pair], v1 = x[base + pair + halfRot];
        x[base + pair] = fround(v0 * c - v1 * sn);
        x[base + pair + halfRot] = fround(v1 * c + v0 * sn);
      }
    }
  }
}

/* ------------------------------------------------------------------------ */
/* qwen35 attention output gate: att *= 1 / (1 + exp(-gate)) in place        */
/* (src/wasm-backend.ts:1152-1157; WGSL twin sigmoid_gate,                   */
/* src/kernels.ts:1249-1262).                                               */
/* ------------------------------------------------------------------------ */
void oracle_sigmoid_gate(const float *gate, float *att, long n) {
  for (long i = 0; i < n; i++) att[i] = fround((double)att[i] * (1.0 / (1.0 + exp(-(double)gate[i]))));
}
