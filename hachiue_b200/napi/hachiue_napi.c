/* hachiue_napi.c - the Node-API addon that puts libhachiue_cuda behind the
 * reference engine's op seam.
 *
 * The reference (TypeScript under Node) drives every hot-path op through
 * HachiueEngine.dispatch(pass, shaderName, uniformBuf, storageBufs, gx)
 * (src/engine.ts:1056-1075).  A 'cuda' backend (BackendType, src/types.ts:161,
 * 179) loads this addon and routes the ops it accelerates to `dispatch`, with
 * the same op names, the eight uniform words of mkUniform (src/engine.ts:
 * 1040-1054) and the buffers in binding order, each a device pointer the
 * addon's `alloc` returned.  Failures are thrown as Error('hachiue: ...'),
 * the reference's own error text (src/engine.ts:1066).
 *
 * Exports (JS):
 *   version() -> number
 *   create(device, workspaceBytes) -> handle      (an External; hcu_destroy when collected)
 *   destroy(handle)                                (hcu_destroy now; later use of the handle throws)
 *   alloc(handle, bytes) -> bigint                 (device pointer)
 *   free(handle, ptr)
 *   copyToDevice(handle, dst: bigint, src: TypedArray)
 *   copyToHost(handle, dst: TypedArray, src: bigint)
 *   sync(handle)                                   (flushDeviceQueue, src/engine.ts:927-933)
 *   dispatch(handle, shader, words: Uint32Array(8), buffers: BigUint64Array)
 *   setQ8Convention(handle, format)                (HCU_KV_Q8_0 = 3 or HCU_KV_Q8_0_WGSL = 4)
 *   setOption(handle, option, value)               (HCU_OPT_*)
 *   deviceStatus(handle, clear: boolean) -> number (the onDeviceLost analogue)
 *
 * Built by node-gyp (binding.gyp beside this file) against Node's node_api.h
 * and libhachiue_cuda.so.  A handle is used from one JS thread, as the engine
 * uses its device. */
#include <node_api.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "hachiue_cuda.h"

#define NAPI_OK_OR_NULL(call)  \
  do {                         \
    if ((call) != napi_ok) {   \
      return NULL;             \
    }                          \
  } while (0)

static napi_value throw_msg(napi_env env, const char *msg) {
  napi_throw_error(env, NULL, msg);
  return NULL;
}

/* A failed library call: its thread-local message, already "hachiue: ..." or
 * "hcu_...: ...", becomes the thrown Error. */
static napi_value throw_last(napi_env env) {
  const char *m = hcu_last_error();
  return throw_msg(env, (m && m[0]) ? m : "hachiue: CUDA library call failed");
}

static napi_value undefined(napi_env env) {
  napi_value u;
  napi_get_undefined(env, &u);
  return u;
}

static int get_args(napi_env env, napi_callback_info info, size_t want, napi_value *argv) {
  size_t argc = want;
  if (napi_get_cb_info(env, info, &argc, argv, NULL, NULL) != napi_ok) return 0;
  if (argc < want) {
    throw_msg(env, "hachiue: too few arguments");
    return 0;
  }
  return 1;
}

/* The External's payload: the library handle plus a tag, so that an External
 * made by another addon is refused rather than misread, and destroy() can
 * release the handle before the garbage collector runs the finalizer. */
#define HANDLE_TAG 0x68637531u /* "hcu1" */
struct shim_handle {
  uint32_t tag;
  hcu_handle h;
};

static int get_handle(napi_env env, napi_value v, hcu_handle *h) {
  void *p = NULL;
  if (napi_get_value_external(env, v, &p) != napi_ok || !p || ((struct shim_handle *)p)->tag != HANDLE_TAG) {
    throw_msg(env, "hachiue: expected a handle from create()");
    return 0;
  }
  if (!((struct shim_handle *)p)->h) {
    throw_msg(env, "hachiue: the handle was destroyed");
    return 0;
  }
  *h = ((struct shim_handle *)p)->h;
  return 1;
}

static int get_ptr(napi_env env, napi_value v, void **p) {
  uint64_t x = 0;
  bool lossless = false;
  if (napi_get_value_bigint_uint64(env, v, &x, &lossless) != napi_ok || !lossless) {
    throw_msg(env, "hachiue: expected a device pointer (bigint)");
    return 0;
  }
  *p = (void *)(uintptr_t)x;
  return 1;
}

static int get_u32(napi_env env, napi_value v, uint32_t *x) {
  if (napi_get_value_uint32(env, v, x) != napi_ok) {
    throw_msg(env, "hachiue: expected a number");
    return 0;
  }
  return 1;
}

/* Byte counts and option values: a JS number, exact up to 2^53. */
static int get_i64(napi_env env, napi_value v, int64_t *x) {
  if (napi_get_value_int64(env, v, x) != napi_ok) {
    throw_msg(env, "hachiue: expected a number");
    return 0;
  }
  return 1;
}

static int get_size(napi_env env, napi_value v, size_t *x) {
  int64_t y = 0;
  if (!get_i64(env, v, &y)) return 0;
  if (y < 0) {
    throw_msg(env, "hachiue: a size must not be negative");
    return 0;
  }
  *x = (size_t)y;
  return 1;
}

static int get_bytes(napi_env env, napi_value v, void **data, size_t *bytes) {
  napi_typedarray_type type;
  size_t length = 0, offset = 0;
  napi_value buffer;
  if (napi_get_typedarray_info(env, v, &type, &length, data, &buffer, &offset) != napi_ok) {
    throw_msg(env, "hachiue: expected a TypedArray");
    return 0;
  }
  size_t es = 1;
  switch (type) {
    case napi_int16_array: case napi_uint16_array: es = 2; break;
    case napi_int32_array: case napi_uint32_array: case napi_float32_array: es = 4; break;
    case napi_float64_array: case napi_bigint64_array: case napi_biguint64_array: es = 8; break;
    default: es = 1; break;
  }
  *bytes = length * es;
  return 1;
}

static void finalize_handle(napi_env env, void *data, void *hint) {
  struct shim_handle *sh = (struct shim_handle *)data;
  (void)env;
  (void)hint;
  if (!sh) return;
  if (sh->h) hcu_destroy(sh->h);
  sh->tag = 0;
  free(sh);
}

static napi_value Version(napi_env env, napi_callback_info info) {
  (void)info;
  napi_value r;
  NAPI_OK_OR_NULL(napi_create_int32(env, hcu_version(), &r));
  return r;
}

/* create(device, workspaceBytes): 0 bytes = the library's default workspace. */
static napi_value Create(napi_env env, napi_callback_info info) {
  napi_value argv[2];
  uint32_t dev;
  size_t ws;
  if (!get_args(env, info, 2, argv) || !get_u32(env, argv[0], &dev) || !get_size(env, argv[1], &ws)) return NULL;
  struct shim_handle *sh = (struct shim_handle *)calloc(1, sizeof *sh);
  if (!sh) return throw_msg(env, "hachiue: out of host memory");
  if (hcu_create((int)dev, ws, &sh->h) != HCU_OK) {
    free(sh);
    return throw_last(env);
  }
  sh->tag = HANDLE_TAG;
  napi_value ext;
  if (napi_create_external(env, sh, finalize_handle, NULL, &ext) != napi_ok) {
    hcu_destroy(sh->h);
    free(sh);
    return throw_msg(env, "hachiue: could not wrap the handle");
  }
  return ext;
}

/* destroy(handle): releases the device context now (hcu_destroy waits for
 * the handle's stream); the External stays alive until collected, and any
 * later call with it throws. */
static napi_value Destroy(napi_env env, napi_callback_info info) {
  napi_value argv[1];
  hcu_handle h;
  void *p = NULL;
  if (!get_args(env, info, 1, argv) || !get_handle(env, argv[0], &h)) return NULL;
  napi_get_value_external(env, argv[0], &p);
  ((struct shim_handle *)p)->h = NULL;
  if (hcu_destroy(h) != HCU_OK) return throw_last(env);
  return undefined(env);
}

static napi_value Alloc(napi_env env, napi_callback_info info) {
  napi_value argv[2];
  hcu_handle h;
  size_t bytes;
  if (!get_args(env, info, 2, argv) || !get_handle(env, argv[0], &h) || !get_size(env, argv[1], &bytes)) return NULL;
  void *p = NULL;
  if (hcu_alloc(h, bytes, &p) != HCU_OK) return throw_last(env);
  napi_value r;
  NAPI_OK_OR_NULL(napi_create_bigint_uint64(env, (uint64_t)(uintptr_t)p, &r));
  return r;
}

static napi_value Free(napi_env env, napi_callback_info info) {
  napi_value argv[2];
  hcu_handle h;
  void *p;
  if (!get_args(env, info, 2, argv) || !get_handle(env, argv[0], &h) || !get_ptr(env, argv[1], &p)) return NULL;
  if (hcu_free(h, p) != HCU_OK) return throw_last(env);
  return undefined(env);
}

static napi_value CopyToDevice(napi_env env, napi_callback_info info) {
  napi_value argv[3];
  hcu_handle h;
  void *dst, *src;
  size_t bytes;
  if (!get_args(env, info, 3, argv) || !get_handle(env, argv[0], &h) || !get_ptr(env, argv[1], &dst) ||
      !get_bytes(env, argv[2], &src, &bytes))
    return NULL;
  if (hcu_copy_to_device(h, dst, src, bytes) != HCU_OK) return throw_last(env);
  return undefined(env);
}

static napi_value CopyToHost(napi_env env, napi_callback_info info) {
  napi_value argv[3];
  hcu_handle h;
  void *dst, *src;
  size_t bytes;
  if (!get_args(env, info, 3, argv) || !get_handle(env, argv[0], &h) || !get_bytes(env, argv[1], &dst, &bytes) ||
      !get_ptr(env, argv[2], &src))
    return NULL;
  if (hcu_copy_to_host(h, dst, src, bytes) != HCU_OK) return throw_last(env);
  return undefined(env);
}

static napi_value Sync(napi_env env, napi_callback_info info) {
  napi_value argv[1];
  hcu_handle h;
  if (!get_args(env, info, 1, argv) || !get_handle(env, argv[0], &h)) return NULL;
  if (hcu_stream_sync(h) != HCU_OK) return throw_last(env);
  return undefined(env);
}

/* dispatch(handle, shader, words: Uint32Array(8), buffers: BigUint64Array):
 * engine.dispatch's op seam (src/engine.ts:1056-1075). */
static napi_value Dispatch(napi_env env, napi_callback_info info) {
  napi_value argv[4];
  hcu_handle h;
  if (!get_args(env, info, 4, argv) || !get_handle(env, argv[0], &h)) return NULL;
  char name[64];
  size_t n = 0;
  if (napi_get_value_string_utf8(env, argv[1], name, sizeof name, &n) != napi_ok)
    return throw_msg(env, "hachiue: expected a shader name");
  if (n + 1 >= sizeof name) return throw_msg(env, "hachiue: shader name too long");
  napi_typedarray_type wt, bt;
  size_t wlen = 0, blen = 0, off = 0;
  void *words = NULL, *bufs = NULL;
  napi_value ab;
  if (napi_get_typedarray_info(env, argv[2], &wt, &wlen, &words, &ab, &off) != napi_ok || wt != napi_uint32_array ||
      wlen != 8)
    return throw_msg(env, "hachiue: uniform words must be a Uint32Array(8)");
  if (napi_get_typedarray_info(env, argv[3], &bt, &blen, &bufs, &ab, &off) != napi_ok || bt != napi_biguint64_array)
    return throw_msg(env, "hachiue: buffers must be a BigUint64Array of device pointers");
  if (hcu_dispatch(h, name, (const uint32_t *)words, (void *const *)bufs, (int)blen) != HCU_OK)
    return throw_last(env);
  return undefined(env);
}

static napi_value SetQ8Convention(napi_env env, napi_callback_info info) {
  napi_value argv[2];
  hcu_handle h;
  uint32_t fmt;
  if (!get_args(env, info, 2, argv) || !get_handle(env, argv[0], &h) || !get_u32(env, argv[1], &fmt)) return NULL;
  if (hcu_set_q8_convention(h, fmt) != HCU_OK) return throw_last(env);
  return undefined(env);
}

static napi_value SetOption(napi_env env, napi_callback_info info) {
  napi_value argv[3];
  hcu_handle h;
  uint32_t opt;
  int64_t value;
  if (!get_args(env, info, 3, argv) || !get_handle(env, argv[0], &h) || !get_u32(env, argv[1], &opt) ||
      !get_i64(env, argv[2], &value))
    return NULL;
  if (hcu_set_option(h, (int)opt, value) != HCU_OK) return throw_last(env);
  return undefined(env);
}

static napi_value DeviceStatus(napi_env env, napi_callback_info info) {
  napi_value argv[2];
  hcu_handle h;
  bool clear = false;
  if (!get_args(env, info, 2, argv) || !get_handle(env, argv[0], &h)) return NULL;
  if (napi_get_value_bool(env, argv[1], &clear) != napi_ok) return throw_msg(env, "hachiue: expected a boolean");
  uint32_t st = 0;
  if (hcu_device_status(h, &st, clear ? 1 : 0) != HCU_OK) return throw_last(env);
  napi_value r;
  NAPI_OK_OR_NULL(napi_create_uint32(env, st, &r));
  return r;
}

static napi_value Init(napi_env env, napi_value exports) {
  static const struct {
    const char *name;
    napi_callback fn;
  } fns[] = {
      {"version", Version},   {"create", Create},   {"destroy", Destroy},
      {"alloc", Alloc},       {"free", Free},       {"copyToDevice", CopyToDevice},
      {"copyToHost", CopyToHost}, {"sync", Sync},   {"dispatch", Dispatch},
      {"setQ8Convention", SetQ8Convention},         {"setOption", SetOption},
      {"deviceStatus", DeviceStatus},
  };
  for (size_t i = 0; i < sizeof fns / sizeof fns[0]; i++) {
    napi_value f;
    NAPI_OK_OR_NULL(napi_create_function(env, fns[i].name, NAPI_AUTO_LENGTH, fns[i].fn, NULL, &f));
    NAPI_OK_OR_NULL(napi_set_named_property(env, exports, fns[i].name, f));
  }
  return exports;
}

NAPI_MODULE(NODE_GYP_MODULE_NAME, Init)
