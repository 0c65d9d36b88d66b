/* mock_napi.c - a small stand-in for the Node-API runtime, enough to load
 * hachiue_b200/napi/hachiue_napi.c and call its exports from Python (ctypes)
 * the way Node would call them from JS.  Test infrastructure only.
 *
 * Values follow the documented Node-API semantics for the calls the addon
 * makes: napi_get_cb_info fills missing arguments with undefined and reports
 * the real count; napi_get_typedarray_info returns the data pointer already
 * advanced by the byte offset; napi_get_value_string_utf8 truncates to the
 * buffer and reports the bytes copied; a callback that returns NULL returns
 * undefined; napi_throw_error leaves one pending exception.  mock_gc() plays
 * the garbage collector: it runs every External's finalizer once. */
#define _POSIX_C_SOURCE 200809L
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "node_api.h"

enum { K_UNDEF, K_NUMBER, K_BOOL, K_STRING, K_BIGINT, K_EXTERNAL, K_TYPEDARRAY, K_FUNCTION, K_OBJECT };

#define MAX_PROPS 64

struct napi_value__ {
  int kind;
  double num;
  bool b;
  uint64_t big;
  bool lossless;
  char *str;
  void *ext;
  napi_finalize fin;
  void *hint;
  bool finalized;
  napi_typedarray_type ta_type;
  void *ta_data;
  size_t ta_len, ta_off;
  napi_callback fn;
  int nprops;
  char *pnames[MAX_PROPS];
  napi_value pvals[MAX_PROPS];
  napi_value next; /* every value of the env, for freeing and for mock_gc */
};

struct napi_env__ {
  napi_value values;
  napi_value exports;
  bool pending;
  char message[512];
};

struct napi_callback_info__ {
  size_t argc;
  napi_value *argv;
};

static napi_value new_value(napi_env env, int kind) {
  napi_value v = (napi_value)calloc(1, sizeof *v);
  v->kind = kind;
  v->next = env->values;
  env->values = v;
  return v;
}

/* ---- the Node-API calls ------------------------------------------------- */

napi_status napi_get_undefined(napi_env env, napi_value *result) {
  if (!env || !result) return napi_invalid_arg;
  *result = new_value(env, K_UNDEF);
  return napi_ok;
}

napi_status napi_throw_error(napi_env env, const char *code, const char *msg) {
  (void)code;
  if (!env || !msg) return napi_invalid_arg;
  if (!env->pending) {
    env->pending = true;
    snprintf(env->message, sizeof env->message, "%s", msg);
  }
  return napi_ok;
}

napi_status napi_get_cb_info(napi_env env, napi_callback_info cbinfo, size_t *argc, napi_value *argv,
                             napi_value *this_arg, void **data) {
  if (!env || !cbinfo) return napi_invalid_arg;
  if (argv) {
    if (!argc) return napi_invalid_arg;
    for (size_t i = 0; i < *argc; i++) {
      if (i < cbinfo->argc) {
        argv[i] = cbinfo->argv[i];
      } else {
        napi_get_undefined(env, &argv[i]);
      }
    }
  }
  if (argc) *argc = cbinfo->argc;
  if (this_arg) napi_get_undefined(env, this_arg);
  if (data) *data = NULL;
  return napi_ok;
}

napi_status napi_create_function(napi_env env, const char *utf8name, size_t length, napi_callback cb, void *data,
                                 napi_value *result) {
  (void)data;
  if (!env || !cb || !result) return napi_invalid_arg;
  napi_value v = new_value(env, K_FUNCTION);
  v->fn = cb;
  if (utf8name) v->str = length == NAPI_AUTO_LENGTH ? strdup(utf8name) : strndup(utf8name, length);
  *result = v;
  return napi_ok;
}

napi_status napi_set_named_property(napi_env env, napi_value object, const char *utf8name, napi_value value) {
  if (!env || !object || !utf8name || !value) return napi_invalid_arg;
  if (object->kind != K_OBJECT) return napi_object_expected;
  if (object->nprops >= MAX_PROPS) return napi_generic_failure;
  object->pnames[object->nprops] = strdup(utf8name);
  object->pvals[object->nprops] = value;
  object->nprops++;
  return napi_ok;
}

napi_status napi_create_int32(napi_env env, int32_t value, napi_value *result) {
  if (!env || !result) return napi_invalid_arg;
  *result = new_value(env, K_NUMBER);
  (*result)->num = value;
  return napi_ok;
}

napi_status napi_create_uint32(napi_env env, uint32_t value, napi_value *result) {
  if (!env || !result) return napi_invalid_arg;
  *result = new_value(env, K_NUMBER);
  (*result)->num = value;
  return napi_ok;
}

napi_status napi_create_bigint_uint64(napi_env env, uint64_t value, napi_value *result) {
  if (!env || !result) return napi_invalid_arg;
  *result = new_value(env, K_BIGINT);
  (*result)->big = value;
  (*result)->lossless = true;
  return napi_ok;
}

napi_status napi_create_external(napi_env env, void *data, napi_finalize finalize_cb, void *finalize_hint,
                                 napi_value *result) {
  if (!env || !result) return napi_invalid_arg;
  napi_value v = new_value(env, K_EXTERNAL);
  v->ext = data;
  v->fin = finalize_cb;
  v->hint = finalize_hint;
  *result = v;
  return napi_ok;
}

napi_status napi_get_value_external(napi_env env, napi_value value, void **result) {
  if (!env || !value || !result) return napi_invalid_arg;
  if (value->kind != K_EXTERNAL) return napi_invalid_arg;
  *result = value->ext;
  return napi_ok;
}

napi_status napi_get_value_uint32(napi_env env, napi_value value, uint32_t *result) {
  if (!env || !value || !result) return napi_invalid_arg;
  if (value->kind != K_NUMBER) return napi_number_expected;
  double d = value->num;
  *result = (d != d) ? 0u : (uint32_t)(int64_t)d; /* ToUint32 for the values a test passes */
  return napi_ok;
}

napi_status napi_get_value_int64(napi_env env, napi_value value, int64_t *result) {
  if (!env || !value || !result) return napi_invalid_arg;
  if (value->kind != K_NUMBER) return napi_number_expected;
  double d = value->num;
  *result = (d != d || d > 9.2e18 || d < -9.2e18) ? 0 : (int64_t)d;
  return napi_ok;
}

napi_status napi_get_value_bool(napi_env env, napi_value value, bool *result) {
  if (!env || !value || !result) return napi_invalid_arg;
  if (value->kind != K_BOOL) return napi_boolean_expected;
  *result = value->b;
  return napi_ok;
}

napi_status napi_get_value_bigint_uint64(napi_env env, napi_value value, uint64_t *result, bool *lossless) {
  if (!env || !value || !result || !lossless) return napi_invalid_arg;
  if (value->kind != K_BIGINT) return napi_bigint_expected;
  *result = value->big;
  *lossless = value->lossless;
  return napi_ok;
}

napi_status napi_get_value_string_utf8(napi_env env, napi_value value, char *buf, size_t bufsize, size_t *result) {
  if (!env || !value) return napi_invalid_arg;
  if (value->kind != K_STRING) return napi_string_expected;
  size_t len = strlen(value->str);
  if (!buf) {
    if (!result) return napi_invalid_arg;
    *result = len;
    return napi_ok;
  }
  size_t n = 0;
  if (bufsize > 0) {
    n = len < bufsize - 1 ? len : bufsize - 1;
    memcpy(buf, value->str, n);
    buf[n] = 0;
  }
  if (result) *result = n;
  return napi_ok;
}

napi_status napi_get_typedarray_info(napi_env env, napi_value typedarray, napi_typedarray_type *type, size_t *length,
                                     void **data, napi_value *arraybuffer, size_t *byte_offset) {
  if (!env || !typedarray) return napi_invalid_arg;
  if (typedarray->kind != K_TYPEDARRAY) return napi_invalid_arg;
  if (type) *type = typedarray->ta_type;
  if (length) *length = typedarray->ta_len;
  if (data) *data = typedarray->ta_data;
  if (arraybuffer) napi_get_undefined(env, arraybuffer);
  if (byte_offset) *byte_offset = typedarray->ta_off;
  return napi_ok;
}

/* ---- the test driver's side (called through ctypes) ---------------------- */

napi_value napi_register_module_v1(napi_env env, napi_value exports);

napi_env mock_env_new(void) { return (napi_env)calloc(1, sizeof(struct napi_env__)); }

int mock_gc(napi_env env) {
  int n = 0;
  for (napi_value v = env->values; v; v = v->next) {
    if (v->kind == K_EXTERNAL && v->fin && !v->finalized) {
      v->finalized = true;
      v->fin(env, v->ext, v->hint);
      n++;
    }
  }
  return n;
}

void mock_env_free(napi_env env) {
  if (!env) return;
  mock_gc(env);
  napi_value v = env->values;
  while (v) {
    napi_value nx = v->next;
    free(v->str);
    for (int i = 0; i < v->nprops; i++) free(v->pnames[i]);
    free(v);
    v = nx;
  }
  free(env);
}

/* Load the addon: Node passes an empty exports object and keeps what the
 * init function returns.  Returns the number of exports, or -1. */
int mock_register(napi_env env) {
  napi_value exports = new_value(env, K_OBJECT);
  napi_value r = napi_register_module_v1(env, exports);
  if (!r || r->kind != K_OBJECT) return -1;
  env->exports = r;
  return r->nprops;
}

const char *mock_export_name(napi_env env, int i) {
  return (env->exports && i >= 0 && i < env->exports->nprops) ? env->exports->pnames[i] : NULL;
}

napi_value mock_undefined(napi_env env) { return new_value(env, K_UNDEF); }

napi_value mock_number(napi_env env, double x) {
  napi_value v = new_value(env, K_NUMBER);
  v->num = x;
  return v;
}

napi_value mock_bool(napi_env env, int x) {
  napi_value v = new_value(env, K_BOOL);
  v->b = x != 0;
  return v;
}

napi_value mock_string(napi_env env, const char *s) {
  napi_value v = new_value(env, K_STRING);
  v->str = strdup(s);
  return v;
}

/* lossless = 0 stands for a bigint outside [0, 2^64), e.g. a negative one. */
napi_value mock_bigint(napi_env env, uint64_t x, int lossless) {
  napi_value v = new_value(env, K_BIGINT);
  v->big = x;
  v->lossless = lossless != 0;
  return v;
}

/* A typed array over caller-owned memory (a numpy array), like a JS view on
 * an ArrayBuffer the caller keeps alive. */
napi_value mock_typedarray(napi_env env, int type, void *data, size_t length) {
  napi_value v = new_value(env, K_TYPEDARRAY);
  v->ta_type = (napi_typedarray_type)type;
  v->ta_data = data;
  v->ta_len = length;
  return v;
}

/* An External some other addon made: no finalizer, arbitrary payload. */
napi_value mock_foreign_external(napi_env env, void *p) {
  napi_value v = new_value(env, K_EXTERNAL);
  v->ext = p;
  return v;
}

/* Call exports[name](...argv).  A NULL return from the callback is undefined. */
napi_value mock_call(napi_env env, const char *name, size_t argc, napi_value *argv) {
  if (!env->exports) return NULL;
  for (int i = 0; i < env->exports->nprops; i++) {
    if (strcmp(env->exports->pnames[i], name) == 0) {
      napi_value f = env->exports->pvals[i];
      if (f->kind != K_FUNCTION) return NULL;
      struct napi_callback_info__ info = {argc, argv};
      napi_value r = f->fn(env, &info);
      return r ? r : new_value(env, K_UNDEF);
    }
  }
  return NULL;
}

/* The pending exception's message, cleared on read; NULL when none. */
const char *mock_take_exception(napi_env env) {
  if (!env->pending) return NULL;
  env->pending = false;
  return env->message;
}

int mock_kind(napi_value v) { return v ? v->kind : -1; }
double mock_as_number(napi_value v) { return v->num; }
uint64_t mock_as_bigint(napi_value v) { return v->big; }
