/*
 * A small in-process N-API runtime for testing the minisample N-API shim
 * (omni.js_b200/csrc/napi_minisample.c) without Node: JS values are C structs,
 * async work runs `execute` on a pthread and `complete` on the calling thread
 * when the test drains the queue (libuv's split between its thread pool and
 * the event loop), promises record how they settled.  The entry points at the
 * end (fake_*) are called from Python with ctypes.
 *
 * Test infrastructure: built and run only by the tests.
 */
#define _GNU_SOURCE
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "node_api.h"

napi_value ms_fake_module_init(napi_env env, napi_value exports);

enum { K_UNDEF, K_NULL, K_BOOL, K_NUM, K_STR, K_OBJ, K_FUNC, K_TA, K_AB, K_PROMISE, K_ERROR };
enum { P_PENDING, P_RESOLVED, P_REJECTED };
#define MAX_PROPS 16

struct napi_value__ {
  int kind;
  double num;
  bool b;
  char* str; /* K_STR; K_ERROR message */
  int nprops;
  char* keys[MAX_PROPS];
  napi_value vals[MAX_PROPS];
  napi_callback fn;
  napi_typedarray_type tt; /* K_TA */
  size_t len;
  void* data;
  void* ab_data; /* K_AB */
  size_t ab_len;
  int state; /* K_PROMISE */
  napi_value settled;
  struct napi_value__* next; /* arena list */
};

struct napi_env__ {
  int has_exc;
  char exc[600];
};

struct napi_callback_info__ {
  size_t argc;
  napi_value argv[8];
};

struct napi_deferred__ {
  napi_value promise;
};

struct napi_async_work__ {
  napi_async_execute_callback execute;
  napi_async_complete_callback complete;
  void* data;
  pthread_t th;
  int queued, started, done, deleted;
  struct napi_async_work__* next;
};

static struct napi_env__ g_env;
static napi_value g_arena = NULL;
static napi_value g_exports = NULL;
static struct napi_async_work__* g_works = NULL;
static int g_defer_start = 0;

static napi_value new_value(int kind) {
  napi_value v = (napi_value)calloc(1, sizeof(struct napi_value__));
  v->kind = kind;
  v->next = g_arena;
  g_arena = v;
  return v;
}

static napi_value make_number(double x) {
  napi_value v = new_value(K_NUM);
  v->num = x;
  return v;
}

static napi_value make_typed(napi_typedarray_type t, void* data, size_t len) {
  napi_value v = new_value(K_TA);
  v->tt = t;
  v->data = data;
  v->len = len;
  return v;
}

static napi_status set_prop(napi_value o, const char* k, napi_value v) {
  for (int i = 0; i < o->nprops; i++)
    if (!strcmp(o->keys[i], k)) {
      o->vals[i] = v;
      return napi_ok;
    }
  if (o->nprops == MAX_PROPS) return napi_generic_failure;
  o->keys[o->nprops] = strdup(k);
  o->vals[o->nprops++] = v;
  return napi_ok;
}

static napi_value get_prop(napi_value o, const char* k) {
  if (!o || (o->kind != K_OBJ && o->kind != K_ERROR)) return NULL;
  for (int i = 0; i < o->nprops; i++)
    if (!strcmp(o->keys[i], k)) return o->vals[i];
  return NULL;
}

/* ---- N-API */
napi_status napi_get_cb_info(napi_env env, napi_callback_info cbinfo, size_t* argc, napi_value* argv,
                             napi_value* this_arg, void** data) {
  (void)env;
  size_t want = *argc;
  for (size_t i = 0; i < want; i++) argv[i] = i < cbinfo->argc ? cbinfo->argv[i] : new_value(K_UNDEF);
  *argc = cbinfo->argc;
  if (this_arg) *this_arg = NULL;
  if (data) *data = NULL;
  return napi_ok;
}

napi_status napi_typeof(napi_env env, napi_value value, napi_valuetype* result) {
  (void)env;
  static const napi_valuetype map[] = {napi_undefined, napi_null,     napi_boolean, napi_number,
                                       napi_string,    napi_object,   napi_function, napi_object,
                                       napi_object,    napi_object,   napi_object};
  *result = map[value->kind];
  return napi_ok;
}

napi_status napi_get_value_double(napi_env env, napi_value value, double* result) {
  (void)env;
  if (value->kind != K_NUM) return napi_number_expected;
  *result = value->num;
  return napi_ok;
}

napi_status napi_get_value_bool(napi_env env, napi_value value, bool* result) {
  (void)env;
  if (value->kind != K_BOOL) return napi_boolean_expected;
  *result = value->b;
  return napi_ok;
}

napi_status napi_has_named_property(napi_env env, napi_value object, const char* utf8name, bool* result) {
  (void)env;
  if (object->kind != K_OBJ) return napi_object_expected;
  *result = get_prop(object, utf8name) != NULL;
  return napi_ok;
}

napi_status napi_get_named_property(napi_env env, napi_value object, const char* utf8name, napi_value* result) {
  (void)env;
  if (object->kind != K_OBJ) return napi_object_expected;
  napi_value v = get_prop(object, utf8name);
  *result = v ? v : new_value(K_UNDEF);
  return napi_ok;
}

napi_status napi_set_named_property(napi_env env, napi_value object, const char* utf8name, napi_value value) {
  (void)env;
  if (object->kind != K_OBJ) return napi_object_expected;
  return set_prop(object, utf8name, value);
}

napi_status napi_is_typedarray(napi_env env, napi_value value, bool* result) {
  (void)env;
  *result = value->kind == K_TA;
  return napi_ok;
}

napi_status napi_get_typedarray_info(napi_env env, napi_value typedarray, napi_typedarray_type* type,
                                     size_t* length, void** data, napi_value* arraybuffer, size_t* byte_offset) {
  (void)env;
  if (typedarray->kind != K_TA) return napi_invalid_arg;
  if (type) *type = typedarray->tt;
  if (length) *length = typedarray->len;
  if (data) *data = typedarray->data;
  if (arraybuffer) *arraybuffer = NULL;
  if (byte_offset) *byte_offset = 0;
  return napi_ok;
}

napi_status napi_create_arraybuffer(napi_env env, size_t byte_length, void** data, napi_value* result) {
  (void)env;
  napi_value v = new_value(K_AB);
  v->ab_data = calloc(1, byte_length ? byte_length : 1);
  v->ab_len = byte_length;
  *data = v->ab_data;
  *result = v;
  return napi_ok;
}

napi_status napi_create_typedarray(napi_env env, napi_typedarray_type type, size_t length, napi_value arraybuffer,
                                   size_t byte_offset, napi_value* result) {
  (void)env;
  if (arraybuffer->kind != K_AB || type != napi_int32_array || byte_offset + 4 * length > arraybuffer->ab_len)
    return napi_invalid_arg;
  *result = make_typed(type, (char*)arraybuffer->ab_data + byte_offset, length);
  return napi_ok;
}

napi_status napi_create_object(napi_env env, napi_value* result) {
  (void)env;
  *result = new_value(K_OBJ);
  return napi_ok;
}

napi_status napi_create_int32(napi_env env, int32_t value, napi_value* result) {
  (void)env;
  *result = make_number(value);
  return napi_ok;
}

napi_status napi_create_string_utf8(napi_env env, const char* str, size_t length, napi_value* result) {
  (void)env;
  napi_value v = new_value(K_STR);
  v->str = length == NAPI_AUTO_LENGTH ? strdup(str) : strndup(str, length);
  *result = v;
  return napi_ok;
}

napi_status napi_create_error(napi_env env, napi_value code, napi_value msg, napi_value* result) {
  (void)env;
  (void)code;
  if (msg->kind != K_STR) return napi_string_expected;
  napi_value v = new_value(K_ERROR);
  v->str = strdup(msg->str);
  *result = v;
  return napi_ok;
}

static napi_status throw_kind(napi_env env, const char* kind, const char* msg) {
  if (env->has_exc) return napi_pending_exception;
  env->has_exc = 1;
  snprintf(env->exc, sizeof env->exc, "%s: %s", kind, msg);
  return napi_ok;
}

napi_status napi_throw_error(napi_env env, const char* code, const char* msg) {
  (void)code;
  return throw_kind(env, "Error", msg);
}

napi_status napi_throw_type_error(napi_env env, const char* code, const char* msg) {
  (void)code;
  return throw_kind(env, "TypeError", msg);
}

napi_status napi_throw_range_error(napi_env env, const char* code, const char* msg) {
  (void)code;
  return throw_kind(env, "RangeError", msg);
}

napi_status napi_define_properties(napi_env env, napi_value object, size_t property_count,
                                   const napi_property_descriptor* properties) {
  (void)env;
  for (size_t i = 0; i < property_count; i++) {
    napi_value f = new_value(K_FUNC);
    f->fn = properties[i].method;
    if (set_prop(object, properties[i].utf8name, f) != napi_ok) return napi_generic_failure;
  }
  return napi_ok;
}

napi_status napi_create_promise(napi_env env, napi_deferred* deferred, napi_value* promise) {
  (void)env;
  napi_value p = new_value(K_PROMISE);
  struct napi_deferred__* d = (struct napi_deferred__*)calloc(1, sizeof *d);
  d->promise = p;
  *deferred = d;
  *promise = p;
  return napi_ok;
}

static napi_status settle(napi_deferred d, int state, napi_value v) {
  if (!d || d->promise->state != P_PENDING) return napi_generic_failure;
  d->promise->state = state;
  d->promise->settled = v;
  free(d); /* a deferred is released once it settles */
  return napi_ok;
}

napi_status napi_resolve_deferred(napi_env env, napi_deferred deferred, napi_value resolution) {
  (void)env;
  return settle(deferred, P_RESOLVED, resolution);
}

napi_status napi_reject_deferred(napi_env env, napi_deferred deferred, napi_value rejection) {
  (void)env;
  return settle(deferred, P_REJECTED, rejection);
}

napi_status napi_create_async_work(napi_env env, napi_value async_resource, napi_value async_resource_name,
                                   napi_async_execute_callback execute, napi_async_complete_callback complete,
                                   void* data, napi_async_work* result) {
  (void)env;
  (void)async_resource;
  (void)async_resource_name;
  struct napi_async_work__* w = (struct napi_async_work__*)calloc(1, sizeof *w);
  w->execute = execute;
  w->complete = complete;
  w->data = data;
  w->next = g_works;
  g_works = w;
  *result = w;
  return napi_ok;
}

napi_status napi_delete_async_work(napi_env env, napi_async_work work) {
  (void)env;
  work->deleted = 1; /* freed by fake_reset */
  return napi_ok;
}

static void* work_thread(void* arg) {
  struct napi_async_work__* w = (struct napi_async_work__*)arg;
  w->execute(&g_env, w->data);
  return NULL;
}

static void start_work(struct napi_async_work__* w) {
  w->started = 1;
  pthread_create(&w->th, NULL, work_thread, w);
}

napi_status napi_queue_async_work(napi_env env, napi_async_work work) {
  (void)env;
  work->queued = 1;
  if (!g_defer_start) start_work(work);
  return napi_ok;
}

/* ---- entry points for the tests */

void fake_reset(void);

/* Registers the module; returns the number of exported functions. */
int fake_load(void) {
  if (!g_exports) {
    fake_reset();
    g_exports = ms_fake_module_init(&g_env, new_value(K_OBJ));
    g_arena = NULL; /* the exports and their functions outlive fake_reset */
  }
  return g_exports ? g_exports->nprops : -1;
}

/* 1: queued async work starts only at fake_drain (so the test may change the
 * inputs between the call and the run); 0: it starts when queued. */
void fake_set_deferred_start(int on) { g_defer_start = on; }

/* Runs every queued work to the end, then its completion; returns how many. */
int fake_drain(void) {
  int n = 0;
  for (struct napi_async_work__* w = g_works; w; w = w->next)
    if (w->queued && !w->started) start_work(w);
  for (struct napi_async_work__* w = g_works; w; w = w->next)
    if (w->started && !w->done) {
      pthread_join(w->th, NULL);
      w->done = 1;
      w->complete(&g_env, napi_ok, w->data);
      n++;
    }
  return n;
}

/* Frees the values and works of earlier calls (promise handles die with it). */
void fake_reset(void) {
  fake_drain();
  while (g_works) {
    struct napi_async_work__* w = g_works;
    g_works = w->next;
    free(w);
  }
  while (g_arena) {
    napi_value v = g_arena;
    g_arena = v->next;
    for (int i = 0; i < v->nprops; i++) free(v->keys[i]);
    free(v->str);
    free(v->ab_data);
    free(v);
  }
  g_env.has_exc = 0;
}

static napi_value call_export(const char* name, size_t argc, napi_value* argv, char* err, size_t errlen) {
  napi_value f = get_prop(g_exports, name);
  if (!f || f->kind != K_FUNC) {
    snprintf(err, errlen, "no export %s", name);
    return NULL;
  }
  struct napi_callback_info__ info;
  info.argc = argc;
  for (size_t i = 0; i < argc; i++) info.argv[i] = argv[i];
  g_env.has_exc = 0;
  napi_value r = f->fn(&g_env, &info);
  if (g_env.has_exc) {
    snprintf(err, errlen, "%s", g_env.exc);
    g_env.has_exc = 0;
    return NULL;
  }
  if (!r) snprintf(err, errlen, "no result and no exception");
  return r;
}

/* Builds sample(...)'s seven arguments.  NULL logits: a number in its place;
 * NULL history/offsets/uniforms: JS null.  opts[5] = doSample, temperature,
 * topK, topP, repetitionPenalty, each present when its bit in opts_mask is set
 * (doSample as a boolean). */
static void make_args(napi_value* a, float* logits, size_t nlog, double B, double V, int32_t* hist, size_t nh,
                      int32_t* off, size_t no, const double* opts, int opts_mask, double* u, size_t nu) {
  a[0] = logits ? make_typed(napi_float32_array, logits, nlog) : make_number(0);
  a[1] = make_number(B);
  a[2] = make_number(V);
  a[3] = hist ? make_typed(napi_int32_array, hist, nh) : new_value(K_NULL);
  a[4] = off ? make_typed(napi_int32_array, off, no) : new_value(K_NULL);
  a[5] = new_value(K_OBJ);
  static const char* keys[5] = {"doSample", "temperature", "topK", "topP", "repetitionPenalty"};
  for (int i = 0; i < 5; i++)
    if (opts_mask & (1 << i)) {
      napi_value v;
      if (i == 0) {
        v = new_value(K_BOOL);
        v->b = opts[0] != 0.0;
      } else {
        v = make_number(opts[i]);
      }
      set_prop(a[5], keys[i], v);
    }
  a[6] = u ? make_typed(napi_float64_array, u, nu) : new_value(K_NULL);
}

static int read_ids(napi_value r, int32_t* out, size_t cap, char* err, size_t errlen) {
  if (!r || r->kind != K_TA || r->tt != napi_int32_array || r->len > cap) {
    snprintf(err, errlen, "result is not an Int32Array of at most %zu ids", cap);
    return -1;
  }
  memcpy(out, r->data, r->len * 4);
  return (int)r->len;
}

/* sample(...): the number of ids written to out, or -1 with the thrown error in err. */
int fake_sample(float* logits, size_t nlog, double B, double V, int32_t* hist, size_t nh, int32_t* off, size_t no,
                const double* opts, int opts_mask, double* u, size_t nu, int32_t* out, size_t cap, char* err,
                size_t errlen) {
  napi_value a[7];
  make_args(a, logits, nlog, B, V, hist, nh, off, no, opts, opts_mask, u, nu);
  napi_value r = call_export("sample", 7, a, err, errlen);
  return r ? read_ids(r, out, cap, err, errlen) : -1;
}

/* sampleAsync(...): the promise, or NULL with the thrown error in err. */
void* fake_sample_async(float* logits, size_t nlog, double B, double V, int32_t* hist, size_t nh, int32_t* off,
                        size_t no, const double* opts, int opts_mask, double* u, size_t nu, char* err,
                        size_t errlen) {
  napi_value a[7];
  make_args(a, logits, nlog, B, V, hist, nh, off, no, opts, opts_mask, u, nu);
  napi_value r = call_export("sampleAsync", 7, a, err, errlen);
  if (r && r->kind != K_PROMISE) {
    snprintf(err, errlen, "sampleAsync returned no promise");
    return NULL;
  }
  return r;
}

/* A promise's state: the number of ids when resolved (copied to out), -1
 * rejected (the error's message in err), -2 pending. */
int fake_promise(void* p, int32_t* out, size_t cap, char* err, size_t errlen) {
  napi_value v = (napi_value)p;
  if (v->state == P_PENDING) return -2;
  if (v->state == P_REJECTED) {
    snprintf(err, errlen, "%s", v->settled && v->settled->kind == K_ERROR ? v->settled->str : "(not an Error)");
    return -1;
  }
  return read_ids(v->settled, out, cap, err, errlen);
}

/* status().abi, or -1. */
int fake_status_abi(void) {
  char err[64];
  napi_value r = call_export("status", 0, NULL, err, sizeof err);
  napi_value abi = r ? get_prop(r, "abi") : NULL;
  return abi && abi->kind == K_NUM ? (int)abi->num : -1;
}
