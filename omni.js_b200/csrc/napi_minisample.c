/*
 * Node-API shim: exposes libminisample to mini.js as `addon.sample(...)`.
 *
 *   sample(logits: Float32Array, B: number, V: number,
 *          history: Int32Array | null, historyOffsets: Int32Array | null,
 *          opts: {doSample, temperature, topK, topP, repetitionPenalty},
 *          uniforms: Float64Array | null) -> Int32Array(B)
 *   sampleAsync(...same arguments...) -> Promise<Int32Array(B)>
 *   status() -> {abi: number}   (the library's MS_ABI_VERSION)
 *
 * `opts` is the object normalizeOptions returns (src/generation.js:57-68).
 * `sample` is synchronous, like generateTokens (src/generation.js:97-114).
 * `sampleAsync` copies its inputs, samples on a libuv worker thread and
 * settles the promise on the JS thread, so generateAsync
 * (src/generation.js:121-142) does not block the event loop; async calls share
 * one context of their own, one at a time (a context belongs to one host
 * thread at a time).
 * Every libminisample error becomes a thrown JS Error carrying
 * ms_last_error(); nothing falls back to the JS sampler.
 *
 * Build (on a machine with Node headers):
 *   cc -O2 -fPIC -shared -I<node>/include/node -Iinclude \
 *      omni.js_b200/csrc/napi_minisample.c -Lomni.js_b200/minisample -lminisample \
 *      -Wl,-rpath,'$ORIGIN' -o omni.js_b200/minisample/minisample.node
 * This machine has no Node runtime or headers, so the shim is not built here;
 * the ctypes binding in omni.js_b200/minisample/_native.py drives the same ABI.
 */
#include <node_api.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../../include/minisample.h"

static ms_ctx* g_ctx = NULL;

#define NAPI_OK(env, call)                                            \
  do {                                                                \
    if ((call) != napi_ok) {                                          \
      napi_throw_error((env), NULL, "minisample: N-API call failed"); \
      return NULL;                                                    \
    }                                                                 \
  } while (0)

static int get_number(napi_env env, napi_value obj, const char* key, double* out) {
  napi_value v;
  bool has = false;
  if (napi_has_named_property(env, obj, key, &has) != napi_ok || !has) return 0;
  if (napi_get_named_property(env, obj, key, &v) != napi_ok) return 0;
  napi_valuetype t;
  napi_typeof(env, v, &t);
  if (t == napi_boolean) {
    bool b;
    napi_get_value_bool(env, v, &b);
    *out = b ? 1.0 : 0.0;
    return 1;
  }
  if (t != napi_number) return 0;
  return napi_get_value_double(env, v, out) == napi_ok;
}

static void* typed_data(napi_env env, napi_value v, napi_typedarray_type want, size_t* len) {
  bool is = false;
  if (napi_is_typedarray(env, v, &is) != napi_ok || !is) return NULL;
  napi_typedarray_type t;
  void* data = NULL;
  napi_value ab;
  size_t off = 0;
  if (napi_get_typedarray_info(env, v, &t, len, &data, &ab, &off) != napi_ok || t != want) return NULL;
  return data;
}

/* One sampling call.  A synchronous call reads the JS arrays in place; an
 * asynchronous one owns copies (`own`), since the JS arrays may change before
 * the worker runs. */
typedef struct sample_job {
  const float* logits;
  int64_t B, V;
  const int32_t* hist; /* NULL: no history */
  int64_t* off;        /* always owned: the Int32Array offsets widened */
  const double* u;     /* NULL: greedy */
  ms_params p;
  int32_t* out;        /* owned */
  int own;
  int rc;
  char err[512];
  napi_async_work work;
  napi_deferred deferred;
} sample_job;

static void job_free(sample_job* j) {
  if (!j) return;
  if (j->own) {
    free((void*)j->logits);
    free((void*)j->hist);
    free((void*)j->u);
  }
  free(j->off);
  free(j->out);
  free(j);
}

/* A malloc'd copy of n bytes of src (n may be 0); NULL when out of memory. */
static void* dup_bytes(const void* src, size_t n) {
  void* d = malloc(n ? n : 1);
  if (d && n) memcpy(d, src, n);
  return d;
}

/* Parses sample(...)'s seven arguments into a new job (NULL after throwing).
 * copy != 0: the job owns copies of the input arrays. */
static sample_job* parse_job(napi_env env, napi_callback_info info, int copy) {
  size_t argc = 7;
  napi_value a[7];
  if (napi_get_cb_info(env, info, &argc, a, NULL, NULL) != napi_ok || argc < 7) {
    napi_throw_type_error(env, NULL, "minisample.sample: 7 arguments expected");
    return NULL;
  }
  size_t nlog = 0, nh = 0, no = 0, nu = 0;
  const float* logits = (const float*)typed_data(env, a[0], napi_float32_array, &nlog);
  double Bd = 0, Vd = 0;
  napi_get_value_double(env, a[1], &Bd);
  napi_get_value_double(env, a[2], &Vd);
  const int64_t B = (int64_t)Bd, V = (int64_t)Vd;
  if (!logits || B < 1 || V < 1 || (int64_t)nlog < B * V) {
    napi_throw_type_error(env, NULL, "minisample.sample: logits must be a Float32Array of B*V");
    return NULL;
  }
  const int32_t* hist = (const int32_t*)typed_data(env, a[3], napi_int32_array, &nh);
  const int32_t* off32 = (const int32_t*)typed_data(env, a[4], napi_int32_array, &no);
  const double* u = (const double*)typed_data(env, a[6], napi_float64_array, &nu);
  if (u && (int64_t)nu < B) {
    napi_throw_type_error(env, NULL, "minisample.sample: uniforms must have B entries");
    return NULL;
  }
  sample_job* j = (sample_job*)calloc(1, sizeof(sample_job));
  if (!j) {
    napi_throw_error(env, NULL, "minisample: out of host memory");
    return NULL;
  }
  j->B = B;
  j->V = V;
  j->logits = logits; /* borrowed (own == 0) until the copies below */
  j->u = u;
  if (hist && off32) {
    if ((int64_t)no != B + 1) {
      job_free(j);
      napi_throw_type_error(env, NULL, "minisample.sample: historyOffsets must have B+1 entries");
      return NULL;
    }
    /* offsets must index inside `history`: off[0] >= 0, ascending, off[B] <= its length */
    int ok = off32[0] >= 0 && (int64_t)off32[B] <= (int64_t)nh;
    for (int64_t i = 0; ok && i < B; i++) ok = off32[i + 1] >= off32[i];
    if (!ok) {
      job_free(j);
      napi_throw_range_error(env, NULL,
                             "minisample.sample: historyOffsets must ascend from >= 0 to <= history.length");
      return NULL;
    }
    j->hist = hist;
    j->off = (int64_t*)malloc(sizeof(int64_t) * (size_t)(B + 1));
    if (!j->off) {
      job_free(j);
      napi_throw_error(env, NULL, "minisample: out of host memory");
      return NULL;
    }
    for (int64_t i = 0; i <= B; i++) j->off[i] = off32[i];
  }
  double v;
  j->p.do_sample = get_number(env, a[5], "doSample", &v) ? (v != 0.0) : 1;
  j->p.temperature = get_number(env, a[5], "temperature", &v) ? v : 1.0;
  j->p.top_k = get_number(env, a[5], "topK", &v) ? (int32_t)v : 50;
  j->p.top_p = get_number(env, a[5], "topP", &v) ? v : 0.95;
  j->p.repetition_penalty = get_number(env, a[5], "repetitionPenalty", &v) ? v : 1.0;
  j->out = (int32_t*)malloc(sizeof(int32_t) * (size_t)B);
  int ok = j->out != NULL;
  if (copy) {
    /* borrowed pointers are replaced one by one, so job_free frees only copies */
    const float* l = j->logits;
    const double* uu = j->u;
    const int32_t* h = j->hist;
    j->logits = NULL;
    j->u = NULL;
    j->hist = NULL;
    j->own = 1;
    ok = ok && (j->logits = (const float*)dup_bytes(l, sizeof(float) * (size_t)(B * V))) != NULL;
    ok = ok && (!uu || (j->u = (const double*)dup_bytes(uu, sizeof(double) * (size_t)B)) != NULL);
    ok = ok && (!h || (j->hist = (const int32_t*)dup_bytes(h, sizeof(int32_t) * nh)) != NULL);
  }
  if (!ok) {
    job_free(j);
    napi_throw_error(env, NULL, "minisample: out of host memory");
    return NULL;
  }
  return j;
}

static void run_job(ms_ctx* ctx, sample_job* j) {
  j->rc = ms_sample(ctx, j->logits, j->B, j->V, j->V, j->off ? j->hist : NULL, j->off, &j->p, j->u, j->out, NULL,
                    MS_HOST_PTRS, NULL);
  if (j->rc != MS_OK) snprintf(j->err, sizeof j->err, "%s", ms_last_error(ctx));
}

static napi_value ids_array(napi_env env, const sample_job* j) {
  napi_value ab, out;
  void* outp = NULL;
  if (napi_create_arraybuffer(env, (size_t)j->B * 4, &outp, &ab) != napi_ok ||
      napi_create_typedarray(env, napi_int32_array, (size_t)j->B, ab, 0, &out) != napi_ok)
    return NULL;
  memcpy(outp, j->out, (size_t)j->B * 4);
  return out;
}

static napi_value js_sample(napi_env env, napi_callback_info info) {
  if (!g_ctx && ms_create(&g_ctx, NULL, 0) != MS_OK) {
    napi_throw_error(env, NULL, "minisample: no CUDA device for the 'cuda' sampler backend");
    return NULL;
  }
  sample_job* j = parse_job(env, info, 0);
  if (!j) return NULL;
  run_job(g_ctx, j);
  napi_value out = NULL;
  if (j->rc != MS_OK) napi_throw_error(env, NULL, j->err);
  else if (!(out = ids_array(env, j))) napi_throw_error(env, NULL, "minisample: cannot allocate the result");
  job_free(j);
  return out;
}

/* ---- sampleAsync: the same call on a libuv worker thread */
static pthread_mutex_t g_async_mu = PTHREAD_MUTEX_INITIALIZER;
static ms_ctx* g_async_ctx = NULL;

static void async_execute(napi_env env, void* data) {  /* worker thread: no N-API calls here */
  (void)env;
  sample_job* j = (sample_job*)data;
  pthread_mutex_lock(&g_async_mu);
  if (!g_async_ctx && ms_create(&g_async_ctx, NULL, 0) != MS_OK) {
    g_async_ctx = NULL;
    j->rc = MS_ERR_STATE;
    snprintf(j->err, sizeof j->err, "minisample: no CUDA device for the 'cuda' sampler backend");
  } else {
    run_job(g_async_ctx, j);
  }
  pthread_mutex_unlock(&g_async_mu);
}

static void async_complete(napi_env env, napi_status status, void* data) {  /* JS thread */
  sample_job* j = (sample_job*)data;
  napi_value result = NULL, msg = NULL;
  if (status == napi_ok && j->rc == MS_OK && (result = ids_array(env, j))) {
    napi_resolve_deferred(env, j->deferred, result);
  } else {
    const char* text = j->rc != MS_OK ? j->err : "minisample: asynchronous sample failed";
    napi_create_string_utf8(env, text, NAPI_AUTO_LENGTH, &msg);
    napi_create_error(env, NULL, msg, &result);
    napi_reject_deferred(env, j->deferred, result);
  }
  napi_delete_async_work(env, j->work);
  job_free(j);
}

static napi_value js_sample_async(napi_env env, napi_callback_info info) {
  sample_job* j = parse_job(env, info, 1);
  if (!j) return NULL;
  napi_value promise, name;
  if (napi_create_promise(env, &j->deferred, &promise) != napi_ok ||
      napi_create_string_utf8(env, "minisample.sampleAsync", NAPI_AUTO_LENGTH, &name) != napi_ok ||
      napi_create_async_work(env, NULL, name, async_execute, async_complete, j, &j->work) != napi_ok ||
      napi_queue_async_work(env, j->work) != napi_ok) {
    if (j->work) napi_delete_async_work(env, j->work);
    job_free(j);
    napi_throw_error(env, NULL, "minisample: cannot queue the asynchronous sample");
    return NULL;
  }
  return promise;
}

static napi_value js_status(napi_env env, napi_callback_info info) {
  (void)info;
  napi_value o, abi;
  NAPI_OK(env, napi_create_object(env, &o));
  NAPI_OK(env, napi_create_int32(env, ms_version(), &abi));
  NAPI_OK(env, napi_set_named_property(env, o, "abi", abi));
  return o;
}

static napi_value init(napi_env env, napi_value exports) {
  napi_property_descriptor d[] = {
      {"sample", NULL, js_sample, NULL, NULL, NULL, napi_default, NULL},
      {"sampleAsync", NULL, js_sample_async, NULL, NULL, NULL, napi_default, NULL},
      {"status", NULL, js_status, NULL, NULL, NULL, napi_default, NULL},
  };
  napi_define_properties(env, exports, 3, d);
  return exports;
}

NAPI_MODULE(NODE_GYP_MODULE_NAME, init)
