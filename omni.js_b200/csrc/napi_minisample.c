/*
 * Node-API shim: exposes libminisample to mini.js as `addon.sample(...)`.
 *
 *   sample(logits: Float32Array, B: number, V: number,
 *          history: Int32Array | null, historyOffsets: Int32Array | null,
 *          opts: {doSample, temperature, topK, topP, repetitionPenalty},
 *          uniforms: Float64Array | null) -> Int32Array(B)
 *   status() -> {abi: number}   (the library's MS_ABI_VERSION)
 *
 * `opts` is the object normalizeOptions returns (src/generation.js:57-68).
 * The call is synchronous, like generateTokens (src/generation.js:97-114).
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
#include <stdint.h>
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

static napi_value js_sample(napi_env env, napi_callback_info info) {
  size_t argc = 7;
  napi_value a[7];
  NAPI_OK(env, napi_get_cb_info(env, info, &argc, a, NULL, NULL));
  if (argc < 7) {
    napi_throw_type_error(env, NULL, "minisample.sample: 7 arguments expected");
    return NULL;
  }
  if (!g_ctx && ms_create(&g_ctx, NULL, 0) != MS_OK) {
    napi_throw_error(env, NULL, "minisample: no CUDA device for the 'cuda' sampler backend");
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
  int64_t* off = NULL;
  if (hist && off32) {
    if ((int64_t)no != B + 1) {
      napi_throw_type_error(env, NULL, "minisample.sample: historyOffsets must have B+1 entries");
      return NULL;
    }
    /* offsets must index inside `history`: off[0] >= 0, ascending, off[B] <= its length */
    int ok = off32[0] >= 0 && (int64_t)off32[B] <= (int64_t)nh;
    for (int64_t i = 0; ok && i < B; i++) ok = off32[i + 1] >= off32[i];
    if (!ok) {
      napi_throw_range_error(env, NULL,
                             "minisample.sample: historyOffsets must ascend from >= 0 to <= history.length");
      return NULL;
    }
    off = (int64_t*)malloc(sizeof(int64_t) * (size_t)(B + 1));
    if (!off) {
      napi_throw_error(env, NULL, "minisample: out of host memory");
      return NULL;
    }
    for (int64_t i = 0; i <= B; i++) off[i] = off32[i];
  }
  ms_params p;
  double v;
  p.do_sample = get_number(env, a[5], "doSample", &v) ? (v != 0.0) : 1;
  p.temperature = get_number(env, a[5], "temperature", &v) ? v : 1.0;
  p.top_k = get_number(env, a[5], "topK", &v) ? (int32_t)v : 50;
  p.top_p = get_number(env, a[5], "topP", &v) ? v : 0.95;
  p.repetition_penalty = get_number(env, a[5], "repetitionPenalty", &v) ? v : 1.0;
  const double* u = (const double*)typed_data(env, a[6], napi_float64_array, &nu);
  if (u && (int64_t)nu < B) {
    free(off);
    napi_throw_type_error(env, NULL, "minisample.sample: uniforms must have B entries");
    return NULL;
  }
  napi_value ab, out;
  void* outp = NULL;
  if (napi_create_arraybuffer(env, (size_t)B * 4, &outp, &ab) != napi_ok ||
      napi_create_typedarray(env, napi_int32_array, (size_t)B, ab, 0, &out) != napi_ok) {
    free(off);
    napi_throw_error(env, NULL, "minisample: cannot allocate the result");
    return NULL;
  }
  const int rc = ms_sample(g_ctx, logits, B, V, V, off ? hist : NULL, off, &p, u, (int32_t*)outp, NULL,
                           MS_HOST_PTRS, NULL);
  free(off);
  if (rc != MS_OK) {
    napi_throw_error(env, NULL, ms_last_error(g_ctx));
    return NULL;
  }
  return out;
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
      {"status", NULL, js_status, NULL, NULL, NULL, napi_default, NULL},
  };
  napi_define_properties(env, exports, 2, d);
  return exports;
}

NAPI_MODULE(NODE_GYP_MODULE_NAME, init)
