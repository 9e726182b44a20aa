// libminisample C ABI (include/minisample.h): contexts, scratch, host staging,
// row sharding over the context's devices, and error reporting.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <algorithm>
#include <array>
#include <vector>

#include "ms_device.cuh"

namespace ms {
cudaError_t launch_sample(const Args& A, cudaStream_t stream, cudaEvent_t* ev, int64_t* launched);
cudaError_t launch_shard(const Args& A, cudaStream_t stream);
cudaError_t launch_merge(const Args& A, cudaStream_t stream);
cudaError_t launch_exp(const double* x, double* y, int64_t n, cudaStream_t stream);
cudaError_t launch_history_append(int32_t* hist, int32_t* len, int64_t B, int64_t cap, const int32_t* ids,
                                  cudaStream_t stream);
size_t finalize_smem_bytes();
}  // namespace ms

namespace {

struct DevState {
  int device = 0;
  cudaStream_t stream = nullptr;
  void* scratch = nullptr;  // stats, candidates, penalty bitmap
  size_t scratch_bytes = 0;
  void* io = nullptr;       // device copies of host arguments
  size_t io_bytes = 0;
  int32_t* status = nullptr;    // device status word: the epoch of the last call whose wait ran out
  int32_t epoch = 0;            // epoch of the last call launched on this device (never 0 once used)
  std::vector<int64_t> host_offs;  // host staging of the rebased history offsets (lives until the call's sync)
  int32_t* counters = nullptr;  // per-row chunk counters; kernels leave them at zero
  int64_t counters_cap = 0;
  std::vector<std::array<cudaEvent_t, 3>> prof_pending;  // MS_PROFILE calls not yet read
  std::vector<std::array<cudaEvent_t, 3>> prof_free;
  int64_t launches = 0;  // kernels launched on this device
};

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

struct Plan {
  int mode = ms::kGreedy;
  int use_pen = 0;
  int temper = 0;
  float a = 0.f;
  int k = 0;
  int kw = 1;
  int use_topp = 0;
  int n_chunks = 1;
};

Plan make_plan(int64_t V, const ms_params* p, bool have_hist) {
  Plan P;
  const double T = p->temperature;
  const bool greedy = !p->do_sample || T <= 0.0001;
  const double pen = p->repetition_penalty;
  P.use_pen = (have_hist && pen != 0.0 && !std::isnan(pen) && pen != 1.0) ? 1 : 0;
  P.temper = (T != 1.0) ? 1 : 0;
  P.a = (float)(1.4426950408889634 / T);
  P.k = p->top_k;
  P.use_topp = (p->top_p != 0.0 && p->top_p < 1.0) ? 1 : 0;
  P.n_chunks = (int)((V + ms::kChunk - 1) / ms::kChunk);
  if (greedy) {
    P.mode = ms::kGreedy;
  } else if (P.k > 0 && P.k < V && P.k <= ms::kKmax) {
    P.mode = ms::kTopK;
  } else {
    P.mode = ms::kFull;
  }
  // every warp's kw-th largest thread maximum; warps * kw >= keff
  const int warps = ms::kThreads / 32;
  const int keff = (P.mode == ms::kTopK) ? P.k : ms::kKSum;
  P.kw = (keff + warps - 1) / warps;
  if (P.kw < 1) P.kw = 1;
  if (P.kw > 32) P.kw = 32;
  return P;
}

// The Args fields that follow from the params and the plan.
ms::Args param_args(const Plan& P, const ms_params* p) {
  ms::Args A;
  memset(&A, 0, sizeof A);
  A.pen = p->repetition_penalty;
  A.rpen = 1.0 / p->repetition_penalty;
  A.use_pen = P.use_pen;
  A.mode = P.mode;
  A.T = p->temperature;
  A.rT = 1.0 / p->temperature;
  A.temper = P.temper;
  A.a = P.a;
  A.k = P.k;
  A.kw = P.kw;
  A.use_topp = P.use_topp;
  A.top_p = p->top_p;
  A.n_chunks = P.n_chunks;
  A.ksum = ms::kKSum;
  return A;
}

struct ScratchLayout {
  size_t stats = 0, cands = 0, penbits = 0, total = 0;
  // whole-vocabulary rows: chunk histograms, plans, extraction lists
  size_t h_cnt = 0, h_mass = 0, plan = 0, lists = 0, list_cnt = 0;
};

ScratchLayout scratch_layout(int64_t B, int64_t V, const Plan& P) {
  ScratchLayout L;
  size_t off = 0;
  L.stats = off;
  off = align_up(off + (size_t)B * P.n_chunks * sizeof(ms::ChunkStat), 256);
  L.cands = off;
  if (P.mode != ms::kGreedy) off = align_up(off + (size_t)B * P.n_chunks * ms::kCap * sizeof(ms::Cand), 256);
  L.penbits = off;
  if (P.use_pen && P.mode != ms::kGreedy) off = align_up(off + (size_t)B * ((V + 31) / 32) * 4, 256);
  if (P.mode == ms::kFull) {
    L.h_cnt = off;
    off = align_up(off + (size_t)B * P.n_chunks * ms::kNB * sizeof(uint16_t), 256);
    L.h_mass = off;
    off = align_up(off + (size_t)B * P.n_chunks * ms::kNB * sizeof(double), 256);
    L.plan = off;
    off = align_up(off + (size_t)B * sizeof(ms::NucPlan), 256);
    L.lists = off;
    off = align_up(off + (size_t)B * 2 * ms::kListCap * sizeof(ms::Cand), 256);
    L.list_cnt = off;
    off = align_up(off + (size_t)B * 4 * sizeof(int32_t), 256);
  }
  L.total = off;
  return L;
}

}  // namespace

struct ms_ctx {
  std::vector<DevState> devs;
  std::string err = "no error";
  long long inject_wait = 0;   // ms_debug_inject(MS_INJECT_WAIT): cycles, next call only
  bool inject_alloc = false;   // ms_debug_inject(MS_INJECT_ALLOC): fail the next allocation
};

static int fail(ms_ctx* c, int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (c) c->err = buf;
  return code;
}

#define MS_CUDA(ctx, call)                                                                      \
  do {                                                                                          \
    cudaError_t e_ = (call);                                                                    \
    if (e_ != cudaSuccess)                                                                      \
      return fail(ctx, e_ == cudaErrorMemoryAllocation ? MS_ERR_OOM : MS_ERR_CUDA, "%s: %s (%s:%d)", \
                  #call, cudaGetErrorString(e_), __FILE__, __LINE__);                           \
  } while (0)

// Every device allocation of a context goes through here (so a test can make
// one fail, ms_debug_inject).
static int dev_alloc(ms_ctx* ctx, void** p, size_t sz) {
  if (ctx->inject_alloc) {
    ctx->inject_alloc = false;
    *p = nullptr;
    return fail(ctx, MS_ERR_OOM, "cudaMalloc(%zu bytes): out of memory (injected)", sz);
  }
  MS_CUDA(ctx, cudaMalloc(p, sz));
  return MS_OK;
}

static int ensure(ms_ctx* ctx, void** buf, size_t* have, size_t need) {
  if (*have >= need) return MS_OK;
  if (*buf) {
    cudaFree(*buf);
    *buf = nullptr;
    *have = 0;
  }
  size_t sz = need + need / 8;
  int rc = dev_alloc(ctx, buf, sz);
  if (rc) return rc;
  *have = sz;
  return MS_OK;
}

// The status word and the per-row counters of device state s (allocated once,
// grown with B).
static int ensure_state(ms_ctx* ctx, DevState& s, int64_t B) {
  if (!s.status) {
    int rc = dev_alloc(ctx, (void**)&s.status, 256);
    if (rc) return rc;
    MS_CUDA(ctx, cudaMemset(s.status, 0, 256));
  }
  if (s.counters_cap < B) {
    if (s.counters) cudaFree(s.counters);
    s.counters = nullptr;
    s.counters_cap = 0;
    const int64_t cap = B + B / 8 + 64;
    int rc = dev_alloc(ctx, (void**)&s.counters, (size_t)cap * 4);
    if (rc) return rc;
    MS_CUDA(ctx, cudaMemset(s.counters, 0, (size_t)cap * 4));
    s.counters_cap = cap;
  }
  return MS_OK;
}

static int32_t next_epoch(DevState& s) {
  s.epoch = (s.epoch >= INT32_MAX - 1) ? 1 : s.epoch + 1;
  return s.epoch;
}

// Did a wait of the call with this epoch run out?  (after a stream sync)
static int read_status(ms_ctx* ctx, DevState& s, const char* who) {
  int32_t status = 0;
  cudaError_t e = cudaMemcpy(&status, s.status, sizeof status, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return fail(ctx, MS_ERR_CUDA, "%s: %s", who, cudaGetErrorString(e));
  if (status == s.epoch) return fail(ctx, MS_ERR_TIMEOUT, "%s: a kernel wait timed out", who);
  return MS_OK;
}

extern "C" {

int ms_version(void) { return MS_ABI_VERSION; }

int ms_create(ms_ctx** out, const int* devices, int n_devices) {
  if (!out) return MS_ERR_ARG;
  *out = nullptr;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count < 1) return MS_ERR_STATE;
  ms_ctx* c = new ms_ctx();
  std::vector<int> ids;
  if (!devices || n_devices <= 0) {
    int d = 0;
    cudaGetDevice(&d);
    ids.push_back(d);
  } else {
    for (int i = 0; i < n_devices; i++) {
      if (devices[i] < 0 || devices[i] >= count) {
        delete c;
        return MS_ERR_ARG;
      }
      ids.push_back(devices[i]);
    }
  }
  int prev = 0;
  cudaGetDevice(&prev);
  for (int d : ids) {
    DevState s;
    s.device = d;
    if (cudaSetDevice(d) != cudaSuccess || cudaStreamCreateWithFlags(&s.stream, cudaStreamNonBlocking) != cudaSuccess) {
      for (auto& o : c->devs) { cudaSetDevice(o.device); cudaStreamDestroy(o.stream); }
      cudaSetDevice(prev);
      delete c;
      return MS_ERR_CUDA;
    }
    c->devs.push_back(s);
  }
  cudaSetDevice(prev);
  *out = c;
  return MS_OK;
}

int ms_destroy(ms_ctx* c) {
  if (!c) return MS_ERR_ARG;
  int prev = 0;
  cudaGetDevice(&prev);
  for (auto& s : c->devs) {
    cudaSetDevice(s.device);
    if (s.stream) { cudaStreamSynchronize(s.stream); cudaStreamDestroy(s.stream); }
    if (s.scratch) cudaFree(s.scratch);
    if (s.status) cudaFree(s.status);
    if (s.counters) cudaFree(s.counters);
    for (auto& e3 : s.prof_pending) for (auto e : e3) cudaEventDestroy(e);
    for (auto& e3 : s.prof_free) for (auto e : e3) cudaEventDestroy(e);
    if (s.io) cudaFree(s.io);
  }
  cudaSetDevice(prev);
  delete c;
  return MS_OK;
}

const char* ms_last_error(ms_ctx* c) { return c ? c->err.c_str() : "null context"; }

int ms_profile_read(ms_ctx* c, double* stream_ms, double* finalize_ms, int64_t* calls) {
  if (!c) return MS_ERR_ARG;
  double a = 0.0, b = 0.0;
  int64_t n = 0;
  int prev = 0;
  cudaGetDevice(&prev);
  for (auto& s : c->devs) {
    cudaSetDevice(s.device);
    for (auto& e3 : s.prof_pending) {
      float t01 = 0.f, t12 = 0.f;
      if (cudaEventSynchronize(e3[2]) != cudaSuccess || cudaEventElapsedTime(&t01, e3[0], e3[1]) != cudaSuccess ||
          cudaEventElapsedTime(&t12, e3[1], e3[2]) != cudaSuccess) {
        cudaSetDevice(prev);
        return fail(c, MS_ERR_CUDA, "ms_profile_read: event timing failed");
      }
      a += t01;
      b += t12;
      n++;
      s.prof_free.push_back(e3);
    }
    s.prof_pending.clear();
  }
  cudaSetDevice(prev);
  if (stream_ms) *stream_ms = a;
  if (finalize_ms) *finalize_ms = b;
  if (calls) *calls = n;
  return MS_OK;
}

int ms_launch_count(ms_ctx* c, int64_t* kernels) {
  if (!c || !kernels) return MS_ERR_ARG;
  int64_t n = 0;
  for (auto& s : c->devs) n += s.launches;
  *kernels = n;
  return MS_OK;
}

int ms_debug_inject(ms_ctx* c, int what, int64_t arg) {
  if (!c || arg < 0) return MS_ERR_ARG;
  if (what == MS_INJECT_WAIT) c->inject_wait = (long long)arg;
  else if (what == MS_INJECT_ALLOC) c->inject_alloc = arg != 0;
  else return fail(c, MS_ERR_ARG, "ms_debug_inject: unknown injection %d", what);
  return MS_OK;
}

int ms_history_append(ms_ctx* c, int32_t* hist, int32_t* len, int64_t B, int64_t cap, const int32_t* ids,
                      void* stream) {
  if (!c) return MS_ERR_ARG;
  if (B < 0 || cap < 1 || cap > INT32_MAX) return fail(c, MS_ERR_ARG, "ms_history_append: bad B / cap");
  if (B == 0) return MS_OK;
  if (!hist || !len || !ids) return fail(c, MS_ERR_ARG, "ms_history_append: NULL pointer");
  if ((uint64_t)B * (uint64_t)cap > (uint64_t)INT64_MAX / 4) return fail(c, MS_ERR_ARG, "ms_history_append: too large");
  DevState& s = c->devs[0];
  MS_CUDA(c, cudaSetDevice(s.device));
  cudaStream_t st = stream ? (cudaStream_t)stream : s.stream;
  MS_CUDA(c, ms::launch_history_append(hist, len, B, cap, ids, st));
  s.launches += 1;
  return MS_OK;
}

int ms_debug_exp(const double* x, double* y, int64_t n, void* stream) {
  if (n < 0 || (n > 0 && (!x || !y))) return MS_ERR_ARG;
  if (n == 0) return MS_OK;
  return ms::launch_exp(x, y, n, (cudaStream_t)stream) == cudaSuccess ? MS_OK : MS_ERR_CUDA;
}

int ms_scratch_bytes(int64_t B, int64_t V, const ms_params* params, int64_t* out_bytes) {
  if (!params || !out_bytes || B < 0 || V < 1) return MS_ERR_ARG;
  const Plan P = make_plan(V, params, true);
  *out_bytes = (int64_t)scratch_layout(B, V, P).total + (int64_t)align_up((size_t)B * 4, 256) + 256;
  return MS_OK;
}

}  // extern "C"

// Launch one [B, V] slice on device state s; every pointer is device memory.
static int run_device(ms_ctx* ctx, DevState& s, const float* logits, int64_t B, int64_t V, int64_t ld,
                      const int32_t* hist, const int64_t* hist_off, const ms_params* p, const double* u,
                      int32_t* out_ids, const ms_diag* diag, cudaStream_t stream, bool profile) {
  const Plan P = make_plan(V, p, hist != nullptr && hist_off != nullptr);
  const ScratchLayout L = scratch_layout(B, V, P);
  int rc = ensure(ctx, &s.scratch, &s.scratch_bytes, L.total);
  if (rc) return rc;
  rc = ensure_state(ctx, s, B);
  if (rc) return rc;
  char* base = (char*)s.scratch;
  ms::Args A;
  memset(&A, 0, sizeof A);
  A.logits = logits;
  A.ld = ld;
  A.B = (int32_t)B;
  A.V = (int32_t)V;
  A.hist = hist;
  A.hist_off = hist_off;
  A.pen = p->repetition_penalty;
  A.rpen = 1.0 / p->repetition_penalty;
  A.use_pen = P.use_pen;
  A.mode = P.mode;
  A.T = p->temperature;
  A.rT = 1.0 / p->temperature;
  A.temper = P.temper;
  A.a = P.a;
  A.k = P.k;
  A.kw = P.kw;
  A.use_topp = P.use_topp;
  A.top_p = p->top_p;
  A.u = u;
  A.n_chunks = P.n_chunks;
  A.stats = (ms::ChunkStat*)(base + L.stats);
  A.cands = (ms::Cand*)(base + L.cands);
  A.penbits = (P.use_pen && P.mode != ms::kGreedy) ? (uint32_t*)(base + L.penbits) : nullptr;
  if (P.mode == ms::kFull) {
    // counts only for rank selection (top_k above the candidate path)
    A.h_cnt = (P.k > 0 && P.k < V) ? (uint16_t*)(base + L.h_cnt) : nullptr;
    A.h_mass = (double*)(base + L.h_mass);
    A.plan = (ms::NucPlan*)(base + L.plan);
    A.lists = (ms::Cand*)(base + L.lists);
    A.list_cnt = (int32_t*)(base + L.list_cnt);
  }
  A.status = s.status;
  A.epoch = next_epoch(s);
  A.test_wait = ctx->inject_wait;
  ctx->inject_wait = 0;
  A.row_count = s.counters;
  A.ksum = ms::kKSum;
  A.out_ids = out_ids;
  if (diag) {
    A.d_pen = diag->pen_logits;
    A.pen_ld = diag->pen_ld;
    A.cand_cap = diag->cand_cap;
    A.d_cand_ids = diag->cand_cap > 0 ? diag->cand_ids : nullptr;
    A.d_cand_probs = diag->cand_cap > 0 ? diag->cand_probs : nullptr;
    A.d_n_cand = diag->n_cand;
    A.d_row_max = diag->row_max;
    A.d_row_sum = diag->row_sum;
    A.d_total = diag->total;
    A.d_row_flags = diag->row_flags;
  }
  if (P.mode != ms::kGreedy && !u) return fail(ctx, MS_ERR_ARG, "ms_sample: sampled rows need u[B]");
  cudaEvent_t* ev = nullptr;
  if (profile) {
    if (s.prof_free.empty()) {
      std::array<cudaEvent_t, 3> e3;
      for (auto& e : e3) MS_CUDA(ctx, cudaEventCreate(&e));
      s.prof_free.push_back(e3);
    }
    s.prof_pending.push_back(s.prof_free.back());
    s.prof_free.pop_back();
    ev = s.prof_pending.back().data();
  }
  MS_CUDA(ctx, ms::launch_sample(A, stream, ev, &s.launches));
  return MS_OK;
}

extern "C" int ms_sample(ms_ctx* ctx, const float* logits, int64_t B, int64_t V, int64_t ld,
                         const int32_t* hist, const int64_t* hist_off, const ms_params* params,
                         const double* u, int32_t* out_ids, ms_diag* diag, int flags, void* stream) {
  if (!ctx) return MS_ERR_ARG;
  if (!params) return fail(ctx, MS_ERR_ARG, "ms_sample: params is NULL");
  if (B < 0) return fail(ctx, MS_ERR_ARG, "ms_sample: B < 0");
  if (V < 1 || V > (int64_t)65535 * ms::kChunk) return fail(ctx, MS_ERR_ARG, "ms_sample: V out of range");
  if (ld < V) return fail(ctx, MS_ERR_ARG, "ms_sample: ld < V");
  if (B == 0) return MS_OK;
  if (!logits || !out_ids) return fail(ctx, MS_ERR_ARG, "ms_sample: logits/out_ids is NULL");
  if (hist_off != nullptr && hist == nullptr)
    return fail(ctx, MS_ERR_ARG, "ms_sample: hist_off given without hist");
  if (hist_off == nullptr) hist = nullptr;
  const bool host = (flags & MS_HOST_PTRS) != 0, dev = (flags & MS_DEVICE_PTRS) != 0;
  if (host == dev) return fail(ctx, MS_ERR_ARG, "ms_sample: pass exactly one of MS_HOST_PTRS / MS_DEVICE_PTRS");
  if (diag && diag->cand_cap < 0) return fail(ctx, MS_ERR_ARG, "ms_sample: diag->cand_cap < 0");
  if (diag && diag->pen_logits && diag->pen_ld < V) return fail(ctx, MS_ERR_ARG, "ms_sample: diag->pen_ld < V");
  const ms_params pp = *params;
  const bool greedy = !pp.do_sample || pp.temperature <= 0.0001;
  if (!greedy && !u) return fail(ctx, MS_ERR_ARG, "ms_sample: sampled rows need u[B]");
  int prev = 0;
  cudaGetDevice(&prev);

  if (dev) {
    if (flags & MS_ROW_SHARDED) return fail(ctx, MS_ERR_ARG, "ms_sample: MS_ROW_SHARDED needs host pointers");
    DevState& s = ctx->devs[0];
    cudaSetDevice(s.device);
    cudaStream_t st = stream ? (cudaStream_t)stream : s.stream;
    int rc = run_device(ctx, s, logits, B, V, ld, hist, hist_off, &pp, u, out_ids, diag, st,
                        (flags & MS_PROFILE) != 0);
    if (rc == MS_OK && (flags & MS_SYNC)) {
      cudaError_t e = cudaStreamSynchronize(st);
      if (e != cudaSuccess) rc = fail(ctx, MS_ERR_CUDA, "ms_sample: %s", cudaGetErrorString(e));
      if (rc == MS_OK) rc = read_status(ctx, s, "ms_sample");
    }
    cudaSetDevice(prev);
    return rc;
  }

  // ---- host pointers: stage through device memory, one row slice per device
  if (hist_off) {
    if (hist_off[0] < 0) return fail(ctx, MS_ERR_ARG, "ms_sample: hist_off[0] < 0");
    for (int64_t r = 0; r < B; r++)
      if (hist_off[r + 1] < hist_off[r]) return fail(ctx, MS_ERR_ARG, "ms_sample: hist_off not ascending");
  }
  const int nd = (flags & MS_ROW_SHARDED) ? (int)ctx->devs.size() : 1;
  const int64_t per = (B + nd - 1) / nd;
  int rc = MS_OK;
  struct Slice { int64_t r0, rows; size_t o_logits, o_hist, o_off, o_u, o_out, o_cid, o_cp, o_nc, o_mx, o_sum, o_tot, o_fl, o_pen; };
  std::vector<Slice> slices(nd);
  for (int d = 0; d < nd && rc == MS_OK; d++) {
    DevState& s = ctx->devs[d];
    Slice& sl = slices[d];
    sl.r0 = d * per;
    sl.rows = std::min<int64_t>(per, B - sl.r0);
    if (sl.rows <= 0) { sl.rows = 0; continue; }
    cudaSetDevice(s.device);
    const int64_t h0 = hist_off ? hist_off[sl.r0] : 0;
    const int64_t h1 = hist_off ? hist_off[sl.r0 + sl.rows] : 0;
    const int64_t nh = h1 - h0;
    size_t off = 0;
    auto take = [&](size_t bytes) { size_t o = off; off = align_up(off + bytes, 256); return o; };
    sl.o_logits = take((size_t)sl.rows * V * 4);
    sl.o_hist = take((size_t)(nh > 0 ? nh : 1) * 4);
    sl.o_off = take((size_t)(sl.rows + 1) * 8);
    sl.o_u = take((size_t)sl.rows * 8);
    sl.o_out = take((size_t)sl.rows * 4);
    const int cap = diag ? diag->cand_cap : 0;
    sl.o_cid = take((size_t)sl.rows * (cap > 0 ? cap : 1) * 4);
    sl.o_cp = take((size_t)sl.rows * (cap > 0 ? cap : 1) * 4);
    sl.o_nc = take((size_t)sl.rows * 4);
    sl.o_mx = take((size_t)sl.rows * 8);
    sl.o_sum = take((size_t)sl.rows * 8);
    sl.o_tot = take((size_t)sl.rows * 8);
    sl.o_fl = take((size_t)sl.rows * 4);
    sl.o_pen = take(diag && diag->pen_logits ? (size_t)sl.rows * V * 4 : 4);
    rc = ensure(ctx, &s.io, &s.io_bytes, off);
    if (rc) break;
    char* io = (char*)s.io;
    cudaStream_t st = s.stream;
    auto H2D = [&](size_t o, const void* src, size_t bytes) {
      return cudaMemcpyAsync(io + o, src, bytes, cudaMemcpyHostToDevice, st);
    };
    cudaError_t e = cudaSuccess;
    if (ld == V) e = H2D(sl.o_logits, logits + sl.r0 * ld, (size_t)sl.rows * V * 4);
    else e = cudaMemcpy2DAsync(io + sl.o_logits, (size_t)V * 4, logits + sl.r0 * ld, (size_t)ld * 4,
                               (size_t)V * 4, (size_t)sl.rows, cudaMemcpyHostToDevice, st);
    const int32_t* dh = nullptr;
    const int64_t* doff = nullptr;
    if (e == cudaSuccess && hist_off) {
      // rebased offsets, staged in the device state so the host buffer lives
      // until the stream sync below
      std::vector<int64_t>& offs = s.host_offs;
      offs.resize((size_t)sl.rows + 1);
      for (int64_t r = 0; r <= sl.rows; r++) offs[r] = hist_off[sl.r0 + r] - h0;
      if (nh > 0) e = H2D(sl.o_hist, hist + h0, (size_t)nh * 4);
      if (e == cudaSuccess) e = H2D(sl.o_off, offs.data(), offs.size() * 8);
      dh = (const int32_t*)(io + sl.o_hist);
      doff = (const int64_t*)(io + sl.o_off);
    }
    if (e == cudaSuccess && u) e = H2D(sl.o_u, u + sl.r0, (size_t)sl.rows * 8);
    if (e != cudaSuccess) { rc = fail(ctx, MS_ERR_CUDA, "ms_sample: H2D: %s", cudaGetErrorString(e)); break; }
    ms_diag dd;
    ms_diag* dp = nullptr;
    if (diag) {
      dd.cand_cap = diag->cand_cap;
      dd.cand_ids = diag->cand_ids ? (int32_t*)(io + sl.o_cid) : nullptr;
      dd.cand_probs = diag->cand_probs ? (float*)(io + sl.o_cp) : nullptr;
      dd.n_cand = diag->n_cand ? (int32_t*)(io + sl.o_nc) : nullptr;
      dd.row_max = diag->row_max ? (double*)(io + sl.o_mx) : nullptr;
      dd.row_sum = diag->row_sum ? (double*)(io + sl.o_sum) : nullptr;
      dd.total = diag->total ? (double*)(io + sl.o_tot) : nullptr;
      dd.row_flags = diag->row_flags ? (int32_t*)(io + sl.o_fl) : nullptr;
      dd.pen_logits = diag->pen_logits ? (float*)(io + sl.o_pen) : nullptr;
      dd.pen_ld = V;
      dp = &dd;
    }
    rc = run_device(ctx, s, (const float*)(io + sl.o_logits), sl.rows, V, V, dh, doff, &pp,
                    u ? (const double*)(io + sl.o_u) : nullptr, (int32_t*)(io + sl.o_out), dp, st,
                    (flags & MS_PROFILE) != 0);
    if (rc) break;
    auto D2H = [&](void* dst, size_t o, size_t bytes) {
      return cudaMemcpyAsync(dst, io + o, bytes, cudaMemcpyDeviceToHost, st);
    };
    e = D2H(out_ids + sl.r0, sl.o_out, (size_t)sl.rows * 4);
    if (diag && e == cudaSuccess) {
      const int cap = diag->cand_cap;
      if (diag->cand_ids && cap > 0) e = D2H(diag->cand_ids + sl.r0 * cap, sl.o_cid, (size_t)sl.rows * cap * 4);
      if (e == cudaSuccess && diag->cand_probs && cap > 0)
        e = D2H(diag->cand_probs + sl.r0 * cap, sl.o_cp, (size_t)sl.rows * cap * 4);
      if (e == cudaSuccess && diag->n_cand) e = D2H(diag->n_cand + sl.r0, sl.o_nc, (size_t)sl.rows * 4);
      if (e == cudaSuccess && diag->row_max) e = D2H(diag->row_max + sl.r0, sl.o_mx, (size_t)sl.rows * 8);
      if (e == cudaSuccess && diag->row_sum) e = D2H(diag->row_sum + sl.r0, sl.o_sum, (size_t)sl.rows * 8);
      if (e == cudaSuccess && diag->total) e = D2H(diag->total + sl.r0, sl.o_tot, (size_t)sl.rows * 8);
      if (e == cudaSuccess && diag->row_flags) e = D2H(diag->row_flags + sl.r0, sl.o_fl, (size_t)sl.rows * 4);
      if (e == cudaSuccess && diag->pen_logits)
        e = cudaMemcpy2DAsync(diag->pen_logits + sl.r0 * diag->pen_ld, (size_t)diag->pen_ld * 4, io + sl.o_pen,
                              (size_t)V * 4, (size_t)V * 4, (size_t)sl.rows, cudaMemcpyDeviceToHost, st);
    }
    if (e != cudaSuccess) { rc = fail(ctx, MS_ERR_CUDA, "ms_sample: D2H: %s", cudaGetErrorString(e)); break; }
  }
  // wait for every device, then read each status word
  for (int d = 0; d < nd; d++) {
    if (slices[d].rows <= 0) continue;
    DevState& s = ctx->devs[d];
    cudaSetDevice(s.device);
    cudaError_t e = cudaStreamSynchronize(s.stream);
    if (e != cudaSuccess && rc == MS_OK) rc = fail(ctx, MS_ERR_CUDA, "ms_sample: %s", cudaGetErrorString(e));
    if (rc == MS_OK) rc = read_status(ctx, s, "ms_sample");
  }
  cudaSetDevice(prev);
  return rc;
}

// ====================================================== allocation-free entry point
// Scratch for ms_sample_noalloc: a file-scope device array, so the call never
// allocates.  Every GPU that loads this library holds these bytes until the
// process exits.  Host code must not use the symbol's name as an address (it
// is a host-side stand-in); the device address comes from
// cudaGetSymbolAddress, taken once per device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[MS_NOALLOC_SCRATCH_BYTES];

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_addr[64] = {};  // device address of g_noalloc_scratch, per device
}  // namespace

extern "C" int ms_sample_noalloc(const float* logits, int64_t B, int64_t V, int64_t ld, const int32_t* hist,
                                 const int64_t* hist_off, const ms_params* params, const double* u,
                                 int32_t* out_ids, void* stream) {
  if (!params || B < 0 || V < 1 || V > (int64_t)65535 * ms::kChunk || ld < V) return MS_ERR_ARG;
  if (B == 0) return MS_OK;
  if (!logits || !out_ids) return MS_ERR_ARG;
  if (hist_off != nullptr && hist == nullptr) return MS_ERR_ARG;
  if (hist_off == nullptr) hist = nullptr;
  const ms_params pp = *params;
  const Plan P = make_plan(V, &pp, hist != nullptr);
  if (P.mode != ms::kGreedy && !u) return MS_ERR_ARG;
  // [row counters | status word | the kernel's scratch], all inside the array
  const size_t cnt_bytes = align_up((size_t)B * 4, 256);
  const ScratchLayout L = scratch_layout(B, V, P);
  const size_t need = cnt_bytes + 256 + L.total;
  if (need > (size_t)MS_NOALLOC_SCRATCH_BYTES) return MS_ERR_SCRATCH;

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MS_ERR_STATE;
  void* addr = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return MS_ERR_CUDA;
      g_noalloc_addr[dev] = p;
    }
    addr = g_noalloc_addr[dev];
  }
  char* base = (char*)addr;
  cudaStream_t st = (cudaStream_t)stream;
  // the array keeps the last call's contents: counters and status restart at zero
  if (cudaMemsetAsync(base, 0, cnt_bytes + 256, st) != cudaSuccess) return MS_ERR_CUDA;
  char* scratch = base + cnt_bytes + 256;

  ms::Args A;
  memset(&A, 0, sizeof A);
  A.logits = logits;
  A.ld = ld;
  A.B = (int32_t)B;
  A.V = (int32_t)V;
  A.hist = hist;
  A.hist_off = hist_off;
  A.pen = pp.repetition_penalty;
  A.rpen = 1.0 / pp.repetition_penalty;
  A.use_pen = P.use_pen;
  A.mode = P.mode;
  A.T = pp.temperature;
  A.rT = 1.0 / pp.temperature;
  A.temper = P.temper;
  A.a = P.a;
  A.k = P.k;
  A.kw = P.kw;
  A.use_topp = P.use_topp;
  A.top_p = pp.top_p;
  A.u = u;
  A.n_chunks = P.n_chunks;
  A.stats = (ms::ChunkStat*)(scratch + L.stats);
  A.cands = (ms::Cand*)(scratch + L.cands);
  A.penbits = (P.use_pen && P.mode != ms::kGreedy) ? (uint32_t*)(scratch + L.penbits) : nullptr;
  if (P.mode == ms::kFull) {
    // counts only for rank selection (top_k above the candidate path)
    A.h_cnt = (P.k > 0 && P.k < V) ? (uint16_t*)(scratch + L.h_cnt) : nullptr;
    A.h_mass = (double*)(scratch + L.h_mass);
    A.plan = (ms::NucPlan*)(scratch + L.plan);
    A.lists = (ms::Cand*)(scratch + L.lists);
    A.list_cnt = (int32_t*)(scratch + L.list_cnt);
  }
  A.status = (int32_t*)(base + cnt_bytes);
  A.epoch = 1;  // the status word was cleared above: 1 marks a wait of this call that ran out
  A.row_count = (int32_t*)base;
  A.ksum = ms::kKSum;
  A.out_ids = out_ids;
  if (ms::launch_sample(A, st, nullptr, nullptr) != cudaSuccess) return MS_ERR_CUDA;
  return MS_OK;
}

// ---------------------------------------------------------------- vocabulary shards
namespace {
// record bytes per row, or -1 when the params are not supported sharded
int64_t record_bytes(int64_t V, const ms_params* p) {
  const Plan P = make_plan(V, p, false);
  if (P.mode == ms::kGreedy) return ms::kRecHead;
  if (P.mode != ms::kTopK) return -1;
  return ms::kRecHead + (int64_t)(P.k + ms::kTieSlack) * ms::kRecCand;
}
}  // namespace

extern "C" int ms_shard_record_bytes(int64_t V, const ms_params* params, int64_t* rec_bytes) {
  if (!params || !rec_bytes || V < 1) return MS_ERR_ARG;
  const int64_t b = record_bytes(V, params);
  if (b < 0) return MS_ERR_ARG;
  *rec_bytes = b;
  return MS_OK;
}

extern "C" int ms_shard_records(ms_ctx* ctx, const float* logits, int64_t B, int64_t V, int64_t col0, int64_t cols,
                                int64_t ld, const int32_t* hist, const int64_t* hist_off, const ms_params* params,
                                void* records, int64_t rec_bytes, void* stream) {
  if (!ctx) return MS_ERR_ARG;
  if (!params) return fail(ctx, MS_ERR_ARG, "ms_shard_records: params is NULL");
  if (B < 0 || V < 1 || V > (int64_t)65535 * ms::kChunk || col0 < 0 || cols < 1 || col0 + cols > V || ld < cols)
    return fail(ctx, MS_ERR_ARG, "ms_shard_records: bad B / V / col0 / cols / ld");
  if (record_bytes(V, params) != rec_bytes)
    return fail(ctx, MS_ERR_ARG, "ms_shard_records: rec_bytes differs from ms_shard_record_bytes (or top_k unsupported)");
  if (B == 0) return MS_OK;
  if (!logits || !records) return fail(ctx, MS_ERR_ARG, "ms_shard_records: logits/records is NULL");
  if (hist_off != nullptr && hist == nullptr) return fail(ctx, MS_ERR_ARG, "ms_shard_records: hist_off without hist");
  if (hist_off == nullptr) hist = nullptr;
  DevState& s = ctx->devs[0];
  MS_CUDA(ctx, cudaSetDevice(s.device));
  cudaStream_t st = stream ? (cudaStream_t)stream : s.stream;
  Plan P = make_plan(V, params, hist != nullptr);  // the mode and bound follow the whole row
  P.n_chunks = (int)((cols + ms::kChunk - 1) / ms::kChunk);
  if ((int64_t)B * P.n_chunks > (int64_t)INT32_MAX - (1 << 20))
    return fail(ctx, MS_ERR_ARG, "ms_shard_records: B * chunks too large");
  const ScratchLayout L = scratch_layout(B, cols, P);
  int rc = ensure(ctx, &s.scratch, &s.scratch_bytes, L.total + (size_t)B * 4 + 256);
  if (rc) return rc;
  rc = ensure_state(ctx, s, B);
  if (rc) return rc;
  char* base = (char*)s.scratch;
  ms::Args A = param_args(P, params);
  A.logits = logits;
  A.ld = ld;
  A.B = (int32_t)B;
  A.V = (int32_t)cols;
  A.col0 = (int32_t)col0;
  A.hist = hist;
  A.hist_off = hist_off;
  A.stats = (ms::ChunkStat*)(base + L.stats);
  A.cands = (ms::Cand*)(base + L.cands);
  A.status = s.status;
  A.epoch = next_epoch(s);
  A.row_count = s.counters;
  A.out_ids = (int32_t*)(base + align_up(L.total, 256));  // greedy chunk kernel's per-shard ids (unused)
  A.rec = (unsigned char*)records;
  A.rec_bytes = (int32_t)rec_bytes;
  A.k_send = (int32_t)((rec_bytes - ms::kRecHead) / ms::kRecCand);
  MS_CUDA(ctx, ms::launch_shard(A, st));
  s.launches += 2;
  return MS_OK;
}

extern "C" int ms_merge_records(ms_ctx* ctx, const void* records, int64_t B, int64_t G, int64_t V,
                                const ms_params* params, const double* u, int32_t* out_ids, ms_diag* diag,
                                int64_t rec_bytes, void* stream) {
  if (!ctx) return MS_ERR_ARG;
  if (!params) return fail(ctx, MS_ERR_ARG, "ms_merge_records: params is NULL");
  if (B < 0 || V < 1 || V > (int64_t)65535 * ms::kChunk || G < 1 || G > 32)
    return fail(ctx, MS_ERR_ARG, "ms_merge_records: bad B / G / V (1 <= G <= 32)");
  if (record_bytes(V, params) != rec_bytes)
    return fail(ctx, MS_ERR_ARG, "ms_merge_records: rec_bytes differs from ms_shard_record_bytes (or top_k unsupported)");
  const Plan P = make_plan(V, params, false);
  if (P.mode == ms::kTopK && G * (int64_t)(P.k + ms::kTieSlack) > ms::kGathMax)
    return fail(ctx, MS_ERR_ARG, "ms_merge_records: G * (top_k + 32) exceeds 4096 candidates");
  if (B == 0) return MS_OK;
  if (!records || !out_ids) return fail(ctx, MS_ERR_ARG, "ms_merge_records: records/out_ids is NULL");
  if (P.mode != ms::kGreedy && !u) return fail(ctx, MS_ERR_ARG, "ms_merge_records: sampled rows need u[B]");
  DevState& s = ctx->devs[0];
  MS_CUDA(ctx, cudaSetDevice(s.device));
  cudaStream_t st = stream ? (cudaStream_t)stream : s.stream;
  ms::Args A = param_args(P, params);
  A.B = (int32_t)B;
  A.V = (int32_t)V;
  A.u = u;
  A.out_ids = out_ids;
  A.rec = (unsigned char*)records;
  A.rec_bytes = (int32_t)rec_bytes;
  A.G = (int32_t)G;
  if (diag) {
    A.cand_cap = diag->cand_cap;
    A.d_cand_ids = diag->cand_cap > 0 ? diag->cand_ids : nullptr;
    A.d_cand_probs = diag->cand_cap > 0 ? diag->cand_probs : nullptr;
    A.d_n_cand = diag->n_cand;
    A.d_row_max = diag->row_max;
    A.d_row_sum = diag->row_sum;
    A.d_total = diag->total;
    A.d_row_flags = diag->row_flags;
  }
  MS_CUDA(ctx, ms::launch_merge(A, st));
  s.launches += 1;
  return MS_OK;
}
