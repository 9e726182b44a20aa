// Device helpers shared by the sampler kernels (sm_100a).
//
// Arithmetic contract (mini.js src/generation.js): JS computes in IEEE double
// and rounds to fp32 on every Float32Array store.  The helpers below reproduce
// those stores exactly where a value reaches the output:
//   penalty      fp32(double(v) / p)  or fp32(double(v) * p)   (:22-23)
//   temperature  fp32(double(x) / T)                           (:78)
//   softmax term fp32(exp(double(x') - double(mx)))            (:14)
//   probability  fp32(double(e) / sum)                         (:15)
// CUDA's double `/` and `*` are IEEE round-to-nearest; __double2float_rn is the
// fp32 store.  The exact softmax term uses js_exp below, the published fdlibm
// exp method that V8's Math.exp ports, so it equals V8's term bit for bit.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/minisample.h"

namespace ms {

constexpr int kThreads = 512;           // threads per CTA
constexpr int kChunk = 16384;           // logits per chunk CTA (64 KiB of smem)
constexpr int kSub = 4;                 // bulk-copy pieces per chunk (16 KiB each)
constexpr int kSubElems = kChunk / kSub;
constexpr int kCap = 512;               // candidate slots per chunk
constexpr int kKmax = 256;              // largest top_k on the candidate path
constexpr int kGathMax = 4096;          // candidates >= the row threshold the finalizer can hold
constexpr int kFinMax = 1024;           // candidates the finalizer ranks exactly
constexpr int kKSum = 64;               // candidates kept for the sum correction when top_k is off

// Whole-vocabulary rows (top_k off or above kKmax): mass histograms.  A bin is
// 1/16 of a log2 unit of the tempered logit: bin(x) = floor(-x * 16 * log2(e) / T),
// one grid for every chunk of every row; a chunk's histogram covers kNB bins
// from its own top bin down (the last one also holds everything below).
constexpr int kNB = 512;
constexpr int kListCap = 8192;          // elements of one extraction range a row can hold

constexpr int kRecHead = 32;             // vocab-shard record: header bytes
constexpr int kRecCand = 16;             // bytes per listed candidate
constexpr int kTieSlack = 32;            // list room beyond top_k for ties at a shard's k-th value

// The device status word.  A kernel whose bounded wait runs out stores the
// call's epoch there (Args::epoch, never 0); the host and the later kernels of
// the same call compare it with that epoch, so a timeout never leaks into a
// later call and the word needs no clearing between calls.

struct ChunkStat {
  float m;        // max of the penalised logits of the chunk (NaN ignored; -inf if none)
  float tau;      // top-k bound: at least top_k elements of the chunk are >= tau (-inf if unknown)
  double s;       // sum of fast exp2((x - m) * a) over the chunk (NaN if a NaN appeared)
  int32_t n_cand; // elements >= tau (only the first kCap are stored)
  int32_t best_i; // greedy: first index of the max (INT32_MAX if nothing > -inf)
  float zref;     // fast terms are 2^(x * a - zref); NaN: 2^((x - m) * a) (m * a beyond fp32)
  float sig;      // storage threshold: every element >= sig is among the candidates (sig >= tau)
};

static_assert(sizeof(ChunkStat) == 32, "chunk stats: two 16-byte loads");

struct Cand {
  float x;        // penalised (untempered) logit
  int32_t i;      // vocabulary id
};

// Selection plan of one whole-vocabulary row (nucleus_plan_kernel): the row's
// mass histogram located the top-p cut and the draw in one or two bin ranges,
// whose elements nucleus_extract_kernel copies out and nucleus_resolve_kernel
// ranks exactly.
struct NucPlan {
  int32_t flags;         // kPlanDone: outputs already written; kPlanFallback: exact whole-row path
  int32_t b_row;         // absolute histogram bin of the row max (row bin 0)
  int32_t nr;            // extraction ranges (0, 1 or 2)
  int32_t cut_rg;        // range holding the cut (-1: no cut, every element is a candidate)
  int32_t draw_rg;       // range holding the draw
  int32_t lo[2], hi[2];  // the ranges, in row bins (inclusive)
  int32_t pad;
  int64_t cnt_above[2];  // elements in the row bins above each range
  double mass_above[2];  // their fast probability mass
  double mass_tot;       // fast probability mass of the row
  double S;              // softmax denominator
  float M, Mp;           // penalised max, tempered max
};
constexpr int kPlanDone = 1, kPlanFallback = 2;

enum Mode : int32_t { kGreedy = 0, kTopK = 1, kFull = 2 };

struct Args {
  const float* logits;
  int64_t ld;
  int32_t B, V;
  const int32_t* hist;
  const int64_t* hist_off;
  double pen;            // repetition penalty (applied iff use_pen)
  double rpen;           // fp64(1 / pen)
  int32_t use_pen;
  int32_t mode;
  double T;              // temperature
  double rT;             // fp64(1 / T)
  int32_t temper;        // 1 when T != 1.0
  float a;               // fp32(log2(e) / T): scale of the fast exp2 terms
  int32_t k;             // top_k as the reference uses it (0 = off)
  int32_t kw;            // per-warp rank of the thread maxima that bounds tau
  int32_t ksum;          // candidates whose exact terms correct the fast sum (top_k or 64)
  int32_t use_topp;
  double top_p;
  const double* u;
  int32_t n_chunks;
  ChunkStat* stats;      // [B, n_chunks]
  int32_t* row_count;    // [B] chunks finished per row (self-resetting)
  Cand* cands;           // [B, n_chunks, kCap]
  uint32_t* penbits;     // [B, ceil(V/32)] penalty bitmap (slow path), may be null
  int32_t* out_ids;      // [B]
  // whole-vocabulary rows (mode kFull)
  uint16_t* h_cnt;       // [B, n_chunks, kNB] elements per chunk bin
  double* h_mass;        // [B, n_chunks, kNB] their fast masses, in units of the chunk's zref term
  struct NucPlan* plan;  // [B] the row's selection plan (nucleus_plan_kernel)
  Cand* lists;           // [B, 2, kListCap] elements of the plan's extraction ranges
  int32_t* list_cnt;     // [B, 4]: elements in each range, elements above each range
  int32_t* status;       // device status word (see above)
  int32_t epoch;         // this call's epoch (> 0)
  int32_t fuse_fin;      // top-k rows: the chunk kernel's last CTA of each row finalizes it
                         // (small batches: no second launch)
  long long test_wait;   // > 0: the first chunk CTA waits this many cycles on an
                         // mbarrier nothing completes (ms_debug_inject)
  float* d_pen;          // diagnostics: penalised logits [B, pen_ld] (may be null)
  int64_t pen_ld;
  // vocabulary shards (0 / null otherwise)
  int32_t col0;          // global column of local column 0 (penalty ids are global)
  int32_t G;             // merge: shards per row
  unsigned char* rec;    // shard records: [B, rec_bytes] (shard) or [B, G, rec_bytes] (merge)
  int32_t rec_bytes;
  int32_t k_send;        // shard: list capacity of a record
  // diagnostics (each may be null)
  int32_t cand_cap;
  int32_t* d_cand_ids;
  float* d_cand_probs;
  int32_t* d_n_cand;
  double* d_row_max;
  double* d_row_sum;
  double* d_total;
  int32_t* d_row_flags;
};

// ---------------------------------------------------------------- exact helpers

__device__ __forceinline__ float pen_apply(float v, double p) {
  double d = (double)v;
  return __double2float_rn(d > 0.0 ? __ddiv_rn(d, p) : __dmul_rn(d, p));
}

// pen_apply with the divide replaced by a multiply by rp = 1/p (rounded).
// q = fp64(v * rp) is within 3 fp64 ulps of fp64(v / p), so both round to the
// same fp32 unless q lies within a few ulps of an fp32 rounding midpoint (the
// 29 mantissa bits an fp32 store drops read 1000...0); those rare cases, and
// results in the fp32 subnormal range, take the exact divide.
__device__ __forceinline__ float pen_apply_fast(float v, double p, double rp) {
  const double d = (double)v;
  if (!(d > 0.0)) return __double2float_rn(__dmul_rn(d, p));
  const double q = __dmul_rn(d, rp);
  const uint32_t low = (uint32_t)__double_as_longlong(q) & 0x1FFFFFFFu;
  if ((uint32_t)(low - (0x10000000u - 16u)) <= 32u || q < 1.1754943508222875e-38)
    return __double2float_rn(__ddiv_rn(d, p));
  return __double2float_rn(q);
}

__device__ __forceinline__ float temper_exact(float x, double T, int temper) {
  return temper ? __double2float_rn(__ddiv_rn((double)x, T)) : x;
}

// fp32(d / D) from q = d * rD (rD = fp64(1 / D)): q is within 3 fp64 ulps of
// d / D, so both round to the same fp32 unless q lies next to an fp32
// rounding midpoint (the 29 dropped bits read 1000...0), falls in the fp32
// subnormal range, or is not finite; those take the exact divide.
__device__ __forceinline__ float div_to_f32(double d, double D, double rD) {
  const double q = __dmul_rn(d, rD);
  const uint32_t low = (uint32_t)__double_as_longlong(q) & 0x1FFFFFFFu;
  const double aq = fabs(q);
  if ((uint32_t)(low - (0x10000000u - 16u)) <= 32u || (aq < 1.1754943508222875e-38 && aq != 0.0) ||
      !(aq <= 1.7976931348623157e308))
    return __double2float_rn(__ddiv_rn(d, D));
  return __double2float_rn(q);
}
__device__ __forceinline__ float temper_fast(float x, double T, double rT, int temper) {
  return temper ? div_to_f32((double)x, T, rT) : x;
}

// Math.exp as V8 computes it: fdlibm's exp (e_exp.c), which V8 ports in
// src/base/ieee754.cc.  x = k*ln2 + r with |r| <= ln2/2 and ln2 split so that
// k*ln2_hi is exact; on that range r*(e^r + 1)/(e^r - 1) ~ 2 + P1 z + ... + P5 z^5
// (z = r^2, fdlibm's Remez coefficients), so e^r = 1 + r + r*c/(2 - c) with
// c = r - z*(P1 + ...), and e^x = 2^k e^r.  Every step is one IEEE double
// operation in fdlibm's order (explicit _rn intrinsics: nothing is contracted
// into an FMA).
static __device__ __noinline__ double js_exp(double x) {
  const double ln2_hi = 6.93147180369123816490e-01, ln2_lo = 1.90821492927058770002e-10;
  const double inv_ln2 = 1.44269504088896338700e+00;
  const double p1 = 1.66666666666666019037e-01, p2 = -2.77777777770155933842e-03,
               p3 = 6.61375632143793436117e-05, p4 = -1.65339022054652515390e-06,
               p5 = 4.13813679705723846039e-08;
  const long long bx = __double_as_longlong(x);
  const uint32_t hw = (uint32_t)((unsigned long long)bx >> 32);
  const int neg = (int)(hw >> 31);
  const uint32_t ahw = hw & 0x7fffffffu;
  if (ahw >= 0x40862E42u) {  // |x| >= 709.78, or not finite
    if (ahw >= 0x7ff00000u) {
      if (((ahw & 0xfffffu) | (uint32_t)bx) != 0u) return __dadd_rn(x, x);  // NaN
      return neg ? 0.0 : x;
    }
    if (x > 7.09782712893383973096e+02) return __longlong_as_double(0x7ff0000000000000ll);
    if (x < -7.45133219101941108420e+02) return 0.0;
  }
  double hi = 0.0, lo = 0.0, r;
  int k = 0;
  if (ahw > 0x3FD62E42u) {    // |x| > ln2/2
    if (ahw < 0x3FF0A2B2u) {  // |x| < 1.5 ln2: k = +-1
      if (x == 1.0) return 2.718281828459045;  // V8 returns E here
      hi = neg ? __dadd_rn(x, ln2_hi) : __dsub_rn(x, ln2_hi);
      lo = neg ? -ln2_lo : ln2_lo;
      k = neg ? -1 : 1;
    } else {
      k = __double2int_rz(__dadd_rn(__dmul_rn(inv_ln2, x), neg ? -0.5 : 0.5));
      const double t = (double)k;
      hi = __dsub_rn(x, __dmul_rn(t, ln2_hi));  // exact
      lo = __dmul_rn(t, ln2_lo);
    }
    r = __dsub_rn(hi, lo);
  } else if (ahw < 0x3e300000u) {  // |x| < 2^-28
    return __dadd_rn(1.0, x);
  } else {
    r = x;
  }
  const double z = __dmul_rn(r, r);
  double q = __dadd_rn(p4, __dmul_rn(z, p5));
  q = __dadd_rn(p3, __dmul_rn(z, q));
  q = __dadd_rn(p2, __dmul_rn(z, q));
  q = __dadd_rn(p1, __dmul_rn(z, q));
  const double c = __dsub_rn(r, __dmul_rn(z, q));
  if (k == 0) return __dsub_rn(1.0, __dsub_rn(__ddiv_rn(__dmul_rn(r, c), __dsub_rn(c, 2.0)), r));
  const double y = __dsub_rn(1.0, __dsub_rn(__dsub_rn(lo, __ddiv_rn(__dmul_rn(r, c), __dsub_rn(2.0, c))), hi));
  if (k >= -1021) {
    if (k == 1024) return __dmul_rn(__dmul_rn(y, 2.0), __longlong_as_double(0x7fe0000000000000ll));
    return __dmul_rn(y, __longlong_as_double((long long)(0x3ff + k) << 52));  // exact
  }
  return __dmul_rn(__dmul_rn(y, __longlong_as_double((long long)(0x3ff + k + 1000) << 52)),
                   __longlong_as_double(0x0170000000000000ll));  // * 2^-1000
}

__device__ __forceinline__ float term_exact(float xp, float mxp) {
  return __double2float_rn(js_exp(__dsub_rn((double)xp, (double)mxp)));
}

__device__ __forceinline__ float prob_exact(float e, double S) {
  return __double2float_rn(__ddiv_rn((double)e, S));
}

// Fast fp32 softmax term relative to a reference max m: 2^((x - m) * a).  The
// instruction sequence is fixed (no contraction) so the finalize kernel can
// recompute a chunk's terms bit for bit.
__device__ __forceinline__ float ex2_approx(float z) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(z));
  return y;
}
__device__ __forceinline__ float term_fast(float x, float m, float a) {
  return ex2_approx(__fmul_rn(__fsub_rn(x, m), a));
}
// The chunk kernel's form of the fast term: 2^(x * a - zref), one fused
// multiply-add, with zref = fp32(m * a) for the chunk max m.  Relative to
// term_fast(x, m, a) the whole chunk carries the factor 2^(m * a - zref),
// which the finalizer folds into the chunk's scale.
__device__ __forceinline__ float term_fast_z(float x, float a, float zref) {
  return ex2_approx(__fmaf_rn(x, a, -zref));
}

// ---------------------------------------------------------------- paired fp32 (sm_100)
// Two fp32 lanes in one 64-bit register: fma / add on both at once, each lane
// rounded exactly like the scalar instruction.
__device__ __forceinline__ unsigned long long f2_pack(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 f2_unpack(unsigned long long v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b,
                                                     unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// max of three (NaN inputs are ignored, as by fmaxf)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// ---------------------------------------------------------------- float keys
// Order-preserving map of fp32 to uint32 (larger float -> larger key).
__device__ __forceinline__ uint32_t fkey(float x) {
  uint32_t b = __float_as_uint(x);
  return b ^ ((uint32_t)((int32_t)b >> 31) | 0x80000000u);
}
__device__ __forceinline__ float fkey_inv(uint32_t k) {
  uint32_t b = (k & 0x80000000u) ? (k ^ 0x80000000u) : ~k;
  return __uint_as_float(b);
}

// ---------------------------------------------------------------- mbarrier / bulk copy
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
// Untiled TMA bulk copy global -> shared, one destination CTA.  dst, src 16-byte
// aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}
// 4-byte asynchronous copy global -> shared (any 4-byte aligned address).
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
// The barrier's pending count goes up by one now, and comes down once the
// thread's earlier cp.async copies have landed.
__device__ __forceinline__ void cp_async_mbar_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}
// Orders this thread's earlier generic-proxy accesses of shared memory before
// its later async-proxy (bulk copy) accesses.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Bounded wait on phase `parity`; false when ~`max_cycles` passed first.  Each
// try_wait may suspend the thread for up to kSuspendNs (it resumes as soon as
// the phase completes), so a waiting warp issues few instructions.
constexpr uint32_t kSuspendNs = 100000u;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, long long max_cycles) {
  uint32_t a = smem_addr(bar);
  long long t0 = clock64();
  for (;;) {
    uint32_t done;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
        : "=r"(done)
        : "r"(a), "r"(parity), "r"(kSuspendNs)
        : "memory");
    if (done) return true;
    if (clock64() - t0 > max_cycles) return false;
  }
}

// ---------------------------------------------------------------- reductions
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace ms
