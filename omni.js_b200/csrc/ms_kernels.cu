// Sampler kernels for B200 (sm_100a).
//
// One sampling step over a [B, V] fp32 logits block runs as two launches:
//
//   chunk_kernel    grid (ceil(V/16384), B).  A CTA stages one 64 KiB chunk of
//                   one row in shared memory with TMA bulk copies, applies the
//                   repetition penalty to it (src/generation.js:19-25), then
//                   makes two passes over shared memory: (A) the chunk max and
//                   a threshold tau that at least top_k chunk elements reach;
//                   (B) a fast fp32 sum of 2^((x-m)*log2(e)/T) and the list of
//                   elements >= tau.  Logits are read from HBM exactly once.
//   finalize_kernel grid B.  A CTA merges its row's chunk results: the row
//                   max, the softmax denominator (fast sum corrected with the
//                   exact terms of every candidate), the exact fp32
//                   probabilities of the candidates, their order
//                   (prob desc, id asc), the top-k / top-p cut and the draw
//                   (src/generation.js:9-17, 27-49).
//
// Rows whose candidate set cannot be proven complete, and every row when top_k
// is off (top_k <= 0 or >= V) or larger than 256, go through full_path: an
// exact rescan of the row by radix selection over order-preserving float keys.
#include <cfloat>
#include <climits>
#include <cstdio>

#include "ms_device.cuh"

namespace ms {

constexpr long long kWaitCycles = 4000000000LL;  // ~2 s: bound on every wait
constexpr unsigned kAll = 0xffffffffu;

// =============================================================== chunk kernel
template <int MODE, bool PEN>
__global__ void __launch_bounds__(kThreads, 3) chunk_kernel(const Args A) {
  extern __shared__ __align__(128) unsigned char dyn_smem[];
  float* tile = reinterpret_cast<float*>(dyn_smem);
  __shared__ __align__(8) uint64_t bar[kSub];
  __shared__ uint32_t penmask[kChunk / 32];
  __shared__ Cand clist[kCap];
  __shared__ int ccount;
  __shared__ float w_max[kThreads / 32], w_tau[kThreads / 32];
  __shared__ double w_sum[kThreads / 32];
  __shared__ int w_bi[kThreads / 32];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c = blockIdx.x, r = blockIdx.y;
  const int c0 = c * kChunk;
  const int n = min(kChunk, A.V - c0);
  const float* g = A.logits + (int64_t)r * A.ld + c0;
  const bool bulk = ((reinterpret_cast<uintptr_t>(g) & 15) == 0) && ((n & 3) == 0);

  if (tid == 0) {
    ccount = 0;
    if (bulk) {
      for (int s = 0; s < kSub; s++) mbar_init(&bar[s], 1);
      fence_mbar_init();
    }
  }
  __syncthreads();
  if (bulk) {
    if (tid == 0) {
      for (int s = 0; s < kSub; s++) {
        const int b = s * kSubElems, cnt = min(kSubElems, n - b);
        if (cnt > 0) {
          mbar_expect_tx(&bar[s], (uint32_t)cnt * 4u);
          bulk_g2s(tile + b, g + b, (uint32_t)cnt * 4u, &bar[s]);
        }
      }
    }
  } else {
    for (int j = tid; j < n; j += kThreads) tile[j] = __ldg(g + j);
  }
  for (int j = n + tid; j < kChunk; j += kThreads) tile[j] = -INFINITY;
  if (PEN)
    for (int w = tid; w < kChunk / 32; w += kThreads) penmask[w] = 0u;
  int timed_out = 0;
  if (bulk) {
    for (int s = 0; s < kSub; s++)
      if (s * kSubElems < n && !mbar_wait(&bar[s], 0, kWaitCycles)) timed_out = 1;
  }
  if (__syncthreads_or(timed_out)) {
    if (tid == 0) atomicOr(A.status, kStatusTimeout);
    if (bulk)  // let any copy still in flight land before the CTA exits (bounded)
      for (int s = 0; s < kSub; s++)
        if (s * kSubElems < n) mbar_wait(&bar[s], 0, kWaitCycles);
    return;
  }

  // ---- repetition penalty: each distinct in-range id once (Set semantics)
  if (PEN) {
    const int64_t h0 = A.hist_off[r], h1 = A.hist_off[r + 1];
    for (int64_t h = h0 + tid; h < h1; h += kThreads) {
      const int64_t j = (int64_t)A.hist[h] - c0;
      if (j >= 0 && j < n) {
        const uint32_t bit = 1u << (j & 31);
        const uint32_t old = atomicOr(&penmask[j >> 5], bit);
        if (!(old & bit)) tile[j] = pen_apply(tile[j], A.pen);
      }
    }
    __syncthreads();
  }

  const float4* t4 = reinterpret_cast<const float4*>(tile);
  constexpr int kIters = kChunk / 4 / kThreads;  // 16 float4 per thread

  // ---- greedy: first index of the strict max (src/generation.js:51-55)
  if (MODE == kGreedy) {
    float bv = -INFINITY;
    int bi = INT_MAX;
#pragma unroll 4
    for (int i = 0; i < kIters; i++) {
      const int q = tid + i * kThreads;
      const float4 v = t4[q];
      const int j = c0 + 4 * q;
      if (v.x > bv) { bv = v.x; bi = j; }
      if (v.y > bv) { bv = v.y; bi = j + 1; }
      if (v.z > bv) { bv = v.z; bi = j + 2; }
      if (v.w > bv) { bv = v.w; bi = j + 3; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(kAll, bv, o);
      const int oi = __shfl_xor_sync(kAll, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) { w_max[warp] = bv; w_bi[warp] = bi; }
    __syncthreads();
    if (tid == 0) {
      for (int w = 1; w < kThreads / 32; w++)
        if (w_max[w] > bv || (w_max[w] == bv && w_bi[w] < bi)) { bv = w_max[w]; bi = w_bi[w]; }
      ChunkStat st;
      st.m = bv; st.tau = bv; st.s = 0.0; st.n_cand = 0; st.best_i = bi; st.best_v = bv; st.pad = 0;
      A.stats[(int64_t)r * A.n_chunks + c] = st;
    }
    return;
  }

  // ---- pass A: thread maxima -> chunk max and tau
  float tm = -INFINITY;
#pragma unroll 4
  for (int i = 0; i < kIters; i++) {
    const float4 v = t4[tid + i * kThreads];
    tm = fmaxf(tm, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
  }
  // Warp bitonic sort of the 32 thread maxima (ascending).  At least kw of them
  // are >= the warp's kw-th largest, so tau = min over warps of that value is
  // reached by >= 8*kw >= top_k distinct elements of the chunk.
  float sv = tm;
#pragma unroll
  for (int kk = 2; kk <= 32; kk <<= 1) {
#pragma unroll
    for (int jj = kk >> 1; jj > 0; jj >>= 1) {
      const float o = __shfl_xor_sync(kAll, sv, jj);
      const bool up = (lane & kk) == 0, lower = (lane & jj) == 0;
      sv = (lower == up) ? fminf(sv, o) : fmaxf(sv, o);
    }
  }
  const float wm = __shfl_sync(kAll, sv, 31);
  const float wt = __shfl_sync(kAll, sv, 32 - A.kw);
  if (lane == 0) { w_max[warp] = wm; w_tau[warp] = wt; }
  __syncthreads();
  float m = w_max[0], tau = w_tau[0];
#pragma unroll
  for (int w = 1; w < kThreads / 32; w++) { m = fmaxf(m, w_max[w]); tau = fminf(tau, w_tau[w]); }

  // ---- pass B: fast exp sum (Kahan in fp32) and candidates >= tau
  const float mref = (m == -INFINITY) ? 0.f : m;
  const float a = A.a;
  float s = 0.f, comp = 0.f;
  const bool partial = n < kChunk;
  const unsigned lt_mask = (1u << lane) - 1u;
  auto append = [&](bool pred, float x, int idx) {
    const unsigned msk = __ballot_sync(kAll, pred);
    if (msk) {
      const int leader = __ffs(msk) - 1;
      int base = 0;
      if (lane == leader) base = atomicAdd(&ccount, __popc(msk));
      base = __shfl_sync(kAll, base, leader);
      if (pred) {
        const int pos = base + __popc(msk & lt_mask);
        if (pos < kCap) clist[pos] = Cand{x, idx};
      }
    }
  };
#pragma unroll 2
  for (int i = 0; i < kIters; i++) {
    const int q = tid + i * kThreads;
    const float4 v = t4[q];
    const int j = 4 * q;
    float e0 = term_fast(v.x, mref, a), e1 = term_fast(v.y, mref, a);
    float e2 = term_fast(v.z, mref, a), e3 = term_fast(v.w, mref, a);
    if (partial) {
      if (j >= n) e0 = 0.f;
      if (j + 1 >= n) e1 = 0.f;
      if (j + 2 >= n) e2 = 0.f;
      if (j + 3 >= n) e3 = 0.f;
    }
    const float t = __fadd_rn(__fadd_rn(e0, e1), __fadd_rn(e2, e3));
    const float y = __fsub_rn(t, comp);
    const float ss = __fadd_rn(s, y);
    comp = __fsub_rn(__fsub_rn(ss, s), y);
    s = ss;
    const bool p0 = v.x >= tau, p1 = v.y >= tau, p2 = v.z >= tau, p3 = v.w >= tau;
    if (__any_sync(kAll, p0 || p1 || p2 || p3)) {
      append(p0 && j < n, v.x, c0 + j);
      append(p1 && j + 1 < n, v.y, c0 + j + 1);
      append(p2 && j + 2 < n, v.z, c0 + j + 2);
      append(p3 && j + 3 < n, v.w, c0 + j + 3);
    }
  }
  double ds = (double)s - (double)comp;
  ds = warp_sum(ds);
  if (lane == 0) w_sum[warp] = ds;
  __syncthreads();
  const int nc = min(ccount, kCap);
  Cand* dst = A.cands + ((int64_t)r * A.n_chunks + c) * kCap;
  for (int j = tid; j < nc; j += kThreads) dst[j] = clist[j];
  if (tid == 0) {
    double S = 0.0;
    for (int w = 0; w < kThreads / 32; w++) S += w_sum[w];
    ChunkStat st;
    st.m = m; st.tau = tau; st.s = S; st.n_cand = ccount; st.best_i = INT_MAX; st.best_v = m; st.pad = 0;
    A.stats[(int64_t)r * A.n_chunks + c] = st;
  }
}

// =============================================================== full-row path
struct RowInfo {
  const float* row;
  int V;
  const uint32_t* pb;  // penalty bitmap of the row (null: no penalty)
  double pen;
  float M;             // max of the penalised row
  float Mp;            // fp32(M / T): the reference's mx
  double S;            // softmax denominator
  float a;
  double mscale;       // fast mass of x = term_fast(x, M, a) * mscale  (~ prob)
  double T;
  int temper;
};

struct SelShared {
  int cnt[256];
  double mass[256];
  double above;
  uint32_t prefix;
  double total_w;      // weight of all non-NaN elements (first round)
  int red_i[kThreads / 32];
  int red_i2[kThreads / 32];
  double red_d[kThreads / 32];
  unsigned long long pre[kThreads];
  int result;
};

__device__ __forceinline__ float load_x(const RowInfo& R, int i) {
  float v = __ldg(R.row + i);
  if (R.pb && ((R.pb[i >> 5] >> (i & 31)) & 1u)) v = pen_apply(v, R.pen);
  return v;
}
__device__ __forceinline__ double mass_fast(const RowInfo& R, float x) {
  return (double)term_fast(x, R.M, R.a) * R.mscale;
}
__device__ __forceinline__ float prob_of(const RowInfo& R, float x) {
  return prob_exact(term_exact(temper_exact(x, R.T, R.temper), R.Mp), R.S);
}

// Value v of the row such that W(x > v) < target <= W(x >= v), where W counts
// elements (by_mass false) or sums their fast probability mass.  Only
// non-empty buckets qualify; a target above the total selects the smallest
// element.  *above_out = W(x > v).
__device__ float radix_select(const RowInfo& R, bool by_mass, double target, SelShared& sh,
                              double* above_out) {
  const int tid = threadIdx.x;
  uint32_t prefix = 0, pmask = 0;
  double above = 0.0;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int d = tid; d < 256; d += kThreads) { sh.cnt[d] = 0; sh.mass[d] = 0.0; }
    __syncthreads();
    for (int i = tid; i < R.V; i += kThreads) {
      const float x = load_x(R, i);
      if (x != x) continue;
      const uint32_t k = fkey(x);
      if ((k & pmask) == prefix) {
        const int d = (k >> shift) & 255;
        atomicAdd(&sh.cnt[d], 1);
        if (by_mass) atomicAdd(&sh.mass[d], mass_fast(R, x));
      }
    }
    __syncthreads();
    if (tid == 0) {
      double cum = above;
      int chosen = -1, last = -1;
      double tot = 0.0;
      for (int d = 255; d >= 0; d--) tot += by_mass ? sh.mass[d] : (double)sh.cnt[d];
      if (shift == 24) sh.total_w = tot;
      for (int d = 255; d >= 0; d--) {
        if (sh.cnt[d] == 0) continue;
        last = d;
        const double w = by_mass ? sh.mass[d] : (double)sh.cnt[d];
        if (cum + w >= target) { chosen = d; break; }
        cum += w;
      }
      if (chosen < 0) {
        chosen = last < 0 ? 0 : last;
        if (last >= 0) cum -= by_mass ? sh.mass[chosen] : (double)sh.cnt[chosen];
      }
      sh.above = cum;
      sh.prefix = prefix | ((uint32_t)chosen << shift);
    }
    __syncthreads();
    above = sh.above;
    prefix = sh.prefix;
    pmask |= 0xFFu << shift;
    __syncthreads();
  }
  *above_out = above;
  return fkey_inv(prefix);
}

// Keys [lo, hi] with pred(lo) true and pred monotone (true, then false as the
// key grows): returns the largest key with pred true.  Warp 0 evaluates 32
// probes per round.  `dir` -1 searches downward (pred true at hi, returns the
// smallest key with pred true).
template <typename Pred>
__device__ uint32_t warp_boundary_search(uint32_t lo, uint32_t hi, int dir, Pred pred) {
  const int lane = threadIdx.x & 31;
  // map so that we always search "largest true" over [0, span]
  const uint64_t base = dir > 0 ? lo : hi;
  uint64_t L = 0, H = (uint64_t)hi - lo;
  while (H > L) {
    const uint64_t step = (H - L + 31) / 32;
    uint64_t p = L + (uint64_t)(lane + 1) * step;
    if (p > H) p = H;
    const uint32_t key = dir > 0 ? (uint32_t)(base + p) : (uint32_t)(base - p);
    const bool t = pred(key);
    const unsigned msk = __ballot_sync(kAll, t);
    // msk is a prefix of lanes (monotone predicate)
    const int ntrue = __popc(msk);
    const uint64_t p_last = __shfl_sync(kAll, p, ntrue > 0 ? ntrue - 1 : 0);
    const uint64_t p_next = __shfl_sync(kAll, p, ntrue < 32 ? ntrue : 31);
    if (ntrue == 0) {
      H = p_next - 1;  // p_next is lane 0's probe here
    } else {
      L = p_last;
      if (ntrue < 32) H = p_next - 1;
      else if (p_last >= H) H = L;
    }
  }
  return dir > 0 ? (uint32_t)(base + L) : (uint32_t)(base - L);
}

struct GroupSel {
  int index;       // vocabulary id of the selected element
  int64_t rank;    // 1-based position in (prob desc, id asc) order
  double cum;      // fast cumulative mass through it
  double mass_hi;  // fast mass strictly above its tie group
  int64_t cnt_hi;  // elements strictly above its tie group
  float p;         // its exact probability
};

// Resolve the tie group of v (all x with prob_of(x) == prob_of(v)), then the
// element reaching `target` (count or fast mass) inside it in id order.
__device__ GroupSel resolve_group(const RowInfo& R, float v, bool by_mass, double target,
                                  SelShared& sh) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __shared__ float s_lohi[2];
  __shared__ float s_p;
  if (warp == 0) {
    const float pv = prob_of(R, v);
    const uint32_t kv = fkey(v);
    const uint32_t kM = fkey(R.M) > kv ? fkey(R.M) : kv;
    const uint32_t kNegInf = fkey(-INFINITY);
    auto same = [&](uint32_t key) { return prob_of(R, fkey_inv(key)) == pv; };
    const uint32_t khi = warp_boundary_search(kv, kM, +1, same);
    const uint32_t klo = warp_boundary_search(kNegInf <= kv ? kNegInf : kv, kv, -1, same);
    if (lane == 0) { s_lohi[0] = fkey_inv(klo); s_lohi[1] = fkey_inv(khi); s_p = pv; }
  }
  __syncthreads();
  const float xlo = s_lohi[0], xhi = s_lohi[1], pstar = s_p;
  // counts above / inside the group, fast mass above
  int c_hi = 0, c_g = 0;
  double m_hi = 0.0;
  for (int i = tid; i < R.V; i += kThreads) {
    const float x = load_x(R, i);
    if (x > xhi) { c_hi++; m_hi += mass_fast(R, x); }
    else if (x >= xlo) c_g++;
  }
  c_hi = warp_sum_i(c_hi);
  c_g = warp_sum_i(c_g);
  m_hi = warp_sum(m_hi);
  if (lane == 0) { sh.red_i[warp] = c_hi; sh.red_i2[warp] = c_g; sh.red_d[warp] = m_hi; }
  __syncthreads();
  int64_t CH = 0, CG = 0;
  double MH = 0.0;
  for (int w = 0; w < kThreads / 32; w++) { CH += sh.red_i[w]; CG += sh.red_i2[w]; MH += sh.red_d[w]; }
  __syncthreads();
  int64_t j;
  if (by_mass) {
    const double need = target - MH;
    if (need <= 0.0) j = 1;
    else if (pstar > 0.f) j = (int64_t)ceil(need / (double)pstar);
    else j = CG;
  } else {
    j = (int64_t)target - CH;
  }
  if (j < 1) j = 1;
  if (j > CG) j = CG;
  // j-th group element in id order: contiguous segment per thread, scan.
  const int seg = (R.V + kThreads - 1) / kThreads;
  const int s0 = min(R.V, tid * seg), s1 = min(R.V, s0 + seg);
  int cnt = 0;
  for (int i = s0; i < s1; i++) {
    const float x = load_x(R, i);
    cnt += (x >= xlo && x <= xhi);
  }
  sh.pre[tid] = (unsigned long long)cnt;
  if (tid == 0) sh.result = -1;
  __syncthreads();
  if (tid == 0) {
    unsigned long long run = 0;
    for (int t = 0; t < kThreads; t++) { const unsigned long long c = sh.pre[t]; sh.pre[t] = run; run += c; }
  }
  __syncthreads();
  const int64_t before = (int64_t)sh.pre[tid];
  if (before < j && before + cnt >= j) {
    int64_t need = j - before;
    for (int i = s0; i < s1; i++) {
      const float x = load_x(R, i);
      if (x >= xlo && x <= xhi && --need == 0) { sh.result = i; break; }
    }
  }
  __syncthreads();
  GroupSel gsel;
  gsel.index = sh.result < 0 ? 0 : sh.result;
  gsel.rank = CH + j;
  gsel.cum = MH + (double)j * (double)pstar;
  gsel.mass_hi = MH;
  gsel.cnt_hi = CH;
  gsel.p = pstar;
  __syncthreads();
  return gsel;
}

__device__ GroupSel select_rank(const RowInfo& R, int64_t k, SelShared& sh) {
  double above;
  const float v = radix_select(R, false, (double)k, sh, &above);
  return resolve_group(R, v, false, (double)k, sh);
}
__device__ GroupSel select_mass(const RowInfo& R, double target, SelShared& sh) {
  double above;
  const float v = radix_select(R, true, target, sh, &above);
  return resolve_group(R, v, true, target, sh);
}

// Exact top-k / top-p / draw over the whole row (src/generation.js:27-49).
__device__ void full_path(const Args& A, int r, const RowInfo& R, SelShared& sh, int flags) {
  const int tid = threadIdx.x;
  const int V = R.V;
  const bool use_k = A.k > 0 && A.k < V;
  int64_t n;
  double mass_n;
  int last_id;  // id at rank n (fallback of the draw loop)
  if (use_k) {
    const GroupSel gk = select_rank(R, A.k, sh);
    n = A.k;
    mass_n = gk.cum;
    last_id = gk.index;
  } else {
    double t = 0.0;
    for (int i = tid; i < V; i += kThreads) {
      const float x = load_x(R, i);
      if (x == x) t += mass_fast(R, x);
    }
    t = warp_sum(t);
    if ((tid & 31) == 0) sh.red_d[tid >> 5] = t;
    __syncthreads();
    mass_n = 0.0;
    for (int w = 0; w < kThreads / 32; w++) mass_n += sh.red_d[w];
    __syncthreads();
    n = V;
    last_id = -1;
  }
  double total = mass_n;
  if (A.use_topp && mass_n >= A.top_p) {
    const GroupSel gp = select_mass(R, A.top_p, sh);
    if (gp.rank < n) {
      n = gp.rank < 1 ? 1 : gp.rank;
      total = gp.cum;
      last_id = gp.index;
    }
  }
  if (last_id < 0) {
    const GroupSel gl = select_rank(R, n, sh);
    last_id = gl.index;
  }
  const double u = A.u ? A.u[r] : 0.0;
  const double rr = u * total;
  int id;
  if (rr <= 0.0) {
    id = select_rank(R, 1, sh).index;
  } else {
    const GroupSel gd = select_mass(R, rr, sh);
    id = (gd.rank > n) ? last_id : gd.index;
  }
  if (tid == 0) {
    A.out_ids[r] = id;
    if (A.d_n_cand) A.d_n_cand[r] = (int32_t)n;
    if (A.d_total) A.d_total[r] = total;
    if (A.d_row_flags) A.d_row_flags[r] = flags | MS_ROW_FULLVOCAB;
  }
}

// =============================================================== finalize kernel
struct FinShared {
  unsigned long long keys[kNfMax];
  SelShared sel;
  int nf;
  int slow;
  unsigned long long corr;  // fixed-point (2^-50) sum of the candidate corrections
  double S;
  float M, Mp, tau_row;
  int nan_row, overflow;
  double scale0;
};

__device__ __forceinline__ double chunk_scale(const Args& A, float mc, float Mp) {
  // exp(m_c / T - M'): converts a chunk's fast terms to the reference's units
  return (mc == -INFINITY) ? 0.0 : exp((double)mc / A.T - (double)Mp);
}

template <int MODE>
__global__ void __launch_bounds__(kThreads) finalize_kernel(const Args A) {
  extern __shared__ __align__(16) unsigned char fin_smem[];
  FinShared& sh = *reinterpret_cast<FinShared*>(fin_smem);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r = blockIdx.x;
  const ChunkStat* st = A.stats + (int64_t)r * A.n_chunks;

  if (MODE == kGreedy) {
    if (tid == 0) {
      float bv = -INFINITY;
      int bi = INT_MAX;
      for (int c = 0; c < A.n_chunks; c++) {
        const ChunkStat s = st[c];
        if (s.best_v > bv || (s.best_v == bv && s.best_i < bi)) { bv = s.best_v; bi = s.best_i; }
      }
      const float x0 = A.logits[(int64_t)r * A.ld];
      const int id = (x0 != x0 || bv == -INFINITY || bi == INT_MAX) ? 0 : bi;
      A.out_ids[r] = id;
      if (A.d_row_flags) A.d_row_flags[r] = MS_ROW_GREEDY;
      if (A.d_n_cand) A.d_n_cand[r] = 0;
      if (A.d_row_max) A.d_row_max[r] = (double)bv;
    }
    return;
  }

  // ---- row max, NaN detection, overflow, tau_row
  if (tid == 0) {
    float M = -INFINITY, tr = -INFINITY;
    int nanr = 0, ovf = 0;
    for (int c = 0; c < A.n_chunks; c++) {
      const ChunkStat s = st[c];
      M = fmaxf(M, s.m);
      tr = fmaxf(tr, s.tau);
      if (s.s != s.s) nanr = 1;
      if (s.n_cand > kCap) ovf = 1;
    }
    const float Mp = temper_exact(M, A.T, A.temper);
    if (M == -INFINITY || isinf(Mp) || Mp != Mp) nanr = 1;
    sh.M = M; sh.Mp = Mp; sh.tau_row = tr; sh.nan_row = nanr; sh.overflow = ovf;
    sh.nf = 0; sh.slow = ovf; sh.corr = 0ull;
    if (!nanr) {
      double S = 0.0;
      for (int c = 0; c < A.n_chunks; c++) {
        const ChunkStat s = st[c];
        if (s.m != -INFINITY) S += s.s * chunk_scale(A, s.m, Mp);
      }
      sh.S = S;
      sh.scale0 = exp((double)M / A.T - (double)Mp);
    }
  }
  __syncthreads();
  const int V = A.V;
  if (sh.nan_row) {
    // softmax is NaN everywhere: the stable sort keeps id order, no acc reaches
    // topP, r is NaN, and the draw loop falls through to the last candidate.
    if (tid == 0) {
      const bool use_k = A.k > 0 && A.k < V;
      A.out_ids[r] = use_k ? A.k - 1 : V - 1;
      if (A.d_n_cand) A.d_n_cand[r] = use_k ? A.k : V;
      if (A.d_row_max) A.d_row_max[r] = (double)sh.Mp;
      if (A.d_row_sum) A.d_row_sum[r] = __longlong_as_double(0x7ff8000000000000ll);
      if (A.d_total) A.d_total[r] = __longlong_as_double(0x7ff8000000000000ll);
      if (A.d_row_flags) A.d_row_flags[r] = MS_ROW_NAN;
    }
    return;
  }
  const float M = sh.M, Mp = sh.Mp, tau_row = sh.tau_row;

  // ---- gather candidates >= tau_row (complete unless a chunk overflowed)
  Cand* gath = reinterpret_cast<Cand*>(sh.keys);
  for (int c = 0; c < A.n_chunks; c++) {
    const int nc = min(st[c].n_cand, kCap);
    const Cand* src = A.cands + ((int64_t)r * A.n_chunks + c) * kCap;
    for (int j = tid; j < nc; j += kThreads) {
      const Cand cd = src[j];
      if (cd.x >= tau_row) {
        const int pos = atomicAdd(&sh.nf, 1);
        if (pos < kNfMax) gath[pos] = cd;
      }
    }
  }
  __syncthreads();
  const int nf = sh.nf;
  if (nf > kNfMax) { if (tid == 0) sh.slow = 1; }
  // ---- exact terms of the candidates; correct the fast sum with them
  const int nfc = min(nf, kNfMax);
  for (int j = tid; j < nfc; j += kThreads) {
    const Cand cd = gath[j];
    const int c = cd.i / kChunk;
    const float mc = st[c].m;
    const float e = term_exact(temper_exact(cd.x, A.T, A.temper), Mp);
    const double fast = (double)term_fast(cd.x, mc, A.a) * chunk_scale(A, mc, Mp);
    const double corr = (double)e - fast;
    atomicAdd(&sh.corr, (unsigned long long)__double2ll_rn(corr * 1125899906842624.0));  // 2^50
  }
  __syncthreads();
  if (tid == 0) sh.S = sh.S + (double)(long long)sh.corr * (1.0 / 1125899906842624.0);
  __syncthreads();
  const double S = sh.S;

  RowInfo R;
  R.row = A.logits + (int64_t)r * A.ld;
  R.V = V;
  R.pb = nullptr;
  R.pen = A.pen;
  R.M = M;
  R.Mp = Mp;
  R.S = S;
  R.a = A.a;
  R.mscale = sh.scale0 / S;
  R.T = A.T;
  R.temper = A.temper;

  if (MODE == kTopK && !sh.slow) {
    // keys: (prob desc, id asc) as ascending 64-bit keys
    for (int j = tid; j < nfc; j += kThreads) {
      const Cand cd = gath[j];
      const float p = prob_exact(term_exact(temper_exact(cd.x, A.T, A.temper), Mp), S);
      sh.keys[j] = ((unsigned long long)(0xFFFFFFFFu - __float_as_uint(p)) << 32) | (uint32_t)cd.i;
    }
    int np2 = 1;
    while (np2 < nfc) np2 <<= 1;
    for (int j = nfc + tid; j < np2; j += kThreads) sh.keys[j] = ~0ull;
    __syncthreads();
    // bitonic sort ascending
    for (int kk = 2; kk <= np2; kk <<= 1) {
      for (int jj = kk >> 1; jj > 0; jj >>= 1) {
        for (int i = tid; i < np2; i += kThreads) {
          const int ixj = i ^ jj;
          if (ixj > i) {
            const unsigned long long x = sh.keys[i], y = sh.keys[ixj];
            const bool asc = (i & kk) == 0;
            if ((x > y) == asc) { sh.keys[i] = y; sh.keys[ixj] = x; }
          }
        }
        __syncthreads();
      }
    }
    // completeness: every element outside the list has prob <= prob(pred(tau_row))
    if (tid == 0) {
      const int k = A.k;
      if (nfc < k) {
        sh.slow = 1;
      } else if (tau_row != -INFINITY) {
        const float pk = __uint_as_float(0xFFFFFFFFu - (uint32_t)(sh.keys[k - 1] >> 32));
        const float below = fkey_inv(fkey(tau_row) - 1u);
        const float pout = prob_of(R, below);
        if (!(pk > pout)) sh.slow = 1;
      }
    }
    __syncthreads();
    if (!sh.slow) {
      if (tid == 0) {
        // src/generation.js:32-48, sequential fp64 as in the reference
        int n = A.k;
        if (A.use_topp) {
          double acc = 0.0;
          int cut = n;
          for (int i = 0; i < n; i++) {
            acc += (double)__uint_as_float(0xFFFFFFFFu - (uint32_t)(sh.keys[i] >> 32));
            if (acc >= A.top_p) { cut = i + 1; break; }
          }
          n = cut > 1 ? cut : 1;
        }
        double total = 0.0;
        for (int i = 0; i < n; i++) total += (double)__uint_as_float(0xFFFFFFFFu - (uint32_t)(sh.keys[i] >> 32));
        double rr = (A.u ? A.u[r] : 0.0) * total;
        int id = (int)(uint32_t)sh.keys[n - 1];
        for (int i = 0; i < n; i++) {
          rr -= (double)__uint_as_float(0xFFFFFFFFu - (uint32_t)(sh.keys[i] >> 32));
          if (rr <= 0.0) { id = (int)(uint32_t)sh.keys[i]; break; }
        }
        A.out_ids[r] = id;
        if (A.d_n_cand) A.d_n_cand[r] = n;
        if (A.d_total) A.d_total[r] = total;
        if (A.d_row_max) A.d_row_max[r] = (double)Mp;
        if (A.d_row_sum) A.d_row_sum[r] = S;
        if (A.d_row_flags) A.d_row_flags[r] = 0;
        sh.nf = n;
      }
      __syncthreads();
      if (A.d_cand_ids || A.d_cand_probs) {
        const int n = sh.nf;
        for (int i = tid; i < n && i < A.cand_cap; i += kThreads) {
          const unsigned long long kkey = sh.keys[i];
          if (A.d_cand_ids) A.d_cand_ids[(int64_t)r * A.cand_cap + i] = (int32_t)(uint32_t)kkey;
          if (A.d_cand_probs)
            A.d_cand_probs[(int64_t)r * A.cand_cap + i] = __uint_as_float(0xFFFFFFFFu - (uint32_t)(kkey >> 32));
        }
      }
      return;
    }
  }

  // ---- exact rescan of the whole row
  int flags = (MODE == kTopK) ? MS_ROW_SLOWPATH : 0;
  if (A.use_pen && A.penbits) {
    const int W = (V + 31) >> 5;
    uint32_t* pb = A.penbits + (int64_t)r * W;
    for (int w = tid; w < W; w += kThreads) pb[w] = 0u;
    __syncthreads();
    const int64_t h0 = A.hist_off[r], h1 = A.hist_off[r + 1];
    for (int64_t h = h0 + tid; h < h1; h += kThreads) {
      const int id = A.hist[h];
      if (id >= 0 && id < V) atomicOr(&pb[id >> 5], 1u << (id & 31));
    }
    __syncthreads();
    R.pb = pb;
  }
  if (tid == 0) {
    if (A.d_row_max) A.d_row_max[r] = (double)Mp;
    if (A.d_row_sum) A.d_row_sum[r] = S;
  }
  full_path(A, r, R, sh.sel, flags);
  (void)lane; (void)warp;
}

// explicit instantiations
template __global__ void chunk_kernel<kGreedy, false>(const Args);
template __global__ void chunk_kernel<kGreedy, true>(const Args);
template __global__ void chunk_kernel<kTopK, false>(const Args);
template __global__ void chunk_kernel<kTopK, true>(const Args);
template __global__ void chunk_kernel<kFull, false>(const Args);
template __global__ void chunk_kernel<kFull, true>(const Args);
template __global__ void finalize_kernel<kGreedy>(const Args);
template __global__ void finalize_kernel<kTopK>(const Args);
template __global__ void finalize_kernel<kFull>(const Args);

// =============================================================== launch
size_t finalize_smem_bytes() { return sizeof(FinShared); }

cudaError_t launch_sample(const Args& A, cudaStream_t stream, cudaEvent_t* ev) {
  const dim3 block(kThreads);
  const size_t chunk_smem = (size_t)kChunk * sizeof(float);
  const size_t fin_smem = sizeof(FinShared);
  static bool attrs_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attrs_done[dev]) {
#define MS_SET_ATTR(fn, bytes)                                                                   \
  do {                                                                                           \
    cudaError_t e_ = cudaFuncSetAttribute((const void*)fn, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                          (int)(bytes));                                         \
    if (e_ != cudaSuccess) return e_;                                                            \
  } while (0)
    MS_SET_ATTR((chunk_kernel<kGreedy, false>), chunk_smem);
    MS_SET_ATTR((chunk_kernel<kGreedy, true>), chunk_smem);
    MS_SET_ATTR((chunk_kernel<kTopK, false>), chunk_smem);
    MS_SET_ATTR((chunk_kernel<kTopK, true>), chunk_smem);
    MS_SET_ATTR((chunk_kernel<kFull, false>), chunk_smem);
    MS_SET_ATTR((chunk_kernel<kFull, true>), chunk_smem);
    MS_SET_ATTR(finalize_kernel<kGreedy>, fin_smem);
    MS_SET_ATTR(finalize_kernel<kTopK>, fin_smem);
    MS_SET_ATTR(finalize_kernel<kFull>, fin_smem);
#undef MS_SET_ATTR
    attrs_done[dev] = true;
  }
  // rows in slices of at most 65535 (grid.y limit)
  for (int64_t r0 = 0; r0 < A.B; r0 += 65535) {
    Args S = A;
    const int rows = (int)((A.B - r0) < 65535 ? (A.B - r0) : 65535);
    S.B = rows;
    S.logits = A.logits + r0 * A.ld;
    if (A.hist_off) S.hist_off = A.hist_off + r0;
    if (A.u) S.u = A.u + r0;
    S.stats = A.stats + r0 * A.n_chunks;
    S.cands = A.cands + r0 * A.n_chunks * kCap;
    if (A.penbits) S.penbits = A.penbits + r0 * ((A.V + 31) / 32);
    S.out_ids = A.out_ids + r0;
    if (A.d_cand_ids) S.d_cand_ids = A.d_cand_ids + r0 * A.cand_cap;
    if (A.d_cand_probs) S.d_cand_probs = A.d_cand_probs + r0 * A.cand_cap;
    if (A.d_n_cand) S.d_n_cand = A.d_n_cand + r0;
    if (A.d_row_max) S.d_row_max = A.d_row_max + r0;
    if (A.d_row_sum) S.d_row_sum = A.d_row_sum + r0;
    if (A.d_total) S.d_total = A.d_total + r0;
    if (A.d_row_flags) S.d_row_flags = A.d_row_flags + r0;
    const dim3 grid_c(A.n_chunks, rows);
    const bool pen = A.use_pen != 0;
    const bool prof = ev != nullptr && r0 == 0 && A.B <= 65535;
    if (prof) cudaEventRecord(ev[0], stream);
    switch (A.mode) {
      case kGreedy:
        if (pen) chunk_kernel<kGreedy, true><<<grid_c, block, chunk_smem, stream>>>(S);
        else chunk_kernel<kGreedy, false><<<grid_c, block, chunk_smem, stream>>>(S);
        if (prof) cudaEventRecord(ev[1], stream);
        finalize_kernel<kGreedy><<<rows, block, 0, stream>>>(S);
        break;
      case kTopK:
        if (pen) chunk_kernel<kTopK, true><<<grid_c, block, chunk_smem, stream>>>(S);
        else chunk_kernel<kTopK, false><<<grid_c, block, chunk_smem, stream>>>(S);
        if (prof) cudaEventRecord(ev[1], stream);
        finalize_kernel<kTopK><<<rows, block, fin_smem, stream>>>(S);
        break;
      default:
        if (pen) chunk_kernel<kFull, true><<<grid_c, block, chunk_smem, stream>>>(S);
        else chunk_kernel<kFull, false><<<grid_c, block, chunk_smem, stream>>>(S);
        if (prof) cudaEventRecord(ev[1], stream);
        finalize_kernel<kFull><<<rows, block, fin_smem, stream>>>(S);
        break;
    }
    if (prof) cudaEventRecord(ev[2], stream);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace ms
