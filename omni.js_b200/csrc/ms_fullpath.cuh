// Exact top-k / top-p / draw over a whole row (src/generation.js:27-49), for
// the rows the candidate path cannot settle: top_k off (<= 0 or >= V), top_k
// larger than the candidate path takes, or a candidate set that could not be
// proven complete.  One CTA (the row's finalizer) runs it on the row in HBM/L2.
//
// Order is (prob desc, id asc) with the reference's exact fp32 probabilities.
// A selection finds the element at a given rank, or where the running
// probability mass reaches a target, by range refinement:
//   level 0  1024 buckets, 1/16 nat wide, below the row max (one pass, kept
//            for every selection of the row);
//   level 1  1024 buckets splitting the chosen level-0 bucket (one pass);
//   key      if that bucket still holds more than kExtCap elements, its exact
//            key range is split 1024 ways, repeatedly (one pass each);
//   extract  the elements of the final range, widened to whole probability-tie
//            groups, go to shared memory, are ranked by exact (prob, id) and
//            resolved (one pass).
// Bucket membership is monotone in the logit, so every bucket is an interval
// of logits; cumulative masses above the final range use the fast fp32 terms,
// masses inside it the exact probabilities.
#pragma once
#include "ms_device.cuh"

namespace ms {

constexpr int kBins = 1024;      // buckets per refinement level
constexpr int kExtCap = 1024;    // elements resolved exactly in shared memory
constexpr int kFWarps = kThreads / 32;  // most warps a row CTA has

struct RowInfo {
  const float* row;
  int V;
  const uint32_t* pb;  // penalty bitmap of the row (null: no penalty)
  double pen, rpen;
  float M;             // max of the penalised row
  float Mp;            // fp32(M / T): the reference's mx
  double S;            // softmax denominator
  float a;             // fp32(log2(e) / T)
  double mscale;       // fast mass of x = term_fast(x, M, a) * mscale  (~ prob)
  float nat16;         // fp32(16 / T): level-0 buckets per logit unit
  double T;
  int temper;
  double rT, rS;       // fp64(1 / T), fp64(1 / S): divides by multiplication (exact-divide fallback)
};

struct Hist {
  int cnt[kBins];
  double mass[kBins];
  uint32_t kmin[kBins], kmax[kBins];
};

struct FullSmem {
  Hist h0;                          // level 0, kept for the whole row
  Hist h1;                          // deeper levels
  unsigned long long key[kExtCap];  // exact (prob desc, id asc) keys of the final range
  int n_ext;
  int sel_bin;
  long long above_c;
  double above_m;
  uint32_t klo, khi;
  int red_i[kFWarps];
  long long red_l[kFWarps];
  double red_d[kFWarps];
  int result;
  long long rank_out;
  double cum_out;
};

__device__ __forceinline__ float load_x(const RowInfo& R, int i) {
  float v = __ldg(R.row + i);
  if (R.pb && ((R.pb[i >> 5] >> (i & 31)) & 1u)) v = pen_apply_fast(v, R.pen, R.rpen);
  return v;
}
__device__ __forceinline__ double mass_fast(const RowInfo& R, float x) {
  return (double)term_fast(x, R.M, R.a) * R.mscale;
}
// The reference's probability of logit x: fp32(fp32(exp(fp32(x / T) - mx)) / sum),
// each divide a multiplication by the reciprocal unless the product sits next
// to an fp32 rounding midpoint (div_to_f32), so the result is the same.
__device__ __forceinline__ float prob_of(const RowInfo& R, float x) {
  return div_to_f32((double)term_exact(temper_fast(x, R.T, R.rT, R.temper), R.Mp), R.S, R.rS);
}
__device__ __forceinline__ int bin0(const RowInfo& R, float x) {
  // 1/16-nat buckets below the max; monotone (non-increasing) in x
  const float t = __fmul_rn(__fsub_rn(R.M, x), R.nat16);
  return t < (float)(kBins - 1) ? (int)t : kBins - 1;
}
__device__ __forceinline__ int bin1(const RowInfo& R, float x, int b0) {
  // 1024 sub-buckets of level-0 bucket b0; monotone (non-increasing) in x
  const float t = __fmul_rn(__fsub_rn(__fmul_rn(__fsub_rn(R.M, x), R.nat16), (float)b0), (float)kBins);
  return t <= 0.f ? 0 : (t < (float)(kBins - 1) ? (int)t : kBins - 1);
}

// Calls f(x, i) for every element of the row (penalised), 16-byte vector loads
// when the row allows, four loads in flight per thread.
template <typename F>
__device__ __forceinline__ void for_row(const RowInfo& R, F f) {
  const int tid = threadIdx.x;
  if ((reinterpret_cast<uintptr_t>(R.row) & 15) == 0) {
    const int V4 = R.V >> 2;
    const float4* r4 = reinterpret_cast<const float4*>(R.row);
    for (int q0 = tid; q0 < V4; q0 += 4 * (int)blockDim.x) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int q = q0 + u * (int)blockDim.x;
        v[u] = q < V4 ? __ldg(r4 + q) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int q = q0 + u * (int)blockDim.x;
        if (q >= V4) break;
        const int i = 4 * q;
        float e[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
        if (R.pb) {
          const uint32_t bits = (R.pb[i >> 5] >> (i & 31)) & 0xFu;
          if (bits) {
#pragma unroll
            for (int t = 0; t < 4; t++)
              if ((bits >> t) & 1u) e[t] = pen_apply_fast(e[t], R.pen, R.rpen);
          }
        }
#pragma unroll
        for (int t = 0; t < 4; t++) f(e[t], i + t);
      }
    }
    for (int i = 4 * V4 + tid; i < R.V; i += (int)blockDim.x) f(load_x(R, i), i);
  } else {
    for (int i = tid; i < R.V; i += (int)blockDim.x) f(load_x(R, i), i);
  }
}

// Keys [lo, hi] with pred(lo) true and pred monotone (true, then false as the
// key grows): returns the largest key with pred true.  One warp: a first round
// probes the offsets 2^0 .. 2^31 from the start (a probability-tie group
// usually spans few keys), then each round splits what is left 32 ways.  `dir`
// -1 searches downward (pred true at hi, returns the smallest key with pred true).
template <typename Pred>
__device__ uint32_t warp_boundary_search(uint32_t lo, uint32_t hi, int dir, Pred pred) {
  const int lane = threadIdx.x & 31;
  const uint64_t base = dir > 0 ? lo : hi;
  uint64_t L = 0, H = (uint64_t)hi - lo;
  auto at = [&](uint64_t p) { return dir > 0 ? (uint32_t)(base + p) : (uint32_t)(base - p); };
  if (H > 0) {  // galloping round
    const uint64_t p = min((uint64_t)1 << lane, H);
    const unsigned msk = __ballot_sync(0xffffffffu, pred(at(p)));
    const int ntrue = __popc(msk);  // pred is monotone: the lanes below the boundary
    if (ntrue > 0) L = min((uint64_t)1 << (ntrue - 1), H);
    if (ntrue < 32) H = min((uint64_t)1 << ntrue, H) - 1;
    if (L > H) H = L;
  }
  while (H > L) {
    const uint64_t step = (H - L + 31) / 32;
    uint64_t p = L + (uint64_t)(lane + 1) * step;
    if (p > H) p = H;
    const bool t = pred(at(p));
    const unsigned msk = __ballot_sync(0xffffffffu, t);
    const int ntrue = __popc(msk);
    const uint64_t p_last = __shfl_sync(0xffffffffu, p, ntrue > 0 ? ntrue - 1 : 0);
    const uint64_t p_next = __shfl_sync(0xffffffffu, p, ntrue < 32 ? ntrue : 31);
    if (ntrue == 0) {
      H = p_next - 1;
    } else {
      L = p_last;
      if (ntrue < 32) H = p_next - 1;
      else if (p_last >= H) H = L;
    }
  }
  return at(L);
}

// Smallest / largest x with prob_of(x) == prob_of(v); one full warp.  The
// search runs only when the neighbouring fp32 value shares v's probability.
__device__ float tie_low(const RowInfo& R, float v) {
  if (v == -INFINITY) return v;
  const float pv = prob_of(R, v);
  if (prob_of(R, fkey_inv(fkey(v) - 1u)) < pv) return v;
  const uint32_t kv = fkey(v);
  const uint32_t kNegInf = fkey(-INFINITY);
  auto same = [&](uint32_t key) { return prob_of(R, fkey_inv(key)) == pv; };
  return fkey_inv(warp_boundary_search(kNegInf <= kv ? kNegInf : kv, kv, -1, same));
}
__device__ float tie_high(const RowInfo& R, float v) {
  const uint32_t kv = fkey(v), kM = fkey(R.M);
  if (kv >= kM) return v;
  const float pv = prob_of(R, v);
  if (prob_of(R, fkey_inv(kv + 1u)) > pv) return v;
  auto same = [&](uint32_t key) { return prob_of(R, fkey_inv(key)) == pv; };
  return fkey_inv(warp_boundary_search(kv, kM, +1, same));
}


// Warp 0: the first non-empty bucket (ascending index = descending logit)
// where the running weight reaches `need`, or the last non-empty one.  pre_c /
// pre_m receive the count / fast mass of the buckets before it.
__device__ void warp_pick(const Hist& h, bool by_mass, double need, int* bin, long long* pre_c, double* pre_m) {
  const int lane = threadIdx.x & 31;
  constexpr int kPer = kBins / 32;
  long long lc = 0;
  double lm = 0.0;
  int lastne = -1;
  for (int t = 0; t < kPer; t++) {
    const int b = lane * kPer + t;
    const int c = h.cnt[b];
    lc += c;
    lm += h.mass[b];
    if (c) lastne = b;
  }
  long long ic = lc;
  double im = lm;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const long long tc = __shfl_up_sync(0xffffffffu, ic, o);
    const double tm = __shfl_up_sync(0xffffffffu, im, o);
    if (lane >= o) { ic += tc; im += tm; }
  }
  const long long ec = ic - lc;
  const double em = im - lm;
  // first lane whose buckets reach `need`
  const bool reach = lastne >= 0 && (by_mass ? (im >= need) : ((double)ic >= need));
  const unsigned rm = __ballot_sync(0xffffffffu, reach);
  int outb = -1;
  long long oc = 0;
  double om = 0.0;
  if (rm) {
    const int L = __ffs(rm) - 1;
    if (lane == L) {
      long long cc = ec;
      double mm = em;
      for (int t = 0; t < kPer; t++) {
        const int b = lane * kPer + t;
        const int c = h.cnt[b];
        if (c) {
          const double w = by_mass ? h.mass[b] : (double)c;
          if ((by_mass ? mm : (double)cc) + w >= need) { outb = b; oc = cc; om = mm; break; }
        }
        cc += c;
        mm += h.mass[b];
      }
      if (outb < 0) { outb = lastne; oc = cc - h.cnt[lastne]; om = mm - h.mass[lastne]; }
    }
    outb = __shfl_sync(0xffffffffu, outb, L);
    oc = __shfl_sync(0xffffffffu, oc, L);
    om = __shfl_sync(0xffffffffu, om, L);
  } else {
    const unsigned nm = __ballot_sync(0xffffffffu, lastne >= 0);
    const int L = nm ? 31 - __clz(nm) : 0;
    long long cc = 0;
    double mm = 0.0;
    if (lane == L && lastne >= 0) {
      cc = ic - h.cnt[lastne];
      mm = im - h.mass[lastne];
      outb = lastne;
    }
    outb = __shfl_sync(0xffffffffu, outb, L);
    oc = __shfl_sync(0xffffffffu, cc, L);
    om = __shfl_sync(0xffffffffu, mm, L);
  }
  *bin = outb < 0 ? 0 : outb;
  *pre_c = oc;
  *pre_m = om;
}

// Histogram of the elements that satisfy `in`, bucketed by `bin` (all threads).
// Masses are summed exactly as integers in units of 2^-52 (a fast mass is at
// most 1, the row's total about 1), with two 32-bit shared atomics per element
// (the low word's returned old value gives the carry into the high word;
// 64-bit shared atomics are emulated and far slower), and turned into doubles
// at the end.
template <typename In, typename Bin>
__device__ void block_hist(const RowInfo& R, Hist& h, In in, Bin binf) {
  uint32_t* mw = reinterpret_cast<uint32_t*>(h.mass);  // [2b] low word, [2b+1] high word
  for (int b = threadIdx.x; b < kBins; b += (int)blockDim.x) {
    h.cnt[b] = 0;
    mw[2 * b] = 0u;
    mw[2 * b + 1] = 0u;
    h.kmin[b] = 0xFFFFFFFFu;
    h.kmax[b] = 0u;
  }
  __syncthreads();
  for_row(R, [&](float x, int) {
    if (x != x || !in(x)) return;
    const int b = binf(x);
    const uint32_t k = fkey(x);
    atomicAdd(&h.cnt[b], 1);
    const unsigned long long m = (unsigned long long)__double2ll_rn(mass_fast(R, x) * 4503599627370496.0);
    const uint32_t lo = (uint32_t)m, hi = (uint32_t)(m >> 32);
    const uint32_t old = atomicAdd(&mw[2 * b], lo);
    const uint32_t up = hi + (old + lo < old ? 1u : 0u);
    if (up) atomicAdd(&mw[2 * b + 1], up);
    atomicMin(&h.kmin[b], k);
    atomicMax(&h.kmax[b], k);
  });
  __syncthreads();
  for (int b = threadIdx.x; b < kBins; b += (int)blockDim.x) {
    // this thread alone reads the bucket's two words and writes the double over them
    const double v = ((double)mw[2 * b + 1] * 4294967296.0 + (double)mw[2 * b]) * (1.0 / 4503599627370496.0);
    h.mass[b] = v;
  }
  __syncthreads();
}

__device__ __forceinline__ long long block_sum_ll(long long v, FullSmem& sm) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (lane == 0) sm.red_l[warp] = v;
  __syncthreads();
  long long t = 0;
  for (int w = 0; w < (int)(blockDim.x >> 5); w++) t += sm.red_l[w];
  __syncthreads();
  return t;
}
__device__ __forceinline__ double block_sum_d(double v, FullSmem& sm) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) sm.red_d[warp] = v;
  __syncthreads();
  double t = 0.0;
  for (int w = 0; w < (int)(blockDim.x >> 5); w++) t += sm.red_d[w];
  __syncthreads();
  return t;
}

// Index of the j-th (1-based) element, in id order, with glo <= x <= ghi.
// Warps own contiguous id ranges; the owner of the j-th scans its range.
__device__ int index_select(const RowInfo& R, float glo, float ghi, long long j, FullSmem& sm) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (int)(blockDim.x >> 5);
  const int seg = (((R.V + nwarps - 1) / nwarps) + 31) & ~31;
  const int s0 = min(R.V, warp * seg), s1 = min(R.V, s0 + seg);
  int cnt = 0;
  for (int i = s0 + lane; i < s1; i += 32) {
    const float x = load_x(R, i);
    cnt += (x >= glo && x <= ghi);
  }
  cnt = warp_sum_i(cnt);
  if (lane == 0) sm.red_i[warp] = cnt;
  if (threadIdx.x == 0) sm.result = -1;
  __syncthreads();
  long long before = 0;
  for (int w = 0; w < warp; w++) before += sm.red_i[w];
  if (before < j && before + cnt >= j) {
    long long need = j - before;
    for (int i0 = s0; i0 < s1; i0 += 32) {
      const int i = i0 + lane;
      const float x = i < s1 ? load_x(R, i) : -INFINITY;
      const bool f = i < s1 && x >= glo && x <= ghi;
      const unsigned m = __ballot_sync(0xffffffffu, f);
      if ((long long)__popc(m) >= need) {
        if (f && (long long)__popc(m & ((1u << lane) - 1u)) + 1 == need) sm.result = i;
        break;
      }
      need -= __popc(m);
    }
  }
  __syncthreads();
  const int res = sm.result < 0 ? 0 : sm.result;
  __syncthreads();
  return res;
}

struct FullSel {
  int id;          // vocabulary id of the selected element
  long long rank;  // 1-based position in (prob desc, id asc) order
  double cum;      // probability mass through it (fast above the final range)
};

// The element reaching `target`: the target-th by rank, or the first whose
// running probability mass is >= target.  Beyond the end: the last element.
__device__ FullSel select_full(const RowInfo& R, FullSmem& sm, bool by_mass, double target) {
  const int tid = threadIdx.x, warp = tid >> 5;
  // ---- level 0 (histogram kept from the row's first pass)
  if (warp == 0) {
    int b;
    long long pc;
    double pm;
    warp_pick(sm.h0, by_mass, target, &b, &pc, &pm);
    if ((tid & 31) == 0) {
      sm.sel_bin = b;
      sm.above_c = pc;
      sm.above_m = pm;
      sm.klo = sm.h0.kmin[b];
      sm.khi = sm.h0.kmax[b];
    }
  }
  __syncthreads();
  long long count = sm.h0.cnt[sm.sel_bin];
  // ---- level 1: the level-0 bucket split 1024 ways
  if (count > kExtCap) {
    const int b0 = sm.sel_bin;
    block_hist(R, sm.h1, [&](float x) { return bin0(R, x) == b0; }, [&](float x) { return bin1(R, x, b0); });
    if (warp == 0) {
      int b;
      long long pc;
      double pm;
      const double need = by_mass ? target - sm.above_m : target - (double)sm.above_c;
      warp_pick(sm.h1, by_mass, need, &b, &pc, &pm);
      if ((tid & 31) == 0) {
        sm.above_c += pc;
        sm.above_m += pm;
        sm.klo = sm.h1.kmin[b];
        sm.khi = sm.h1.kmax[b];
        sm.sel_bin = b;
      }
    }
    __syncthreads();
    count = sm.h1.cnt[sm.sel_bin];
  }
  // ---- key levels: the exact key range split 1024 ways until it fits
  while (count > kExtCap && sm.khi > sm.klo) {
    const uint32_t klo = sm.klo, khi = sm.khi;
    const uint64_t span = (uint64_t)khi - klo + 1;
    int shift = 0;
    while ((span >> shift) > (uint64_t)kBins) shift++;
    __syncthreads();
    block_hist(R, sm.h1, [&](float x) { const uint32_t k = fkey(x); return k >= klo && k <= khi; },
               [&](float x) { return (int)((khi - fkey(x)) >> shift); });
    if (warp == 0) {
      int b;
      long long pc;
      double pm;
      const double need = by_mass ? target - sm.above_m : target - (double)sm.above_c;
      warp_pick(sm.h1, by_mass, need, &b, &pc, &pm);
      if ((tid & 31) == 0) {
        sm.above_c += pc;
        sm.above_m += pm;
        sm.klo = sm.h1.kmin[b];
        sm.khi = sm.h1.kmax[b];
        sm.sel_bin = b;
      }
    }
    __syncthreads();
    count = sm.h1.cnt[sm.sel_bin];
  }

  // ---- the final range, widened to whole probability-tie groups at both ends:
  // G_b (top end, prob pb), G_a (bottom end, prob pa) and the elements between
  __shared__ float g_lohi[4];
  __shared__ float g_p[2];
  if (warp == 0) {
    const float xa = fkey_inv(sm.klo), xb = fkey_inv(sm.khi);
    const float bl = tie_low(R, xb), bh = tie_high(R, xb);
    const float al = tie_low(R, xa), ah = tie_high(R, xa);
    const float pb = prob_of(R, xb), pa = prob_of(R, xa);
    if ((tid & 31) == 0) {
      g_lohi[0] = bl; g_lohi[1] = bh; g_lohi[2] = al; g_lohi[3] = ah;
      g_p[0] = pb; g_p[1] = pa;
      sm.n_ext = 0;
    }
  }
  __syncthreads();
  const float gb_lo = g_lohi[0], gb_hi = g_lohi[1], ga_lo = g_lohi[2], ga_hi = g_lohi[3];
  const bool same = ga_lo == gb_lo;
  const float pb = g_p[0], pa = g_p[1];
  long long c_above = 0, c_gb = 0, c_ga = 0;
  double m_above = 0.0;
  for_row(R, [&](float x, int i) {
    if (x != x) return;
    if (x > gb_hi) {
      c_above++;
      m_above += mass_fast(R, x);
    } else if (x >= gb_lo) {
      c_gb++;
    } else if (!same && x > ga_hi) {
      const int pos = atomicAdd(&sm.n_ext, 1);
      if (pos < kExtCap) {
        const float p = prob_of(R, x);
        sm.key[pos] = ((unsigned long long)(0xFFFFFFFFu - __float_as_uint(p)) << 32) | (uint32_t)i;
      }
    } else if (!same && x >= ga_lo) {
      c_ga++;
    }
  });
  c_above = block_sum_ll(c_above, sm);
  c_gb = block_sum_ll(c_gb, sm);
  c_ga = block_sum_ll(c_ga, sm);
  m_above = block_sum_d(m_above, sm);
  const int n_mid = min(sm.n_ext, kExtCap);
  // ---- rank the middle exactly: bitonic sort of (prob desc, id asc) keys
  int np2 = 1;
  while (np2 < n_mid) np2 <<= 1;
  for (int j = n_mid + tid; j < np2; j += (int)blockDim.x) sm.key[j] = ~0ull;
  __syncthreads();
  for (int kk = 2; kk <= np2; kk <<= 1) {
    for (int jj = kk >> 1; jj > 0; jj >>= 1) {
      for (int i = tid; i < np2; i += (int)blockDim.x) {
        const int ixj = i ^ jj;
        if (ixj > i) {
          const unsigned long long x = sm.key[i], y = sm.key[ixj];
          if ((x > y) == ((i & kk) == 0)) { sm.key[i] = y; sm.key[ixj] = x; }
        }
      }
      __syncthreads();
    }
  }
  // ---- walk: above, G_b, middle, G_a
  FullSel out;
  out.id = -1;
  out.rank = 0;
  out.cum = 0.0;
  int grp = 0;        // 1: inside G_b, 3: inside G_a (index selection needed)
  long long gj = 0;   // position inside that group
  if (tid == 0) {
    long long rank = c_above;
    double cum = m_above;
    bool done = false;
    auto in_group = [&](long long cg, float p, int which) {
      if (done || cg <= 0) return;
      long long j = -1;
      if (by_mass) {
        if (p > 0.f && cum + (double)cg * (double)p >= target) {
          const double need = target - cum;
          j = need <= 0.0 ? 1 : (long long)ceil(need / (double)p);
        }
      } else if ((double)(rank + cg) >= target) {
        j = (long long)target - rank;
      }
      if (j >= 0) {
        j = j < 1 ? 1 : (j > cg ? cg : j);
        grp = which;
        gj = j;
        out.rank = rank + j;
        out.cum = cum + (double)j * (double)p;
        done = true;
      } else {
        rank += cg;
        cum += (double)cg * (double)p;
      }
    };
    in_group(c_gb, pb, 1);
    for (int i = 0; i < n_mid && !done; i++) {
      const unsigned long long k = sm.key[i];
      const double p = (double)__uint_as_float(0xFFFFFFFFu - (uint32_t)(k >> 32));
      rank++;
      cum += p;
      if (by_mass ? (cum >= target) : ((double)rank >= target)) {
        out.id = (int)(uint32_t)k;
        out.rank = rank;
        out.cum = cum;
        done = true;
      }
    }
    if (!same) in_group(c_ga, pa, 3);
    if (!done) {
      // beyond the end: the last element of the final range
      if (!same && c_ga > 0) { grp = 3; gj = c_ga; }
      else if (n_mid > 0) out.id = (int)(uint32_t)sm.key[n_mid - 1];
      else { grp = 1; gj = c_gb; }
      out.rank = rank;
      out.cum = cum;
    }
    sm.result = out.id;
    sm.rank_out = out.rank;
    sm.cum_out = out.cum;
    sm.sel_bin = grp;
    sm.above_c = gj;
  }
  __syncthreads();
  out.id = sm.result;
  out.rank = sm.rank_out;
  out.cum = sm.cum_out;
  grp = sm.sel_bin;
  gj = sm.above_c;
  __syncthreads();
  if (grp == 1) out.id = index_select(R, gb_lo, gb_hi, gj, sm);
  else if (grp == 3) out.id = index_select(R, ga_lo, ga_hi, gj, sm);
  return out;
}

// Diagnostics of a whole-row selection: the first c = min(n, cand_cap, kExtCap)
// candidates in (prob desc, id asc) order with their exact probabilities.  The
// element at rank c fixes the last key kc; every candidate has x >= the low end
// of kc's probability tie group, and exactly c elements have a key <= kc.
__device__ void full_emit_cands(const Args& A, int r, const RowInfo& R, FullSmem& sm, long long n) {
  const int c = (int)min((long long)min(A.cand_cap, kExtCap), n);
  if (c <= 0 || !(A.d_cand_ids || A.d_cand_probs)) return;
  const int tid = threadIdx.x, warp = tid >> 5;
  const FullSel s = select_full(R, sm, false, (double)c);
  __shared__ float e_xlo;
  __shared__ unsigned long long e_kc;
  if (warp == 0) {
    const float xc = load_x(R, s.id);
    const float xlo = tie_low(R, xc);
    if ((tid & 31) == 0) {
      e_xlo = xlo;
      e_kc = ((unsigned long long)(0xFFFFFFFFu - __float_as_uint(prob_of(R, xc))) << 32) | (uint32_t)s.id;
      sm.n_ext = 0;
    }
  }
  __syncthreads();
  const float xlo = e_xlo;
  const unsigned long long kc = e_kc;
  for_row(R, [&](float x, int i) {
    if (!(x >= xlo)) return;
    const unsigned long long k =
        ((unsigned long long)(0xFFFFFFFFu - __float_as_uint(prob_of(R, x))) << 32) | (uint32_t)i;
    if (k > kc) return;
    const int pos = atomicAdd(&sm.n_ext, 1);
    if (pos < kExtCap) sm.key[pos] = k;
  });
  __syncthreads();
  const int m = min(sm.n_ext, kExtCap);  // == c
  int np2 = 1;
  while (np2 < m) np2 <<= 1;
  for (int j = m + tid; j < np2; j += (int)blockDim.x) sm.key[j] = ~0ull;
  __syncthreads();
  for (int kk = 2; kk <= np2; kk <<= 1) {
    for (int jj = kk >> 1; jj > 0; jj >>= 1) {
      for (int i = tid; i < np2; i += (int)blockDim.x) {
        const int ixj = i ^ jj;
        if (ixj > i) {
          const unsigned long long x = sm.key[i], y = sm.key[ixj];
          if ((x > y) == ((i & kk) == 0)) { sm.key[i] = y; sm.key[ixj] = x; }
        }
      }
      __syncthreads();
    }
  }
  for (int i = tid; i < m; i += (int)blockDim.x) {
    const unsigned long long k = sm.key[i];
    if (A.d_cand_ids) A.d_cand_ids[(int64_t)r * A.cand_cap + i] = (int32_t)(uint32_t)k;
    if (A.d_cand_probs)
      A.d_cand_probs[(int64_t)r * A.cand_cap + i] = __uint_as_float(0xFFFFFFFFu - (uint32_t)(k >> 32));
  }
  __syncthreads();
}

// Top-k / top-p / draw for one row over the whole vocabulary (src/generation.js:27-49).
__device__ __forceinline__ void full_path(const Args& A, int r, const RowInfo& R, FullSmem& sm, int flags) {
  const int tid = threadIdx.x;
  const int V = R.V;
  block_hist(R, sm.h0, [](float) { return true; }, [&](float x) { return bin0(R, x); });
  double tm = 0.0;
  for (int b = tid; b < kBins; b += (int)blockDim.x) tm += sm.h0.mass[b];
  const double total_all = block_sum_d(tm, sm);
  const bool use_k = A.k > 0 && A.k < V;
  long long n;
  double mass_n;
  int last_id = -1;  // id at rank n (the draw loop's fallback)
  if (use_k) {
    const FullSel gk = select_full(R, sm, false, (double)A.k);
    n = A.k;
    mass_n = gk.cum;
    last_id = gk.id;
  } else {
    n = V;
    mass_n = total_all;
  }
  double total = mass_n;
  if (A.use_topp && mass_n >= A.top_p) {
    const FullSel gp = select_full(R, sm, true, A.top_p);
    if (gp.rank < n) {
      n = gp.rank < 1 ? 1 : gp.rank;
      total = gp.cum;
      last_id = gp.id;
    }
  }
  const double u = A.u ? A.u[r] : 0.0;
  const double rr = u * total;
  int id;
  if (rr <= 0.0) {
    id = select_full(R, sm, false, 1.0).id;
  } else {
    const FullSel gd = select_full(R, sm, true, rr);
    if (gd.rank > n) {
      if (last_id < 0) last_id = select_full(R, sm, false, (double)n).id;
      id = last_id;
    } else {
      id = gd.id;
    }
  }
  if (tid == 0) {
    A.out_ids[r] = id;
    if (A.d_n_cand) A.d_n_cand[r] = (int32_t)n;
    if (A.d_total) A.d_total[r] = total;
    if (A.d_row_flags) A.d_row_flags[r] = flags | MS_ROW_FULLVOCAB;
  }
  full_emit_cands(A, r, R, sm, n);
}
}  // namespace ms
