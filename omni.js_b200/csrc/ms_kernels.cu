// Sampler kernel for B200 (sm_100a).
//
// One sampling step over a [B, V] fp32 logits block is ONE launch of
// sample_kernel, grid (B, ceil(V/16384)), 256 threads for sampled rows (512 for
// greedy ones), 64 KiB of shared memory per CTA (3 CTAs per SM).  Each CTA owns
// one 16384-logit chunk of one row:
//
//   1. thread 0 starts four 16 KiB TMA bulk copies of the chunk into shared
//      memory; meanwhile all threads read the row's id history in 16-byte
//      blocks and set the bits of the chunk's penalised ids in a bitmap (so
//      repeated ids count once, the reference's Set, src/generation.js:20);
//   2. the penalty is applied in shared memory to the flagged logits
//      (src/generation.js:19-25), each by the thread that reads it in the
//      streaming passes (the bitmap is laid out per thread), so no barrier
//      separates it from them;
//   3. pass A: chunk max and a threshold tau that at least top_k elements of
//      the chunk reach (from the sorted per-thread maxima of every warp);
//   4. pass B: fast fp32 sum of 2^((x - m) * log2(e)/T) and the list of
//      elements >= tau (>= sig, a storage threshold, in a partial chunk);
//   5. the chunk results go to global scratch; the row is finalized either by
//      the last CTA of the row to finish (atomic row counter) or by a second
//      grid of one CTA per row, launched as a programmatic dependent of the
//      first (greedy rows always use the first form): softmax denominator
//      (fast sum corrected with the exact terms of the top candidates), the
//      exact fp32 probabilities of the candidates, their order
//      (prob desc, id asc), top-k, top-p and the draw (src/generation.js:9-17,
//      27-49).
// Logits are read from HBM exactly once; everything after the load works on
// shared memory or on the small candidate lists.
//
// Rows whose candidate set cannot be proven complete, and every row when top_k
// is off (top_k <= 0 or >= V) or larger than 256, go through full_path: an
// exact rescan of the row by radix selection over order-preserving float keys.
#include <cfloat>
#include <climits>
#include <cstdio>
#include <algorithm>

#include "ms_device.cuh"
#include "ms_fullpath.cuh"

namespace ms {

constexpr long long kWaitCycles = 4000000000LL;  // ~2 s: bound on every wait
constexpr unsigned kAll = 0xffffffffu;
constexpr int kFinChunks = 256;  // chunks whose scale the finalizer caches
constexpr int kFuseRows = 16;    // top-k calls of at most this many rows finalize in the chunk kernel

// =============================================================== shared scratch
// =============================================================== finalize
struct FinSmem {
  Cand gath[kGathMax];              // candidates >= tau_row; later their sort keys
  unsigned long long keys[kFinMax];  // the boundary bucket of the selection
  unsigned long long top[kKmax];     // the selected top_k keys
  int h1[256], h2[256];              // selection histograms
  int b1, b2, need, n_keep, n_bkt, n_top;
  int off[33];                       // merge: list offsets of the shards
  uint32_t kx;                       // kth_largest_x: the selected key
  int nf, nF, slow, nan_row, bad, overflow;
  unsigned long long corr;  // fixed-point (2^-50) sum of the candidate corrections
  double S, S_fast, scale0, u;
  float M, Mp, tau_row, pout;
  float cm[kFinChunks];      // chunk maxima (first kFinChunks chunks)
  float cz[kFinChunks];      // their fast-term offsets
  double cs[kFinChunks];     // chunk_scale of each
};

__device__ __forceinline__ double chunk_scale(const Args& A, float mc, float zc, float Mp) {
  // exp(m_c / T - M') converts fast terms relative to the chunk max to the
  // reference's units.  2^(x*a - zref) = 2^((x - m_c)*a) * 2^(m_c*a - zref), so
  // 2^(zref - m_c*a) (the exponent is exact in fp64) undoes zref's rounding.
  if (mc == -INFINITY) return 0.0;
  double sc = exp((double)mc * A.rT - (double)Mp);
  if (zc == zc) sc *= exp2((double)zc - (double)mc * (double)A.a);
  return sc;
}

// a chunk's fast term of x, recomputed bit for bit
__device__ __forceinline__ float chunk_term(const Args& A, float x, float mc, float zc) {
  return (zc == zc) ? term_fast_z(x, A.a, zc) : term_fast(x, mc, A.a);
}

__device__ __forceinline__ double key_prob(unsigned long long key) {
  return (double)__uint_as_float(0xFFFFFFFFu - (uint32_t)(key >> 32));
}

// Bucket of a 256-bin histogram (ascending) where the running count reaches
// target (1 <= target <= total), and how many of that bucket's entries it
// takes.  Called by one full warp.
__device__ void scan_pick(const int* h, int target, int* bin_out, int* need_out) {
  const int lane = threadIdx.x & 31;
  int c[8], s = 0;
#pragma unroll
  for (int i = 0; i < 8; i++) { c[i] = h[8 * lane + i]; s += c[i]; }
  int incl = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(kAll, incl, o);
    if (lane >= o) incl += t;
  }
  const int excl = incl - s;
  if (excl < target && incl >= target) {
    int run = excl;
#pragma unroll
    for (int i = 0; i < 8; i++) {
      if (run + c[i] >= target) { *bin_out = 8 * lane + i; *need_out = target - run; break; }
      run += c[i];
    }
  }
}

// An fp32 probability p >= 2^-30 in units of 2^-53 (exact: its last bit is
// worth at least 2^-53).
__device__ __forceinline__ long long p_units(uint32_t pb) {
  const int e = (int)(pb >> 23) - 127;
  return (long long)((pb & 0x7FFFFFu) | 0x800000u) << (e + 30);
}

// Top-k, top-p and the draw over the first A.k sorted candidates
// (src/generation.js:32-48), called by one full warp.  The reference sums in
// fp64 sequentially.  When every probability is >= 2^-30 and the k
// probabilities sum below 1, every partial sum is a multiple of 2^-53 below 1
// and so exact in fp64: the sums are then done in integers (units of 2^-53),
// in parallel, with the same results bit for bit.  The comparisons acc >= P
// become units >= ceil(P * 2^53) (the scaling is exact).  Otherwise lane 0
// runs the sequential loops.
__device__ void topk_draw(const Args& A, int r, const unsigned long long* sorted, float Mp, double S, double u,
                          int* n_out) {
  const int lane = threadIdx.x & 31;
  const int k = A.k;
  const int per = (k + 31) / 32;
  const int i0 = min(k, lane * per), i1 = min(k, i0 + per);
  long long ls = 0;
  bool ok = true;
  for (int i = i0; i < i1; i++) {
    const uint32_t pb = 0xFFFFFFFFu - (uint32_t)(sorted[i] >> 32);
    ok &= pb >= 0x30800000u && pb < 0x3F800000u;  // 2^-30 <= p < 1
    if (ok) ls += p_units(pb);
  }
  long long incl = ls;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const long long t = __shfl_up_sync(kAll, incl, o);
    if (lane >= o) incl += t;
  }
  const long long total_k = __shfl_sync(kAll, incl, 31);
  const bool exact = __all_sync(kAll, ok) && total_k < (1ll << 53);
  int n = k, id = 0;
  double total = 0.0;
  if (exact) {
    auto units = [&](int i) { return p_units(0xFFFFFFFFu - (uint32_t)(sorted[i] >> 32)); };
    // first i < limit with prefix_i >= target, or UINT_MAX
    auto first_reach = [&](long long target, int limit) {
      long long acc = incl - ls;
      unsigned hit = UINT_MAX;
      for (int i = i0; i < min(i1, limit); i++) {
        acc += units(i);
        if (acc >= target) { hit = (unsigned)i; break; }
      }
      return __reduce_min_sync(kAll, hit);
    };
    if (A.use_topp) {  // top_p < 1 here; below -1 it behaves as -1 (the first acc reaches it)
      const unsigned h = first_reach((long long)ceil(fmax(A.top_p, -1.0) * 9007199254740992.0), k);
      n = (h == UINT_MAX) ? k : (int)h + 1;
    }
    // total = prefix_{n-1}, held by the lane owning n-1
    long long acc = incl - ls, tot = 0;
    for (int i = i0; i < i1; i++) {
      acc += units(i);
      if (i == n - 1) tot = acc;
    }
    total = (double)__shfl_sync(kAll, tot, (n - 1) / per) * (1.0 / 9007199254740992.0);
    const double rr = u * total;
    // rr beyond every prefix (NaN, or u >= 1) draws the last candidate, as the
    // reference's subtraction loop falls through
    const long long rt = (rr <= 2.0) ? (long long)ceil(fmax(rr, -1.0) * 9007199254740992.0) : LLONG_MAX;
    const unsigned h = first_reach(rt, n);
    id = (int)(uint32_t)sorted[h == UINT_MAX ? n - 1 : h];
  } else if (lane == 0) {
    if (A.use_topp) {
      double a2 = 0.0;
      int cut = n;
      for (int i = 0; i < n; i++) {
        a2 += key_prob(sorted[i]);
        if (a2 >= A.top_p) { cut = i + 1; break; }
      }
      n = cut > 1 ? cut : 1;
    }
    for (int i = 0; i < n; i++) total += key_prob(sorted[i]);
    double rr = u * total;
    id = (int)(uint32_t)sorted[n - 1];
    for (int i = 0; i < n; i++) {
      rr -= key_prob(sorted[i]);
      if (rr <= 0.0) { id = (int)(uint32_t)sorted[i]; break; }
    }
  }
  if (lane == 0) {
    A.out_ids[r] = id;
    if (A.d_n_cand) A.d_n_cand[r] = n;
    if (A.d_total) A.d_total[r] = total;
    if (A.d_row_max) A.d_row_max[r] = (double)Mp;
    if (A.d_row_sum) A.d_row_sum[r] = S;
    if (A.d_row_flags) A.d_row_flags[r] = 0;
    *n_out = n;
  }
}

// Top-k by (prob desc, id asc) over the nfc gathered candidates, whose x
// already holds the exact softmax term, then top-p and the draw; the id goes
// to A.out_ids[r].  Before the call F.pout holds the largest probability any
// element outside the candidates can have (-1: there is none), and F.h1, F.h2,
// F.n_top, F.n_bkt are zero; F.pout is read after the first barrier here.
// Returns false, with nothing written, when the candidates cannot settle the
// row (a probability outside them could tie with the k-th).
__device__ bool topk_from_terms(const Args& A, int r, FinSmem& F, int nfc, double S, double rS, float Mp) {
  const int tid = threadIdx.x, warp = tid >> 5;
  const int nt = (int)blockDim.x;
  const int k = A.k;
  // ---- sort keys (prob desc, id asc) of the candidates, in place, and the
  // histogram of their top byte
  unsigned long long* key = reinterpret_cast<unsigned long long*>(F.gath);
  for (int j = tid; j < nfc; j += nt) {
    const Cand cd = F.gath[j];
    const float p = div_to_f32((double)cd.x, S, rS);
    const unsigned long long kk = ((unsigned long long)(0xFFFFFFFFu - __float_as_uint(p)) << 32) | (uint32_t)cd.i;
    key[j] = kk;
    atomicAdd(&F.h1[(int)(kk >> 56)], 1);
  }
  __syncthreads();
  // ---- the k smallest keys: the k-th falls in bucket (b1, b2) of the keys'
  // top 16 bits; what lies below it is in, and its own keys are ranked
  if (warp == 0) scan_pick(F.h1, k, &F.b1, &F.need);
  __syncthreads();
  const uint32_t b1 = (uint32_t)F.b1;
  for (int j = tid; j < nfc; j += nt) {
    const unsigned long long kk = key[j];
    if ((uint32_t)(kk >> 56) == b1) atomicAdd(&F.h2[(int)(kk >> 48) & 255], 1);
  }
  __syncthreads();
  if (warp == 0) scan_pick(F.h2, F.need, &F.b2, &F.need);
  __syncthreads();
  const uint32_t p16 = (b1 << 8) | (uint32_t)F.b2;
  const int need = F.need;  // keys of the bucket still to take (>= 1)
  for (int j = tid; j < nfc; j += nt) {
    const unsigned long long kk = key[j];
    const uint32_t hi = (uint32_t)(kk >> 48);
    if (hi < p16) {
      const int q = atomicAdd(&F.n_top, 1);
      if (q < kKmax) F.top[q] = kk;
    } else if (hi == p16) {
      const int q = atomicAdd(&F.n_bkt, 1);
      if (q < kFinMax) F.keys[q] = kk;
    }
  }
  __syncthreads();
  const int nb = F.n_bkt;
  if (nb <= kFinMax) {
    for (int t = tid; t < nb; t += nt) {  // keys are distinct: the ids differ
      const unsigned long long kk = F.keys[t];
      int rank = 0;
      for (int j = 0; j < nb; j++) rank += F.keys[j] < kk;
      if (rank < need) {
        const int q = atomicAdd(&F.n_top, 1);
        if (q < kKmax) F.top[q] = kk;
      }
    }
  }
  __syncthreads();
  if (nb <= kFinMax && F.n_top == k) {
    // ---- the k keys in order (rank sort, into the bucket's space)
    unsigned long long* sorted = F.keys;
    for (int t = tid; t < k; t += nt) {
      const unsigned long long kk = F.top[t];
      int rank = 0;
      for (int j = 0; j < k; j++) rank += F.top[j] < kk;
      sorted[rank] = kk;
    }
    __syncthreads();
    // the k-th probability must beat every probability outside the
    // candidates (else ties reach past them: rescan)
    if (F.pout < (float)key_prob(sorted[k - 1])) {
      if (warp == 0) topk_draw(A, r, sorted, Mp, S, F.u, &F.nF);
      __syncthreads();
      if (A.d_cand_ids || A.d_cand_probs) {
        const int n = F.nF;  // set by topk_draw
        for (int i = tid; i < n && i < A.cand_cap; i += nt) {
          const unsigned long long kkey = sorted[i];
          if (A.d_cand_ids) A.d_cand_ids[(int64_t)r * A.cand_cap + i] = (int32_t)(uint32_t)kkey;
          if (A.d_cand_probs)
            A.d_cand_probs[(int64_t)r * A.cand_cap + i] = __uint_as_float(0xFFFFFFFFu - (uint32_t)(kkey >> 32));
        }
      }
      return true;
    }
  }
  __syncthreads();
  return false;
}

// Row statistics from the chunk stats (warp 0): max, tempered max, tau_row,
// NaN and overflow flags, fast sum in units of exp(x' - Mp), chunk scales;
// warp 1 prefetches u and clears the selection state.  Ends with a barrier.
__device__ void row_stats(const Args& A, int r, FinSmem& F) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const ChunkStat* st = A.stats + (int64_t)r * A.n_chunks;
  if (warp == 0) {
    // a chunk's stats in two 16-byte loads (the array is 32-byte aligned); the
    // lane's first chunk is kept for the second loop
    auto load_stat = [&](int c) {
      ChunkStat v;
      const int4* p = reinterpret_cast<const int4*>(st + c);
      int4* q = reinterpret_cast<int4*>(&v);
      q[0] = __ldcg(p);
      q[1] = __ldcg(p + 1);
      return v;
    };
    ChunkStat first;
    float M = -INFINITY, tr = -INFINITY, sg = -INFINITY;
    int nanr = 0, ovf = 0;
    for (int c = lane; c < A.n_chunks; c += 32) {
      const ChunkStat v = load_stat(c);
      if (c == lane) first = v;
      M = fmaxf(M, v.m);
      tr = fmaxf(tr, v.tau);
      sg = fmaxf(sg, v.sig);
      nanr |= (v.s != v.s);
      ovf |= (v.n_cand > kCap);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      M = fmaxf(M, __shfl_xor_sync(kAll, M, o));
      tr = fmaxf(tr, __shfl_xor_sync(kAll, tr, o));
      sg = fmaxf(sg, __shfl_xor_sync(kAll, sg, o));
      nanr |= __shfl_xor_sync(kAll, nanr, o);
      ovf |= __shfl_xor_sync(kAll, ovf, o);
    }
    const float Mp = temper_fast(M, A.T, A.rT, A.temper);
    // a NaN, or a tempered max that is not finite, makes the softmax NaN; so
    // does a row of -inf (the reference's exp(-inf - -inf))
    const int bad = nanr | (Mp != Mp) | (isinf(Mp) && M != -INFINITY);
    nanr = bad | (M == -INFINITY);
    double S = 0.0;
    if (!nanr) {
      for (int c = lane; c < A.n_chunks; c += 32) {
        const ChunkStat v = (c == lane) ? first : load_stat(c);
        const double sc = chunk_scale(A, v.m, v.zref, Mp);
        if (v.m != -INFINITY) S += v.s * sc;
        if (c < kFinChunks) { F.cm[c] = v.m; F.cz[c] = v.zref; F.cs[c] = sc; }
      }
      S = warp_sum(S);
    }
    if (lane == 0) {
      F.M = M; F.Mp = Mp; F.tau_row = tr; F.nan_row = nanr; F.bad = bad; F.overflow = ovf;
      // a chunk that kept only elements >= sig > tau_row may miss candidates
      F.nf = 0; F.slow = ovf | (sg > tr); F.corr = 0ull; F.S_fast = S;
      F.scale0 = nanr ? 0.0 : exp((double)M * A.rT - (double)Mp);
    }
  } else if (warp == 1) {
    if (lane == 0) F.u = A.u ? __ldg(A.u + r) : 0.0;
    for (int b = lane; b < 256; b += 32) { F.h1[b] = 0; F.h2[b] = 0; }
    if (lane == 0) { F.n_top = 0; F.n_bkt = 0; F.n_keep = 0; F.kx = 0u; }
  } else {  // the other warps clear narrow_terms' histograms
    int* wh = reinterpret_cast<int*>(F.keys);
    for (int b = tid - 64; b < 8 * 256; b += (int)blockDim.x - 64) wh[b] = 0;
  }
  __syncthreads();
}

// Candidates >= tau_row of every chunk into F.gath (F.nf counts them, possibly
// beyond kGathMax).  Ends with a barrier.
__device__ void gather_cands(const Args& A, int r, FinSmem& F) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nw = (int)(blockDim.x >> 5);
  const ChunkStat* st = A.stats + (int64_t)r * A.n_chunks;
  const float tau_row = F.tau_row;
  // two chunks per warp at a time (c and c + nw): both list lengths, then
  // eight entries per lane, are in flight together
  for (int c = warp; c < A.n_chunks; c += 2 * nw) {
    const int c2 = c + nw;
    const bool two = c2 < A.n_chunks;
    const int nc0 = min(__ldcg(&st[c].n_cand), kCap);
    const int nc1 = two ? min(__ldcg(&st[c2].n_cand), kCap) : 0;
    const Cand* src0 = A.cands + ((int64_t)r * A.n_chunks + c) * kCap;
    const Cand* src1 = A.cands + ((int64_t)r * A.n_chunks + (two ? c2 : c)) * kCap;
    for (int j0 = 0; j0 < max(nc0, nc1); j0 += 128) {
      float2 v[8];
#pragma unroll
      for (int t = 0; t < 8; t++) {
        const int j = j0 + 32 * (t & 3) + lane;
        const int nc = t < 4 ? nc0 : nc1;
        const Cand* src = t < 4 ? src0 : src1;
        v[t] = j < nc ? __ldcg(reinterpret_cast<const float2*>(src + j)) : make_float2(-INFINITY, 0.f);
      }
#pragma unroll
      for (int t = 0; t < 8; t++) {
        const int j = j0 + 32 * (t & 3) + lane;
        const bool keep = j < (t < 4 ? nc0 : nc1) && v[t].x >= tau_row;
        const unsigned msk = __ballot_sync(kAll, keep);
        if (msk) {
          int base = 0;
          if (lane == 0) base = atomicAdd(&F.nf, __popc(msk));
          base = __shfl_sync(kAll, base, 0);
          const int pos = base + __popc(msk & ((1u << lane) - 1u));
          if (keep && pos < kGathMax) F.gath[pos] = Cand{v[t].x, __float_as_int(v[t].y)};
        }
      }
    }
  }
  __syncthreads();
}

// The exact softmax term of a gathered candidate (src/generation.js:14) and
// its correction of the fast sum (exact minus fast term, in 2^-50 units).
__device__ __forceinline__ float cand_term(const Args& A, const FinSmem& F, const ChunkStat* st, const Cand& cd,
                                           float Mp, long long* corr) {
  const int c = cd.i / kChunk;
  const float mc = c < kFinChunks ? F.cm[c] : __ldcg(&st[c].m);
  const float zc = c < kFinChunks ? F.cz[c] : __ldcg(&st[c].zref);
  const double sc = c < kFinChunks ? F.cs[c] : chunk_scale(A, mc, zc, Mp);
  const float e = term_exact(temper_fast(cd.x, A.T, A.rT, A.temper), Mp);
  *corr += __double2ll_rn(((double)e - (double)chunk_term(A, cd.x, mc, zc) * sc) * 1125899906842624.0);
  return e;
}

// Top-k rows: narrows the nfc gathered candidates (all x >= tau_row, M the row
// max) to those that can still be among the top k.  A 256-bin histogram of x
// over [tau_row, M] (per-warp copies in F.keys, cleared by row_stats, so few
// lanes meet on one counter) finds the bin of the k-th largest x; the
// candidates of that bin and the bins above it go to F.top as Cand, then get
// their exact terms in x (one per thread) and their corrections in F.corr.
// Returns their number (>= k), with *xout the largest x left out (-inf:
// none), or -1 when nothing is narrowed (F.corr, F.h1 and F.h2 are then as
// row_stats left them).  Ends with a barrier.
__device__ int narrow_terms(const Args& A, FinSmem& F, const ChunkStat* st, int nfc, float tau_row, float M,
                            float Mp, float* xout) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nt = (int)blockDim.x;
  const int k = A.k;
  *xout = -INFINITY;
  const float span = M - tau_row;
  // nothing to gain, or no finite range to bin over (uniform across the CTA)
  if (nfc <= 2 * k || !(span > 0.f) || !(span <= FLT_MAX)) return -1;
  const float inv_w = 256.f / span;
  auto bin = [&](float x) { return min(255, max(0, __float2int_rd(__fmul_rn(__fsub_rn(x, tau_row), inv_w)))); };
  int* wh = reinterpret_cast<int*>(F.keys);  // 8 histograms of 256 bins
  int* myh = wh + (warp & 7) * 256;
  for (int j = tid; j < nfc; j += nt) atomicAdd(&myh[bin(F.gath[j].x)], 1);
  __syncthreads();
  if (warp == 0) {  // bins in descending x: F.h1[255 - b] counts bin b
    for (int b = lane; b < 256; b += 32) {
      int t = 0;
#pragma unroll
      for (int w = 0; w < 8; w++) t += wh[w * 256 + b];
      F.h1[255 - b] = t;
    }
    __syncwarp();
    scan_pick(F.h1, k, &F.b1, &F.need);
  }
  __syncthreads();
  const int bk = 255 - F.b1;  // the bin of the k-th largest x: keep bins >= bk
  Cand* keep = reinterpret_cast<Cand*>(F.top);  // room for kKmax candidates
  for (int j = tid; j < nfc; j += nt) {
    const Cand cd = F.gath[j];
    if (bin(cd.x) >= bk) {
      const int q = atomicAdd(&F.n_keep, 1);
      if (q < kKmax) keep[q] = cd;
    } else {
      atomicMax(&F.kx, fkey(cd.x));
    }
  }
  __syncthreads();
  const int nk = F.n_keep;
  if (nk > kKmax) {  // too many in the bin: leave F.h1 as it was
    for (int b = tid; b < 256; b += nt) F.h1[b] = 0;
    __syncthreads();
    return -1;
  }
  // the exact terms, one candidate per thread
  long long corr = 0;
  for (int j = tid; j < nk; j += nt) keep[j].x = cand_term(A, F, st, keep[j], Mp, &corr);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) corr += __shfl_xor_sync(kAll, corr, o);
  if (lane == 0 && corr != 0) atomicAdd(&F.corr, (unsigned long long)corr);
  __syncthreads();
  *xout = F.kx ? fkey_inv(F.kx) : -INFINITY;
  return nk;
}

// topk_from_terms for the n (k <= n <= kKmax) narrowed candidates in F.top:
// every key is ranked against all others in one pass.  Same contract
// otherwise (F.pout read after the first barrier; false: cannot settle).
__device__ bool topk_small(const Args& A, int r, FinSmem& F, int n, double S, double rS, float Mp) {
  const int tid = threadIdx.x, warp = tid >> 5, nt = (int)blockDim.x;
  const int k = A.k;
  const Cand* cands = reinterpret_cast<const Cand*>(F.top);
  unsigned long long* key = F.keys;
  for (int j = tid; j < n; j += nt) {
    const Cand cd = cands[j];
    const float p = div_to_f32((double)cd.x, S, rS);
    key[j] = ((unsigned long long)(0xFFFFFFFFu - __float_as_uint(p)) << 32) | (uint32_t)cd.i;
  }
  __syncthreads();
  unsigned long long* sorted = F.top;  // the candidates are no longer read
  for (int t = tid; t < n; t += nt) {  // keys are distinct: the ids differ
    const unsigned long long kk = key[t];
    int rank = 0;
    for (int j = 0; j < n; j++) rank += key[j] < kk;
    if (rank < k) sorted[rank] = kk;
  }
  __syncthreads();
  if (!(F.pout < (float)key_prob(sorted[k - 1]))) return false;
  if (warp == 0) topk_draw(A, r, sorted, Mp, S, F.u, &F.nF);
  __syncthreads();
  if (A.d_cand_ids || A.d_cand_probs) {
    const int nn = F.nF;  // set by topk_draw
    for (int i = tid; i < nn && i < A.cand_cap; i += nt) {
      const unsigned long long kkey = sorted[i];
      if (A.d_cand_ids) A.d_cand_ids[(int64_t)r * A.cand_cap + i] = (int32_t)(uint32_t)kkey;
      if (A.d_cand_probs)
        A.d_cand_probs[(int64_t)r * A.cand_cap + i] = __uint_as_float(0xFFFFFFFFu - (uint32_t)(kkey >> 32));
    }
  }
  return true;
}

template <int MODE>
__device__ __forceinline__ void finalize_row(const Args& A, int r, FinSmem& F) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nt = (int)blockDim.x;  // 256 or 512 threads
  const ChunkStat* st = A.stats + (int64_t)r * A.n_chunks;
  const int V = A.V;

  if (MODE == kGreedy) {
    if (warp == 0) {
      float bv = -INFINITY;
      int bi = INT_MAX;
      for (int c = lane; c < A.n_chunks; c += 32) {
        const float v = __ldcg(&st[c].m);
        const int i = __ldcg(&st[c].best_i);
        if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(kAll, bv, o);
        const int oi = __shfl_xor_sync(kAll, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      if (lane == 0) {
        // src/generation.js:51-55: a NaN at index 0 is never beaten
        const float x0 = A.logits[(int64_t)r * A.ld];
        const int id = (x0 != x0 || bv == -INFINITY || bi == INT_MAX) ? 0 : bi;
        A.out_ids[r] = id;
        if (A.d_row_flags) A.d_row_flags[r] = MS_ROW_GREEDY;
        if (A.d_n_cand) A.d_n_cand[r] = 0;
        if (A.d_row_max) A.d_row_max[r] = (double)bv;
      }
    }
    return;
  }

  // ---- row max, NaN detection, overflow, tau_row, fast sum
  row_stats(A, r, F);
  if (F.nan_row) {
    // softmax is NaN everywhere: the stable sort keeps id order, no acc reaches
    // topP, r is NaN, and the draw loop falls through to the last candidate.
    if (tid == 0) {
      const bool use_k = A.k > 0 && A.k < V;
      A.out_ids[r] = use_k ? A.k - 1 : V - 1;
      if (A.d_n_cand) A.d_n_cand[r] = use_k ? A.k : V;
      if (A.d_row_max) A.d_row_max[r] = (double)F.Mp;
      if (A.d_row_sum) A.d_row_sum[r] = __longlong_as_double(0x7ff8000000000000ll);
      if (A.d_total) A.d_total[r] = __longlong_as_double(0x7ff8000000000000ll);
      if (A.d_row_flags) A.d_row_flags[r] = MS_ROW_NAN;
    }
    return;
  }
  const float M = F.M, Mp = F.Mp, tau_row = F.tau_row;

  // ---- gather the candidates >= tau_row (all of them unless a chunk overflowed)
  gather_cands(A, r, F);
  const int nf = F.nf;
  int nfc = min(nf, kGathMax);
  if (nf > kGathMax || (MODE == kTopK && nf < A.k)) {
    if (tid == 0) F.slow = 1;
  }
  // ---- top-k rows: only the candidates that can reach the top k go on, with
  // their exact terms (the largest x left out bounds every probability
  // outside them)
  float xout = -INFINITY;
  int nk = -1;
  if (MODE == kTopK && !F.slow && nf <= kGathMax && nf >= A.k) nk = narrow_terms(A, F, st, nfc, tau_row, M, Mp, &xout);

  // ---- otherwise the exact terms of every gathered candidate (kept in place
  // of x) and the fast sum's correction: exact minus fast term, summed in
  // 2^-50 units
  if (nk < 0) {
    long long corr = 0;
    for (int j = tid; j < nfc; j += nt) {
      Cand cd = F.gath[j];
      cd.x = cand_term(A, F, st, cd, Mp, &corr);
      F.gath[j] = cd;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) corr += __shfl_xor_sync(kAll, corr, o);
    if (lane == 0 && corr != 0) atomicAdd(&F.corr, (unsigned long long)corr);
    __syncthreads();
  }
  const double S = F.S_fast + (double)(long long)F.corr * (1.0 / 1125899906842624.0);

  RowInfo R;
  R.row = A.logits + (int64_t)r * A.ld;
  R.V = V;
  R.pb = nullptr;
  R.pen = A.pen;
  R.M = M;
  R.Mp = Mp;
  R.S = S;
  R.a = A.a;
  R.mscale = F.scale0 / S;
  R.T = A.T;
  R.temper = A.temper;
  R.rpen = A.rpen;
  R.nat16 = (float)(16.0 / A.T);
  R.rT = A.rT;
  R.rS = 1.0 / R.S;

  if (MODE == kTopK && !F.slow) {
    // every element outside the candidates has x <= xout (a narrowed-out
    // candidate) or x < tau_row, so its probability is at most that of xout or
    // of the fp32 value below tau_row
    const double rS = 1.0 / S;
    if (tid == 0) {
      float po = -1.f;
      if (xout != -INFINITY || tau_row != -INFINITY) {
        const float xo = (xout != -INFINITY) ? xout : fkey_inv(fkey(tau_row) - 1u);
        po = div_to_f32((double)term_exact(temper_fast(xo, A.T, A.rT, A.temper), Mp), S, rS);
      }
      F.pout = po;
    }
    if (nk >= 0 ? topk_small(A, r, F, nk, S, rS, Mp) : topk_from_terms(A, r, F, nfc, S, rS, Mp)) return;
  }
  // ---- exact rescan of the whole row
  const int flags = (MODE == kTopK) ? MS_ROW_SLOWPATH : 0;
  if (A.use_pen && A.penbits) {
    const int W = (V + 31) >> 5;
    uint32_t* pb = A.penbits + (int64_t)r * W;
    for (int w = tid; w < W; w += nt) pb[w] = 0u;
    __syncthreads();
    const int64_t h0 = A.hist_off[r], h1 = A.hist_off[r + 1];
    for (int64_t h = h0 + tid; h < h1; h += nt) {
      const int id = A.hist[h];
      if (id >= 0 && id < V) atomicOr(&pb[id >> 5], 1u << (id & 31));
    }
    __threadfence_block();
    __syncthreads();
    R.pb = pb;
  }
  if (tid == 0) {
    if (A.d_row_max) A.d_row_max[r] = (double)Mp;
    if (A.d_row_sum) A.d_row_sum[r] = S;
  }
  __syncthreads();  // the finalize scratch is reused by the full-row path
  full_path(A, r, R, *reinterpret_cast<FullSmem*>(&F), flags);
}

// Absolute mass-histogram bin of a logit: floor(-x * a16) with a16 = 16 * a
// (1/16 of a log2 unit of the tempered logit per bin), saturating; the same
// arithmetic wherever a bin is computed, so every pass agrees on it.
__device__ __forceinline__ int nuc_bin(float x, float a16) { return __float2int_rd(__fmul_rn(-x, a16)); }
// Per-bin fixed-point scale of the chunk histogram's masses (see sample_kernel).
__device__ __forceinline__ float nuc_scale(int b) { return ex2_approx(21.f + (float)b * 0.0625f); }
__device__ __forceinline__ int nuc_local(int bin, int top) {
  const long long d = (long long)bin - (long long)top;
  return (int)(d < 0 ? 0 : (d > kNB - 1 ? kNB - 1 : d));
}

// =============================================================== the kernel
// The row's history ids (positions [h0, h1) of A.hist) that fall in chunk
// [c0, c0 + n) set their bits in the chunk's penalty bitmap, so a repeated id
// counts once (the reference's Set, src/generation.js:20).  The ids are read in
// aligned 16-byte blocks: the first and the last block of the row may reach
// past the row's ids (never past the 16-byte block holding one of them, so
// never outside the buffer's pages) and those ids are masked off.
//
// Bit layouts: chunk position d is bit d of the bitmap (row-major), or, with
// OWNER, the bit of the thread that reads d in the chunk kernel's streaming
// loops: d lies in float4 q = d / 4, read by thread q % NT at step q / NT, and
// its bit is 4 * (q / NT) + d % 4 of that thread's kChunk / NT bits (words
// thread * kChunk / (32 * NT) onwards).
template <int NT, bool OWNER>
__device__ __forceinline__ void pen_scan(const Args& A, int64_t h0, int64_t h1, int c0, int n, uint32_t* penmask) {
  constexpr int kWordsPerThread = kChunk / 32 / NT;
  const int hn = (int)(h1 - h0);
  if (hn <= 0) return;
  const int32_t* hrow = A.hist + h0;
  const int lead = (int)((reinterpret_cast<uintptr_t>(hrow) >> 2) & 3);  // ids of block 0 before the row
  const int4* blk = reinterpret_cast<const int4*>(hrow - lead);
  const int nb = (lead + hn + 3) >> 2;
  const uint32_t base = (uint32_t)(A.col0 + c0);
  for (int b = threadIdx.x; b < nb; b += NT) {
    const int4 q = __ldg(blk + b);
    const int e0 = 4 * b - lead;  // row position of q.x
    // ids of the block inside the row: positions [max(0, -e0), min(4, hn - e0))
    const uint32_t keep = (0xFu >> max(0, 4 - (hn - e0))) & (0xFu << max(0, -e0)) & 0xFu;
    const uint32_t dd[4] = {(uint32_t)q.x - base, (uint32_t)q.y - base,   // ids outside the
                            (uint32_t)q.z - base, (uint32_t)q.w - base};  // chunk wrap past n
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const uint32_t d = dd[k];
      if ((keep & (1u << k)) && d < (uint32_t)n) {
        if (OWNER) {
          const uint32_t f4 = d >> 2, bit = ((f4 / NT) << 2) | (d & 3);
          atomicOr(&penmask[(f4 % NT) * kWordsPerThread + (bit >> 5)], 1u << (bit & 31));
        } else {
          atomicOr(&penmask[d >> 5], 1u << (d & 31));
        }
      }
    }
  }
}

template <int NT>
__device__ __forceinline__ void pen_bitmap(const Args& A, int r, int c0, int n, uint32_t* penmask) {
  pen_scan<NT, false>(A, A.hist_off[r], A.hist_off[r + 1], c0, n, penmask);
}

// Threads of a chunk CTA.  Sampled rows take 256 (64 logits per thread: the
// per-thread work outside the streaming loops is paid once per 64 logits);
// greedy rows keep 512, since their CTAs also run the row finalize.
template <int MODE>
__host__ __device__ constexpr int chunk_threads() { return MODE == kGreedy ? kThreads : 256; }

// FIN (top-k rows of small batches only): the last CTA of each row finalizes
// it here, as greedy rows do, instead of a second grid.
template <int MODE, bool PEN, bool FIN = false>
__global__ void __launch_bounds__(chunk_threads<MODE>(), 3) sample_kernel(const __grid_constant__ Args A) {
  constexpr int NT = chunk_threads<MODE>(), NW = NT / 32;
  constexpr int kPenWords = kChunk / 32 / NT;  // penalty bitmap words per thread
  extern __shared__ __align__(128) unsigned char dyn_smem[];
  float* tile = reinterpret_cast<float*>(dyn_smem);
  __shared__ __align__(8) uint64_t bar[kSub];
  __shared__ __align__(8) uint64_t stall_bar;  // test hook: an mbarrier nothing completes
  __shared__ uint32_t penmask[kChunk / 32];  // penalty bits, thread-major (pen_scan OWNER)
  __shared__ int is_last;
  __shared__ int q_cnt;  // candidates found (may exceed kCap: overflow)
  __shared__ float w_max[NW];
  __shared__ uint32_t w_mk[NW], w_tk[NW];
  __shared__ double w_sum[NW];
  __shared__ int w_bi[NW];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r = blockIdx.x, c = blockIdx.y;  // rows vary fastest in launch order
  const int c0 = c * kChunk;
  const int n = min(kChunk, A.V - c0);
  const float* g = A.logits + (int64_t)r * A.ld + c0;
  const bool bulk = ((reinterpret_cast<uintptr_t>(g) & 15) == 0) && ((n & 3) == 0);
  const bool stall = A.test_wait > 0 && r == 0 && c == 0;
  // the row's history range, loaded now so the load overlaps the setup
  int64_t h0 = 0, h1 = 0;
  if (PEN) {
    h0 = __ldg(A.hist_off + r);
    h1 = __ldg(A.hist_off + r + 1);
  }

  if (tid == 0) {
    if (bulk)
      for (int s = 0; s < kSub; s++) mbar_init(&bar[s], 1);
    if (stall) mbar_init(&stall_bar, 1);
    if (bulk || stall) fence_mbar_init();
  }
  if (PEN)
#pragma unroll
    for (int q = 0; q < kPenWords; q++) penmask[tid + q * NT] = 0u;
  if (tid == 0) q_cnt = 0;
  // whole-vocabulary rows: the chunk's mass histogram.  Counts (packed u16
  // pairs) only when a rank is selected (top_k above kKmax).  Masses in one
  // 32-bit word per bin, scaled per bin: an element of local bin b has a fast
  // term e within 2^(+-1/16) of 2^(-b/16), so q = e * hscale[b] with
  // hscale[b] = 2^(21 + b/16) is below 2^21.1, rounded to within 2^-22 of
  // its value (one atomic per element, no carry word).  A bin of kWrapCount
  // elements or more may have wrapped its word: its mass is written as NaN
  // and the row takes the exact whole-row path.  Both adds are fire and
  // forget: nothing waits for their results.
  uint32_t* hcnt = reinterpret_cast<uint32_t*>(dyn_smem + kChunk * sizeof(float));
  uint32_t* hq = hcnt + kNB / 2;
  float* hscale = reinterpret_cast<float*>(hq + kNB);
  constexpr uint32_t kWrapCount = 1900;  // below 2^32 / 2^21.0625, the bound on q
  if constexpr (MODE == kFull) {
    for (int b = tid; b < kNB / 2 + kNB; b += NT) hcnt[b] = 0u;
    for (int b = tid; b < kNB; b += NT) hscale[b] = nuc_scale(b);
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
    for (int j = tid; j < n; j += NT) tile[j] = __ldg(g + j);
  }
  for (int j = n + tid; j < kChunk; j += NT) tile[j] = -INFINITY;

  // ---- penalty bitmap of this chunk, built while the copies are in flight
  if (PEN) pen_scan<NT, true>(A, h0, h1, c0, n, penmask);
  // one thread waits for the copies; the rest park at the barrier
  int timed_out = 0;
  if (bulk && tid == 0) {
    for (int s = 0; s < kSub; s++)
      if (s * kSubElems < n && !mbar_wait(&bar[s], 0, kWaitCycles)) timed_out = 1;
  }
  // test hook (ms_debug_inject): no arrival ever completes stall_bar's phase, so
  // this wait runs out after A.test_wait cycles; no copy is issued against it
  if (stall && tid == 0 && !mbar_wait(&stall_bar, 0, A.test_wait)) timed_out = 1;
  if (__syncthreads_or(timed_out)) {
    // The call fails (status word = this call's epoch); the CTA still runs to
    // the end on whatever the tile holds, so the row counters stay consistent.
    if (tid == 0) {
      atomicExch(A.status, A.epoch);
      if (bulk)  // let any copy still in flight land before going on (bounded)
        for (int s = 0; s < kSub; s++)
          if (s * kSubElems < n) mbar_wait(&bar[s], 0, kWaitCycles);
    }
    __syncthreads();
  }

  // ---- the penalty, applied in shared memory by the thread that reads each
  // flagged element in the streaming loops (its bits of the thread-major
  // bitmap), so no barrier is needed before those loops
  if (PEN) {
#pragma unroll
    for (int q = 0; q < kPenWords; q++) {
      uint32_t w = penmask[tid * kPenWords + q];
      while (w) {
        const int b = 32 * q + __ffs(w) - 1;  // bit 4 * step + lane of the float4
        w &= w - 1;
        const int j = 4 * (tid + (b >> 2) * NT) + (b & 3);
        tile[j] = pen_apply_fast(tile[j], A.pen, A.rpen);
      }
    }
  }

  // diagnostics: the penalised logits, the reference's `work` before the
  // temperature divide (src/generation.js:72-75); called after a barrier that
  // follows the first streaming loop
  auto write_pen_diag = [&]() {
    float* dp = A.d_pen + (int64_t)r * A.pen_ld + c0;
    for (int j = tid; j < n; j += NT) dp[j] = tile[j];
  };

  const float4* t4 = reinterpret_cast<const float4*>(tile);
  constexpr int kIters = kChunk / 4 / NT;  // float4 per thread
  static_assert(kIters <= 32, "one candidate-mask bit per float4 of a thread");

  if (MODE == kGreedy) {
    // first index of the strict max (src/generation.js:51-55)
    float bv = -INFINITY;
    int bi = INT_MAX;
#pragma unroll 4
    for (int i = 0; i < kIters; i++) {
      const int q = tid + i * NT;
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
    if (A.d_pen) write_pen_diag();
    if (tid == 0) {
      for (int w = 1; w < NW; w++)
        if (w_max[w] > bv || (w_max[w] == bv && w_bi[w] < bi)) { bv = w_max[w]; bi = w_bi[w]; }
      ChunkStat st;
      st.m = bv; st.tau = bv; st.s = 0.0; st.n_cand = 0; st.best_i = bi; st.zref = 0.f; st.sig = bv;
      A.stats[(int64_t)r * A.n_chunks + c] = st;
    }
  } else {
    // ---- pass A: thread maxima -> chunk max and tau
    float tm = -INFINITY;
#pragma unroll 4
    for (int i = 0; i < kIters; i++) {
      const float4 v = t4[tid + i * NT];
      tm = fmax3(fmax3(tm, v.x, v.y), v.z, v.w);
    }
    // The warp's kw-th largest thread maximum, by kw rounds of a warp max
    // reduction over order-preserving keys, removing one instance per round.
    // At least kw thread maxima of every warp are >= it, so tau = min over
    // warps is reached by >= NW*kw >= top_k distinct elements of the chunk.
    // A partial chunk (n < 4 * NT) has data in its first w_act warps only, and
    // takes a larger per-warp rank so those warps still cover keff.
    const int keff = (MODE == kTopK) ? A.k : A.ksum;
    const int w_act = (n >= 4 * NT) ? NW : min(NW, ((n + 3) / 4 + 31) / 32);
    const int kwc = min(32, max(1, (keff + w_act - 1) / w_act));
    const uint32_t tkey = fkey(tm);  // tm is never NaN
    const uint32_t wmk = __reduce_max_sync(kAll, tkey);
    uint32_t kk = tkey, wtk = wmk;
    for (int t = 0; t < kwc; t++) {
      wtk = __reduce_max_sync(kAll, kk);
      const unsigned eq = __ballot_sync(kAll, kk == wtk);
      if (lane == __ffs(eq) - 1) kk = 0u;  // below every float key
    }
    if (lane == 0) { w_mk[warp] = wmk; w_tk[warp] = wtk; }
    __syncthreads();
    if (A.d_pen) write_pen_diag();
    const float m = fkey_inv(__reduce_max_sync(kAll, lane < NW ? w_mk[lane] : 0u));
    // Warps whose kwc-th thread maximum is -inf (padding past the row end, or
    // -inf logits) are left out of the minimum.  The minimum over the others
    // is the chunk's top-k bound tau when they alone hold keff elements
    // (kwc each); otherwise tau = -inf.  sig is the storage threshold: every
    // element >= sig becomes a candidate, and the finalizer falls back to the
    // exact rescan when some chunk's sig is above the row's tau.
    const uint32_t wk = lane < NW ? w_tk[lane] : 0u;
    const bool wok = wk > fkey(-INFINITY);
    const int n_ok = __popc(__ballot_sync(kAll, wok));
    const float tmin = n_ok ? fkey_inv(__reduce_min_sync(kAll, wok ? wk : 0xFFFFFFFFu)) : -INFINITY;
    const float tau = (n_ok * kwc >= keff) ? tmin : -INFINITY;
    // a chunk too small for a bound keeps everything when it fits its list
    const float sig = (tau == -INFINITY && n <= kCap) ? -INFINITY : tmin;

    // ---- pass B: fast exp sum (Kahan in fp32) and the float4 that hold
    // candidates (elements >= sig)
    const float mref = (m == -INFINITY) ? 0.f : m;
    const float a = A.a;
    // fast terms 2^(x * a - zref) with zref = fp32(m * a); a chunk whose m * a
    // leaves the fp32 range keeps the two-step form 2^((x - m) * a) (zref NaN)
    const float zr = __fmul_rn(mref, a);
    const bool zok = fabsf(zr) <= FLT_MAX;
    const float zref = zok ? zr : __int_as_float(0x7fc00000);
    float s = 0.f, comp = 0.f;
    uint32_t cmask = 0;  // bit i: this thread's float4 of step i holds an element >= sig
    const float a16 = __fmul_rn(a, 16.f);
    const int btop = nuc_bin(m, a16);  // the chunk's top bin (INT_MAX: a chunk of -inf)
    const bool hcounts = A.h_cnt != nullptr;
    auto hist_add = [&](float x, float e) {
      if (x != x) return;  // a NaN makes the whole row NaN
      const int lb = nuc_local(nuc_bin(x, a16), btop);
      atomicAdd(&hcnt[lb >> 1], 1u << ((lb & 1) << 4));  // u16 pairs: a chunk holds < 2^16
      atomicAdd(&hq[lb], __float2uint_rn(__fmul_rn(e, hscale[lb])));
    };
    auto kahan = [&](float t) {
      const float y = __fsub_rn(t, comp);
      const float ss = __fadd_rn(s, y);
      comp = __fsub_rn(__fsub_rn(ss, s), y);
      s = ss;
    };
    if (n == kChunk && zok) {
      // hot loop: both pairs of a float4 in one paired fma each
      const unsigned long long a2 = f2_pack(a, a), nz2 = f2_pack(-zref, -zref);
#pragma unroll 4
      for (int i = 0; i < kIters; i++) {
        const float4 v = t4[tid + i * NT];
        const float2 z01 = f2_unpack(f2_fma(f2_pack(v.x, v.y), a2, nz2));
        const float2 z23 = f2_unpack(f2_fma(f2_pack(v.z, v.w), a2, nz2));
        const unsigned long long e01 = f2_pack(ex2_approx(z01.x), ex2_approx(z01.y));
        const unsigned long long e23 = f2_pack(ex2_approx(z23.x), ex2_approx(z23.y));
        const float2 t2 = f2_unpack(f2_add(e01, e23));
        kahan(__fadd_rn(t2.x, t2.y));
        cmask |= (uint32_t)(fmaxf(fmax3(v.x, v.y, v.z), v.w) >= sig) << i;
        if constexpr (MODE == kFull) {
          const float2 ea = f2_unpack(e01), eb = f2_unpack(e23);
          hist_add(v.x, ea.x);
          hist_add(v.y, ea.y);
          hist_add(v.z, eb.x);
          hist_add(v.w, eb.y);
        }
      }
    } else {
      // partial chunk, or zref out of range: one element at a time
      for (int i = 0; i < kIters; i++) {
        const int qq = tid + i * NT;
        const float4 v = t4[qq];
        const int j = 4 * qq;
        const float xs[4] = {v.x, v.y, v.z, v.w};
        float e[4];
#pragma unroll
        for (int l = 0; l < 4; l++) {
          e[l] = zok ? term_fast_z(xs[l], a, zref) : term_fast(xs[l], mref, a);
          if (j + l >= n) e[l] = 0.f;  // padding past the row end contributes nothing
          if constexpr (MODE == kFull)
            if (j + l < n) hist_add(xs[l], e[l]);
        }
        kahan(__fadd_rn(__fadd_rn(e[0], e[2]), __fadd_rn(e[1], e[3])));
        cmask |= (uint32_t)(fmaxf(fmax3(v.x, v.y, v.z), v.w) >= sig) << i;
      }
    }
    // candidates: each flagged float4 appends its elements >= sig to the
    // chunk's global list (slots from a shared counter; the list's order is
    // free, the finalizer sorts)
    Cand* dst = A.cands + ((int64_t)r * A.n_chunks + c) * kCap;
    while (cmask) {
      const int i = __ffs(cmask) - 1;
      cmask &= cmask - 1u;
      const int qq = tid + i * NT;
      const float4 v = t4[qq];
      const int j = 4 * qq, gj = c0 + j;
      const bool k0 = v.x >= sig && j < n, k1 = v.y >= sig && j + 1 < n;
      const bool k2 = v.z >= sig && j + 2 < n, k3 = v.w >= sig && j + 3 < n;
      int pos = atomicAdd(&q_cnt, (int)k0 + (int)k1 + (int)k2 + (int)k3);
      if (k0) { if (pos < kCap) dst[pos] = Cand{v.x, gj}; pos++; }
      if (k1) { if (pos < kCap) dst[pos] = Cand{v.y, gj + 1}; pos++; }
      if (k2) { if (pos < kCap) dst[pos] = Cand{v.z, gj + 2}; pos++; }
      if (k3 && pos < kCap) dst[pos] = Cand{v.w, gj + 3};
    }
    double ds = (double)s - (double)comp;
    ds = warp_sum(ds);
    if (lane == 0) w_sum[warp] = ds;
    __syncthreads();
    if (warp == 0) {
      const double S = warp_sum(lane < NW ? w_sum[lane] : 0.0);
      if (lane == 0) {
        ChunkStat st;
        st.m = m; st.tau = tau; st.s = S; st.n_cand = min(q_cnt, kCap + 1);
        // whole-vocabulary rows keep the chunk's top histogram bin here
        st.best_i = (MODE == kFull) ? btop : INT_MAX;
        st.zref = zref; st.sig = sig;
        A.stats[(int64_t)r * A.n_chunks + c] = st;
      }
    }
    if constexpr (MODE == kFull) {
      const int64_t hb = ((int64_t)r * A.n_chunks + c) * kNB;
      for (int b = tid; b < kNB; b += NT) {
        const uint32_t cnt = (hcnt[b >> 1] >> ((b & 1) << 4)) & 0xFFFFu;
        if (hcounts) A.h_cnt[hb + b] = (uint16_t)cnt;
        A.h_mass[hb + b] = cnt >= kWrapCount ? __longlong_as_double(0x7ff8000000000000ll)
                                             : (double)hq[b] / (double)hscale[b];
      }
    }
  }

  // ---- the last chunk of the row to finish finalizes it (unless a separate
  // finalize kernel follows)
  if (MODE != kGreedy && !FIN) {
    // sampled rows: finalize_kernel follows; let it launch while the last
    // chunks stream
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    return;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int old = atomicAdd(&A.row_count[r], 1);
    is_last = (old == A.n_chunks - 1);
    if (is_last) A.row_count[r] = 0;  // ready for the next call
  }
  __syncthreads();
  if (is_last) {
    __threadfence();
    if (*((volatile int32_t*)A.status) != A.epoch) {
      finalize_row<MODE>(A, r, *reinterpret_cast<FinSmem*>(dyn_smem));
    } else if (tid == 0) {  // a wait of this call ran out: the row has no id
      A.out_ids[r] = -1;
      if (A.d_row_flags) A.d_row_flags[r] = MS_ROW_TIMEOUT;
    }
  }
}

// Row finalize as its own grid (one CTA per row), launched as a programmatic
// dependent of sample_kernel: it waits for the whole stream grid's writes.
// NT threads per row: 512, or 256 for large top-k batches, whose rows then fit
// one wave (4 CTAs per SM)
template <int MODE, int NT>
__global__ void __launch_bounds__(NT, kThreads * 2 / NT) finalize_kernel(const __grid_constant__ Args A) {
  extern __shared__ __align__(128) unsigned char fin_smem[];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (*((volatile int32_t*)A.status) == A.epoch) {  // a wait of this call ran out
    if (threadIdx.x == 0) {
      A.out_ids[blockIdx.x] = -1;
      if (A.d_row_flags) A.d_row_flags[blockIdx.x] = MS_ROW_TIMEOUT;
    }
    return;
  }
  finalize_row<MODE>(A, blockIdx.x, *reinterpret_cast<FinSmem*>(fin_smem));
}

// =============================================================== vocabulary shards
// One record per row and shard: a header, then up to k_send candidates.
struct ShardHead {
  float M;         // max of the shard's penalised logits (-inf: none)
  float t;         // every shard element with x >= t is in the list (-inf: the whole shard)
  int32_t n;       // list length
  int32_t flags;   // kRecBad: the softmax is NaN; kRecIncomplete: the list cannot be trusted
  double S;        // fast softmax partial sum, in units of exp(x' - Mp_g), Mp_g = fp32(M / T)
  int32_t best_i;  // greedy: global index of the shard's first max (INT_MAX: none)
  int32_t x0nan;   // greedy: the shard holds column 0 and it is NaN
};
struct ShardCand {
  float x;         // penalised logit
  int32_t id;      // global id
  double f;        // its fast term, in the header's S units
};
static_assert(sizeof(ShardHead) == 32 && sizeof(ShardCand) == 16, "shard record layout");
constexpr int kRecBad = 1, kRecIncomplete = 2;
static_assert(sizeof(ShardHead) == kRecHead && sizeof(ShardCand) == kRecCand, "record sizes");

// The k-th largest x of the nfc gathered candidates (1 <= k <= nfc), ties
// counted: two 8-bit digits of the order-preserving key pick its bucket, whose
// members are ranked.  F.h1, F.h2, F.n_bkt are zero on entry.  NaN when the
// bucket is too large to rank (the caller gives up on the row).
__device__ float kth_largest_x(FinSmem& F, int nfc, int k) {
  const int tid = threadIdx.x, warp = tid >> 5, nt = (int)blockDim.x;
  // larger x first = ascending ~fkey(x)
  for (int j = tid; j < nfc; j += nt) atomicAdd(&F.h1[~fkey(F.gath[j].x) >> 24], 1);
  __syncthreads();
  if (warp == 0) scan_pick(F.h1, k, &F.b1, &F.need);
  __syncthreads();
  const uint32_t b1 = (uint32_t)F.b1;
  for (int j = tid; j < nfc; j += nt) {
    const uint32_t key = ~fkey(F.gath[j].x);
    if ((key >> 24) == b1) atomicAdd(&F.h2[(key >> 16) & 255], 1);
  }
  __syncthreads();
  if (warp == 0) scan_pick(F.h2, F.need, &F.b2, &F.need);
  __syncthreads();
  const uint32_t p16 = (b1 << 8) | (uint32_t)F.b2;
  const int need = F.need;
  for (int j = tid; j < nfc; j += nt) {
    const uint32_t key = ~fkey(F.gath[j].x);
    if ((key >> 16) == p16) {
      const int q = atomicAdd(&F.n_bkt, 1);
      if (q < kFinMax) F.keys[q] = key;
    }
  }
  __syncthreads();
  const int nb = F.n_bkt;
  if (nb > kFinMax) return __int_as_float(0x7fc00000);
  // the need-th smallest key v of the bucket: #(< v) < need <= #(<= v)
  for (int t = tid; t < nb; t += nt) {
    const uint32_t kt = (uint32_t)F.keys[t];
    int lt = 0, le = 0;
    for (int j = 0; j < nb; j++) {
      const uint32_t kj = (uint32_t)F.keys[j];
      lt += kj < kt;
      le += kj <= kt;
    }
    if (lt < need && le >= need) F.kx = kt;  // every writer writes the same value
  }
  __syncthreads();
  return fkey_inv(~F.kx);
}

// softmax NaN everywhere (src/generation.js:9-17 with a NaN sum): the stable
// sort keeps id order, no acc reaches topP, r is NaN, and the draw loop falls
// through to the last candidate
__device__ void nan_row_out(const Args& A, int r, float Mp) {
  const bool use_k = A.k > 0 && A.k < A.V;
  A.out_ids[r] = use_k ? A.k - 1 : A.V - 1;
  if (A.d_n_cand) A.d_n_cand[r] = use_k ? A.k : A.V;
  if (A.d_row_max) A.d_row_max[r] = (double)Mp;
  if (A.d_row_sum) A.d_row_sum[r] = __longlong_as_double(0x7ff8000000000000ll);
  if (A.d_total) A.d_total[r] = __longlong_as_double(0x7ff8000000000000ll);
  if (A.d_row_flags) A.d_row_flags[r] = MS_ROW_NAN;
}

// Row records of one vocabulary shard (one CTA per row), a programmatic
// dependent of the shard's chunk kernel.
template <int MODE>
__global__ void __launch_bounds__(256, 4) shard_kernel(const __grid_constant__ Args A) {
  extern __shared__ __align__(128) unsigned char fin_smem[];
  FinSmem& F = *reinterpret_cast<FinSmem*>(fin_smem);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nt = (int)blockDim.x;
  const int r = blockIdx.x;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  ShardHead* H = reinterpret_cast<ShardHead*>(A.rec + (int64_t)r * A.rec_bytes);
  ShardCand* L = reinterpret_cast<ShardCand*>(H + 1);
  const ChunkStat* st = A.stats + (int64_t)r * A.n_chunks;
  if (MODE == kGreedy) {
    if (warp == 0) {
      float bv = -INFINITY;
      int bi = INT_MAX;
      for (int c = lane; c < A.n_chunks; c += 32) {
        const float v = __ldcg(&st[c].m);
        const int i = __ldcg(&st[c].best_i);
        if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(kAll, bv, o);
        const int oi = __shfl_xor_sync(kAll, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      if (lane == 0) {
        ShardHead h;
        h.M = bv; h.t = -INFINITY; h.n = 0; h.flags = 0; h.S = 0.0;
        h.best_i = (bv == -INFINITY || bi == INT_MAX) ? INT_MAX : A.col0 + bi;
        const float x0 = A.logits[(int64_t)r * A.ld];
        h.x0nan = (A.col0 == 0 && x0 != x0) ? 1 : 0;
        *H = h;
      }
    }
    return;
  }
  const int timed_out = *((volatile int32_t*)A.status) == A.epoch;
  row_stats(A, r, F);
  if (F.nan_row || timed_out) {
    if (tid == 0) {
      ShardHead h;
      h.M = F.M; h.t = -INFINITY; h.n = 0; h.S = 0.0; h.best_i = INT_MAX; h.x0nan = 0;
      h.flags = timed_out ? kRecIncomplete : (F.bad ? kRecBad : 0);
      *H = h;
    }
    return;
  }
  gather_cands(A, r, F);
  const int nf = F.nf, nfc = min(nf, kGathMax);
  bool incomplete = F.slow || nf > kGathMax;
  float t = F.tau_row;  // all gathered: every element >= tau_row
  if (!incomplete && nfc > A.k) {
    t = kth_largest_x(F, nfc, A.k);
    incomplete = (t != t);
  }
  if (tid == 0) F.n_top = 0;
  __syncthreads();
  if (!incomplete) {
    for (int j = tid; j < nfc; j += nt) {
      const Cand cd = F.gath[j];
      if (cd.x >= t) {
        const int q = atomicAdd(&F.n_top, 1);
        if (q < A.k_send) {
          const int c = cd.i / kChunk;
          const float mc = c < kFinChunks ? F.cm[c] : __ldcg(&st[c].m);
          const float zc = c < kFinChunks ? F.cz[c] : __ldcg(&st[c].zref);
          const double sc = c < kFinChunks ? F.cs[c] : chunk_scale(A, mc, zc, F.Mp);
          ShardCand e;
          e.x = cd.x; e.id = A.col0 + cd.i; e.f = (double)chunk_term(A, cd.x, mc, zc) * sc;
          L[q] = e;
        }
      }
    }
  }
  __syncthreads();
  if (tid == 0) {
    const bool full = incomplete || F.n_top > A.k_send;
    ShardHead h;
    h.M = F.M; h.t = t; h.n = full ? 0 : F.n_top; h.flags = full ? kRecIncomplete : 0;
    h.S = F.S_fast; h.best_i = INT_MAX; h.x0nan = 0;
    *H = h;
  }
}

// Merge of the G shard records of each row (one CTA per row).
template <int MODE>
__global__ void __launch_bounds__(256, 4) merge_kernel(const __grid_constant__ Args A) {
  extern __shared__ __align__(128) unsigned char fin_smem[];
  FinSmem& F = *reinterpret_cast<FinSmem*>(fin_smem);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nt = (int)blockDim.x;
  const int r = blockIdx.x, G = A.G;
  const unsigned char* base = A.rec + (int64_t)r * G * A.rec_bytes;
  auto head = [&](int g) { return reinterpret_cast<const ShardHead*>(base + (int64_t)g * A.rec_bytes); };
  auto unsettled = [&]() {
    A.out_ids[r] = -1;
    if (A.d_n_cand) A.d_n_cand[r] = 0;
    if (A.d_row_flags) A.d_row_flags[r] = MS_ROW_UNSETTLED;
  };
  if (MODE == kGreedy) {
    if (warp == 0) {
      float bv = -INFINITY;
      int bi = INT_MAX, x0n = 0;
      for (int g = lane; g < G; g += 32) {
        const ShardHead h = *head(g);
        if (h.best_i != INT_MAX && (h.M > bv || (h.M == bv && h.best_i < bi))) { bv = h.M; bi = h.best_i; }
        x0n |= h.x0nan;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(kAll, bv, o);
        const int oi = __shfl_xor_sync(kAll, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        x0n |= __shfl_xor_sync(kAll, x0n, o);
      }
      if (lane == 0) {
        // src/generation.js:51-55: a NaN at index 0 is never beaten
        A.out_ids[r] = (x0n || bi == INT_MAX) ? 0 : bi;
        if (A.d_row_flags) A.d_row_flags[r] = MS_ROW_GREEDY;
        if (A.d_n_cand) A.d_n_cand[r] = 0;
        if (A.d_row_max) A.d_row_max[r] = (double)bv;
      }
    }
    return;
  }
  if (warp == 0) {
    float M = -INFINITY;
    int fl = 0, n = 0;
    ShardHead h;
    if (lane < G) {
      h = *head(lane);
      M = h.M;
      fl = h.flags;
      n = h.n;
    }
    float Mx = M;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      Mx = fmaxf(Mx, __shfl_xor_sync(kAll, Mx, o));
      fl |= __shfl_xor_sync(kAll, fl, o);
    }
    const float Mp = temper_fast(Mx, A.T, A.rT, A.temper);
    const int bad = (fl & kRecBad) | (Mp != Mp) | (isinf(Mp) && Mx != -INFINITY);
    double S = 0.0, scale = 0.0;
    if (lane < G && M != -INFINITY && !bad) {
      scale = exp((double)temper_fast(M, A.T, A.rT, A.temper) - (double)Mp);
      S = h.S * scale;
    }
    S = warp_sum(S);
    int incl = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(kAll, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane < G) { F.off[lane] = incl - n; F.cs[lane] = scale; F.cm[lane] = h.t; }
    if (lane == 31) F.nf = incl;
    if (lane == 0) {
      F.M = Mx; F.Mp = Mp; F.nan_row = bad | (Mx == -INFINITY); F.slow = (fl & kRecIncomplete) ? 1 : 0;
      F.S_fast = S; F.corr = 0ull; F.u = A.u ? __ldg(A.u + r) : 0.0;
    }
  } else if (warp == 1) {
    for (int b = lane; b < 256; b += 32) { F.h1[b] = 0; F.h2[b] = 0; }
    if (lane == 0) { F.n_top = 0; F.n_bkt = 0; }
  }
  __syncthreads();
  const float Mp = F.Mp;
  if (F.nan_row) {
    if (tid == 0) nan_row_out(A, r, Mp);
    return;
  }
  const int nall = F.nf;
  if (F.slow || nall > kGathMax || nall < A.k) {
    if (tid == 0) unsettled();
    return;
  }
  // exact terms of the union, and the correction of the fast sum
  {
    long long corr = 0;
    for (int j = tid; j < nall; j += nt) {
      int g = 0;
      while (g + 1 < G && F.off[g + 1] <= j) g++;
      const ShardCand* L = reinterpret_cast<const ShardCand*>(head(g) + 1);
      const ShardCand c = L[j - F.off[g]];
      const float e = term_exact(temper_fast(c.x, A.T, A.rT, A.temper), Mp);
      corr += __double2ll_rn(((double)e - c.f * F.cs[g]) * 1125899906842624.0);
      F.gath[j] = Cand{e, c.id};
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) corr += __shfl_xor_sync(kAll, corr, o);
    if (lane == 0 && corr != 0) atomicAdd(&F.corr, (unsigned long long)corr);
  }
  __syncthreads();
  const double S = F.S_fast + (double)(long long)F.corr * (1.0 / 1125899906842624.0);
  const double rS = 1.0 / S;
  // an element outside shard g's list has x < t_g
  if (warp == 0) {
    float po = -1.f;
    if (lane < G) {
      const float t = F.cm[lane];
      if (t != -INFINITY)
        po = div_to_f32((double)term_exact(temper_fast(fkey_inv(fkey(t) - 1u), A.T, A.rT, A.temper), Mp), S, rS);
    }
    po = warp_max(po);
    if (lane == 0) F.pout = po;
  }
  if (!topk_from_terms(A, r, F, nall, S, rS, Mp)) {
    if (tid == 0) unsettled();
  }
}

}  // namespace ms

#include "ms_nucleus.cuh"

namespace ms {

static_assert(sizeof(FinSmem) <= kChunk * sizeof(float), "finalize scratch must fit in the chunk tile");
static_assert(sizeof(FullSmem) <= kChunk * sizeof(float), "full-row scratch must fit in the chunk tile");
static_assert(kChunk / 32 % 256 == 0 && kChunk / 32 % kThreads == 0, "whole penalty bitmap words per thread");

// =============================================================== launch
namespace {
constexpr size_t kSmem = (size_t)kChunk * sizeof(float);
// whole-vocabulary chunk kernels also hold the chunk's mass histogram
constexpr size_t kSmemFull = kSmem + (size_t)(kNB / 2 + 2 * kNB) * sizeof(uint32_t);  // counts, masses, scales
constexpr size_t kResSmem = sizeof(ResSmem) > sizeof(FullSmem) ? sizeof(ResSmem) : sizeof(FullSmem);

template <int MODE>
constexpr size_t chunk_smem() { return MODE == kFull ? kSmemFull : kSmem; }

template <int MODE, bool PEN, bool FIN = false>
cudaError_t set_attrs() {
  return cudaFuncSetAttribute((const void*)sample_kernel<MODE, PEN, FIN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)chunk_smem<MODE>());
}

cudaError_t set_nuc_attrs() {
  cudaError_t e = cudaFuncSetAttribute((const void*)nucleus_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)sizeof(NucSmem));
  for (const void* f : {(const void*)nucleus_extract_kernel<false>, (const void*)nucleus_extract_kernel<true>})
    if (e == cudaSuccess) e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute((const void*)nucleus_resolve_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kResSmem);
  return e;
}

// A launch that may start while the grid before it on the stream finishes
// (it waits with griddepcontrol.wait where it needs that grid's results).
template <typename K>
cudaError_t launch_pdl(K kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, const Args& S) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, S);
}

constexpr size_t kFinSmem = sizeof(FullSmem) > sizeof(FinSmem) ? sizeof(FullSmem) : sizeof(FinSmem);

template <int MODE, int NT>
cudaError_t set_fin_attrs() {
  return cudaFuncSetAttribute((const void*)finalize_kernel<MODE, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)kFinSmem);
}

template <int MODE, bool PEN>
cudaError_t launch_mode(const Args& S, dim3 grid, cudaStream_t stream, cudaEvent_t mid) {
  if constexpr (MODE == kTopK) {
    if (S.fuse_fin) {  // one launch: the last chunk CTA of each row finalizes it
      sample_kernel<MODE, PEN, true><<<grid, dim3(chunk_threads<MODE>()), chunk_smem<MODE>(), stream>>>(S);
      cudaError_t e = cudaGetLastError();
      if (mid) cudaEventRecord(mid, stream);
      return e;
    }
  }
  sample_kernel<MODE, PEN><<<grid, dim3(chunk_threads<MODE>()), chunk_smem<MODE>(), stream>>>(S);
  cudaError_t e = cudaGetLastError();
  if (mid) cudaEventRecord(mid, stream);
  if constexpr (MODE == kGreedy) {
    return e;  // the chunk kernel's last CTA of each row picks its id
  } else if constexpr (MODE == kFull) {
    // whole-vocabulary rows: plan, extract, resolve
    if (e == cudaSuccess) e = launch_pdl(nucleus_plan_kernel, dim3(S.B), dim3(kNB), sizeof(NucSmem), stream, S);
    if (e == cudaSuccess)
      e = launch_pdl(nucleus_extract_kernel<PEN>, dim3(S.B, S.n_chunks), dim3(kThreads), kSmem, stream, S);
    if (e == cudaSuccess) e = launch_pdl(nucleus_resolve_kernel, dim3(S.B), dim3(kNB), kResSmem, stream, S);
    return e;
  } else {
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(S.B);
    const bool narrow = MODE == kTopK && S.B >= 256;
    cfg.blockDim = dim3(narrow ? 256 : kThreads);
    cfg.dynamicSmemBytes = kFinSmem;
    cfg.stream = stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    if constexpr (MODE == kTopK)
      if (narrow) return cudaLaunchKernelEx(&cfg, finalize_kernel<MODE, 256>, S);
    return cudaLaunchKernelEx(&cfg, finalize_kernel<MODE, kThreads>, S);
  }
}
}  // namespace

namespace {
constexpr size_t kShardSmem = sizeof(FinSmem);

template <int MODE>
cudaError_t launch_shard_mode(const Args& S, bool pen, cudaStream_t stream) {
  const dim3 grid(S.B, S.n_chunks);
  if (pen) sample_kernel<MODE, true><<<grid, dim3(chunk_threads<MODE>()), kSmem, stream>>>(S);
  else sample_kernel<MODE, false><<<grid, dim3(chunk_threads<MODE>()), kSmem, stream>>>(S);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(S.B);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = kShardSmem;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, shard_kernel<MODE>, S);
}

bool g_shard_attrs[64] = {false};
cudaError_t shard_attrs(int dev) {
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (g_shard_attrs[dev]) return cudaSuccess;
  cudaError_t e = cudaSuccess;
  if (e == cudaSuccess) e = set_attrs<kGreedy, false>();
  if (e == cudaSuccess) e = set_attrs<kGreedy, true>();
  if (e == cudaSuccess) e = set_attrs<kTopK, false>();
  if (e == cudaSuccess) e = set_attrs<kTopK, true>();
  for (const void* f : {(const void*)shard_kernel<kGreedy>, (const void*)shard_kernel<kTopK>,
                        (const void*)merge_kernel<kGreedy>, (const void*)merge_kernel<kTopK>})
    if (e == cudaSuccess) e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kShardSmem);
  if (e == cudaSuccess) g_shard_attrs[dev] = true;
  return e;
}
}  // namespace

// Chunk kernel over a vocabulary shard, then its row records.
cudaError_t launch_shard(const Args& A, cudaStream_t stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t e = shard_attrs(dev);
  if (e != cudaSuccess) return e;
  return A.mode == kGreedy ? launch_shard_mode<kGreedy>(A, A.use_pen != 0, stream)
                           : launch_shard_mode<kTopK>(A, A.use_pen != 0, stream);
}

// Merge of the shard records, one CTA per row.
cudaError_t launch_merge(const Args& A, cudaStream_t stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t e = shard_attrs(dev);
  if (e != cudaSuccess) return e;
  if (A.mode == kGreedy) merge_kernel<kGreedy><<<dim3(A.B), dim3(256), kShardSmem, stream>>>(A);
  else merge_kernel<kTopK><<<dim3(A.B), dim3(256), kShardSmem, stream>>>(A);
  return cudaGetLastError();
}

// Appends ids[r] to row r's device history (hist[r * cap + len[r]], then
// len[r] + 1); ids < 0 and full rows are skipped.
__global__ void history_append_kernel(int32_t* hist, int32_t* len, int64_t B, int64_t cap, const int32_t* ids) {
  const int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (r >= B) return;
  const int32_t id = ids[r];
  const int32_t n = len[r];
  if (id < 0 || n < 0 || n >= cap) return;
  hist[r * cap + n] = id;
  len[r] = n + 1;
}

cudaError_t launch_history_append(int32_t* hist, int32_t* len, int64_t B, int64_t cap, const int32_t* ids,
                                  cudaStream_t stream) {
  const int64_t blocks = (B + 255) / 256;
  history_append_kernel<<<(unsigned)blocks, 256, 0, stream>>>(hist, len, B, cap, ids);
  return cudaGetLastError();
}

__global__ void exp_kernel(const double* x, double* y, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = js_exp(x[i]);
}

// The exact-term exp over n doubles (test hook: checked against the oracle's).
cudaError_t launch_exp(const double* x, double* y, int64_t n, cudaStream_t stream) {
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, 148 * 8);
  exp_kernel<<<(unsigned)blocks, 256, 0, stream>>>(x, y, n);
  return cudaGetLastError();
}

cudaError_t launch_sample(const Args& A, cudaStream_t stream, cudaEvent_t* ev, int64_t* launched) {
  static bool attrs_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attrs_done[dev]) {
    cudaError_t e = cudaSuccess;
    if (e == cudaSuccess) e = set_attrs<kGreedy, false>();
    if (e == cudaSuccess) e = set_attrs<kGreedy, true>();
    if (e == cudaSuccess) e = set_attrs<kTopK, false>();
    if (e == cudaSuccess) e = set_attrs<kTopK, true>();
    if (e == cudaSuccess) e = set_attrs<kTopK, false, true>();
    if (e == cudaSuccess) e = set_attrs<kTopK, true, true>();
    if (e == cudaSuccess) e = set_attrs<kFull, false>();
    if (e == cudaSuccess) e = set_attrs<kFull, true>();
    if (e == cudaSuccess) e = set_fin_attrs<kTopK, 256>();
    if (e == cudaSuccess) e = set_fin_attrs<kTopK, kThreads>();
    if (e == cudaSuccess) e = set_nuc_attrs();
    if (e != cudaSuccess) return e;
    attrs_done[dev] = true;
  }
  // rows in slices small enough that row * n_chunks stays well inside int
  const int64_t rmax = (INT_MAX - (1 << 20)) / A.n_chunks;
  for (int64_t r0 = 0; r0 < A.B; r0 += rmax) {
    Args S = A;
    const int rows = (int)std::min<int64_t>(A.B - r0, rmax);
    S.B = rows;
    S.logits = A.logits + r0 * A.ld;
    if (A.hist_off) S.hist_off = A.hist_off + r0;
    if (A.u) S.u = A.u + r0;
    S.stats = A.stats + r0 * A.n_chunks;
    S.row_count = A.row_count + r0;
    S.cands = A.cands + r0 * A.n_chunks * kCap;
    if (A.penbits) S.penbits = A.penbits + r0 * ((A.V + 31) / 32);
    if (A.h_cnt) {
      S.h_cnt = A.h_cnt + r0 * A.n_chunks * kNB;
      S.h_mass = A.h_mass + r0 * A.n_chunks * kNB;
      S.plan = A.plan + r0;
      S.lists = A.lists + r0 * 2 * kListCap;
      S.list_cnt = A.list_cnt + r0 * 4;
    }
    S.out_ids = A.out_ids + r0;
    if (A.d_cand_ids) S.d_cand_ids = A.d_cand_ids + r0 * A.cand_cap;
    if (A.d_cand_probs) S.d_cand_probs = A.d_cand_probs + r0 * A.cand_cap;
    if (A.d_n_cand) S.d_n_cand = A.d_n_cand + r0;
    if (A.d_row_max) S.d_row_max = A.d_row_max + r0;
    if (A.d_row_sum) S.d_row_sum = A.d_row_sum + r0;
    if (A.d_total) S.d_total = A.d_total + r0;
    if (A.d_row_flags) S.d_row_flags = A.d_row_flags + r0;
    const dim3 grid(rows, A.n_chunks);
    const bool pen = A.use_pen != 0;
    // small top-k batches: the finalize in the chunk kernel saves the second
    // launch; larger ones keep it as its own one-wave grid
    S.fuse_fin = (A.mode == kTopK && rows <= kFuseRows) ? 1 : 0;
    const bool prof = ev != nullptr && r0 == 0;
    if (prof) cudaEventRecord(ev[0], stream);
    cudaEvent_t mid = prof ? ev[1] : nullptr;
    cudaError_t e;
    switch (A.mode) {
      case kGreedy:
        e = pen ? launch_mode<kGreedy, true>(S, grid, stream, mid)
                : launch_mode<kGreedy, false>(S, grid, stream, mid);
        break;
      case kTopK:
        e = pen ? launch_mode<kTopK, true>(S, grid, stream, mid)
                : launch_mode<kTopK, false>(S, grid, stream, mid);
        break;
      default:
        e = pen ? launch_mode<kFull, true>(S, grid, stream, mid)
                : launch_mode<kFull, false>(S, grid, stream, mid);
        break;
    }
    if (prof) cudaEventRecord(ev[2], stream);
    if (e != cudaSuccess) return e;
    if (launched) *launched += (A.mode == kGreedy || S.fuse_fin) ? 1 : (A.mode == kFull ? 4 : 2);
  }
  return cudaSuccess;
}

}  // namespace ms
