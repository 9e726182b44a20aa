// Whole-vocabulary rows (top_k off, or above the candidate path's kKmax):
// the top-p cut and the draw over the full sorted vocabulary
// (src/generation.js:27-49), spread over the whole GPU instead of one CTA per
// row.  Included by ms_kernels.cu after the finalize helpers it uses.
//
// A step is four launches, each a programmatic dependent of the one before:
//   sample_kernel<kFull>    streams every logit once; besides the chunk max,
//                           fast sum and candidates it writes the chunk's mass
//                           histogram (kNB bins of 1/16 log2 unit, counts and
//                           fast masses) while the chunk is in shared memory;
//   nucleus_plan_kernel     one CTA per row: exact softmax sum (fast sum
//                           corrected by the candidates' exact terms), the
//                           chunk histograms merged onto the row's bins, and
//                           the bin ranges that must hold the top-p cut and
//                           the draw (bounds widened by the fast masses' error);
//   nucleus_extract_kernel  the chunk grid again, in reverse order so most of
//                           the row is still in L2: copies out the elements of
//                           those ranges (a few thousand per row);
//   nucleus_resolve_kernel  one CTA per row: ranks each range's elements by
//                           exact (prob desc, id asc) keys, sub-binned by their
//                           exact probability, and walks to the cut and the draw.
// Rows the plan cannot settle (a range beyond kListCap elements, a target too
// close to the total mass, a sub-bin of more than kExtCap tied elements) go to
// the exact single-CTA whole-row path (full_path) in the resolve kernel.
#pragma once

namespace ms {

constexpr int kNSB = 1024;  // probability sub-bins of an extracted range

struct NucSmem {
  FinSmem F;
  long long ccnt[kNB];  // row-bin counts, then their inclusive prefix
  double cmass[kNB];    // row-bin fast masses (probability units), then their prefix
  long long red_c[32];
  double red_d[32];
  int red_i[32];
  int ctop[kFinChunks];  // the chunks' top bins (first kFinChunks chunks)
};

// Inclusive block scan of one value per thread (blockDim.x == kNB).
template <typename T>
__device__ T block_incl_scan(T v, T* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const T t = __shfl_up_sync(kAll, v, o);
    if (lane >= o) v += t;
  }
  if (lane == 31) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    T w = lane < (int)(blockDim.x >> 5) ? red[lane] : T(0);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const T t = __shfl_up_sync(kAll, w, o);
      if (lane >= o) w += t;
    }
    red[lane] = w;
  }
  __syncthreads();
  if (warp > 0) v += red[warp - 1];
  __syncthreads();
  return v;
}

// First row bin whose inclusive prefix reaches t (kNB if none); binary search.
__device__ __forceinline__ int first_mass_ge(const double* cm, double t) {
  int lo = 0, hi = kNB;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (cm[mid] >= t) hi = mid; else lo = mid + 1;
  }
  return lo;
}
__device__ __forceinline__ int first_cnt_ge(const long long* cc, long long t) {
  int lo = 0, hi = kNB;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (cc[mid] >= t) hi = mid; else lo = mid + 1;
  }
  return lo;
}

__device__ void nuc_nan_out(const Args& A, int r, float Mp) {
  const bool use_k = A.k > 0 && A.k < A.V;
  A.out_ids[r] = use_k ? A.k - 1 : A.V - 1;
  if (A.d_n_cand) A.d_n_cand[r] = use_k ? A.k : A.V;
  if (A.d_row_max) A.d_row_max[r] = (double)Mp;
  if (A.d_row_sum) A.d_row_sum[r] = __longlong_as_double(0x7ff8000000000000ll);
  if (A.d_total) A.d_total[r] = __longlong_as_double(0x7ff8000000000000ll);
  if (A.d_row_flags) A.d_row_flags[r] = MS_ROW_NAN;
}

// =============================================================== plan
__global__ void __launch_bounds__(kNB, 2) nucleus_plan_kernel(const __grid_constant__ Args A) {
  extern __shared__ __align__(128) unsigned char nuc_smem[];
  NucSmem& N = *reinterpret_cast<NucSmem*>(nuc_smem);
  FinSmem& F = N.F;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the chunk kernel's stats and histograms
  const int r = blockIdx.x, tid = threadIdx.x, lane = tid & 31;
  const int nt = (int)blockDim.x;
  NucPlan* P = A.plan + r;
  if (tid < 4) A.list_cnt[4 * r + tid] = 0;
  const bool counts = A.h_cnt != nullptr;  // only rank selection needs element counts
  if (*((volatile int32_t*)A.status) == A.epoch) {  // a wait of this call ran out
    if (tid == 0) {
      A.out_ids[r] = -1;
      if (A.d_row_flags) A.d_row_flags[r] = MS_ROW_TIMEOUT;
      P->flags = kPlanDone;
    }
    return;
  }
  const ChunkStat* st = A.stats + (int64_t)r * A.n_chunks;
  row_stats(A, r, F);
  if (F.nan_row) {
    if (tid == 0) {
      nuc_nan_out(A, r, F.Mp);
      P->flags = kPlanDone;
    }
    return;
  }
  const float M = F.M, Mp = F.Mp;
  // ---- exact softmax sum: the fast sum corrected by the gathered candidates'
  // exact terms (src/generation.js:13-14)
  gather_cands(A, r, F);
  {
    const int nfc = min(F.nf, kGathMax);
    long long corr = 0;
    for (int j = tid; j < nfc; j += nt) {
      const Cand cd = F.gath[j];
      const int c = cd.i / kChunk;
      const float mc = c < kFinChunks ? F.cm[c] : __ldcg(&st[c].m);
      const float zc = c < kFinChunks ? F.cz[c] : __ldcg(&st[c].zref);
      const double sc = c < kFinChunks ? F.cs[c] : chunk_scale(A, mc, zc, Mp);
      const float e = term_exact(temper_fast(cd.x, A.T, A.rT, A.temper), Mp);
      corr += __double2ll_rn(((double)e - (double)chunk_term(A, cd.x, mc, zc) * sc) * 1125899906842624.0);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) corr += __shfl_xor_sync(kAll, corr, o);
    if (lane == 0 && corr != 0) atomicAdd(&F.corr, (unsigned long long)corr);
  }
  __syncthreads();
  const double S = F.S_fast + (double)(long long)F.corr * (1.0 / 1125899906842624.0);
  const double rS = 1.0 / S;

  // ---- the row's top bin, then the chunk histograms on the row's bins
  int bmin = INT_MAX;
  for (int c = tid; c < A.n_chunks; c += nt) {
    const int bi = __ldcg(&st[c].best_i);
    if (c < kFinChunks) N.ctop[c] = bi;
    if (__ldcg(&st[c].m) != -INFINITY) bmin = min(bmin, bi);
  }
  bmin = __reduce_min_sync(kAll, bmin);
  if (lane == 0) N.red_i[tid >> 5] = bmin;
  __syncthreads();
  int b_row = INT_MAX;
  for (int w = 0; w < (nt >> 5); w++) b_row = min(b_row, N.red_i[w]);
  __syncthreads();
  long long cnt = 0, tcnt = 0;
  double mass = 0.0, tmass = 0.0;
  const int t = tid;  // this thread's row bin, and the chunk bin it moves to the tail
  // chunk tops come from shared memory, so the loads of several chunks'
  // histogram words can be in flight at once
#pragma unroll 4
  for (int c = 0; c < A.n_chunks; c++) {
    const float mc = c < kFinChunks ? F.cm[c] : __ldcg(&st[c].m);
    const int64_t hb = ((int64_t)r * A.n_chunks + c) * kNB;
    if (mc == -INFINITY) {  // a chunk of -inf: every element in the tail, mass 0
      if (counts) tcnt += __ldcg(A.h_cnt + hb + t);
      continue;
    }
    const float zc = c < kFinChunks ? F.cz[c] : __ldcg(&st[c].zref);
    const double sc = (c < kFinChunks ? F.cs[c] : chunk_scale(A, mc, zc, Mp)) * rS;
    const long long shift = (long long)(c < kFinChunks ? N.ctop[c] : __ldcg(&st[c].best_i)) - (long long)b_row;
    const long long lb = (long long)t - shift;
    if (t < kNB - 1 && lb >= 0 && lb < kNB - 1) {
      if (counts) cnt += __ldcg(A.h_cnt + hb + lb);
      mass += __ldcg(A.h_mass + hb + lb) * sc;
    }
    if (t == kNB - 1 || (long long)t + shift >= kNB - 1) {
      if (counts) tcnt += __ldcg(A.h_cnt + hb + t);
      tmass += __ldcg(A.h_mass + hb + t) * sc;
    }
  }
  // the tail bin takes every thread's tail part
  tcnt = block_incl_scan<long long>(tcnt, N.red_c);
  tmass = block_incl_scan<double>(tmass, N.red_d);
  if (t == nt - 1) { N.red_c[0] = tcnt; N.red_d[0] = tmass; }
  __syncthreads();
  if (t == kNB - 1) { cnt += N.red_c[0]; mass += N.red_d[0]; }
  __syncthreads();
  N.ccnt[t] = block_incl_scan<long long>(cnt, N.red_c);
  N.cmass[t] = block_incl_scan<double>(mass, N.red_d);
  __syncthreads();

  // ---- the bin ranges of the cut and of the draw
  if (tid == 0) {
    NucPlan pl;
    memset(&pl, 0, sizeof pl);
    pl.b_row = b_row;
    pl.S = S;
    pl.M = M;
    pl.Mp = Mp;
    const double mtot = N.cmass[kNB - 1];
    pl.mass_tot = mtot;
    // the histogram's fast masses are within ~1e-6 of exact ones (per-bin
    // fixed point with 2^-18 resolution per element); the bounds use a wider margin
    const double eps = 1e-5 * mtot + 1e-30;
    const bool use_k = A.k > 0 && A.k < A.V;
    const bool use_p = A.use_topp != 0;
    // a chunk histogram whose bin wrapped (mass NaN) cannot place the targets
    int flags = (mtot == mtot) ? 0 : kPlanFallback;
    int c_lo = kNB, c_hi = kNB;  // kNB: no cut
    if (use_k) c_lo = c_hi = first_cnt_ge(N.ccnt, A.k);
    if (use_p) {
      if (A.top_p < 0.0) {  // the first candidate already reaches it; row bin 0 holds it
        c_lo = c_hi = 0;
      } else {
        const int pl_ = first_mass_ge(N.cmass, A.top_p - eps);
        const int ph_ = first_mass_ge(N.cmass, A.top_p + eps);
        if (pl_ < kNB) {
          if (ph_ >= kNB) flags = kPlanFallback;  // top_p too close to the total mass
          c_lo = min(c_lo, pl_);
          c_hi = min(c_hi, ph_);
        }
      }
    }
    const int first_ne = 0;  // row bin 0 holds the row max
    double t_lo, t_hi;
    int nr = 0;
    if (c_lo < kNB) {
      c_lo = max(c_lo, first_ne);
      c_hi = max(c_hi, c_lo);
      pl.lo[0] = c_lo;
      pl.hi[0] = c_hi;
      pl.cut_rg = 0;
      nr = 1;
      t_lo = c_lo > 0 ? N.cmass[c_lo - 1] : 0.0;
      t_hi = N.cmass[c_hi];
    } else {
      pl.cut_rg = -1;
      t_lo = t_hi = mtot;
    }
    // the draw: r = u * total, total between the mass above the cut range and
    // the mass through it; never past the cut
    const double u = A.u ? A.u[r] : 0.0;
    int d_lo, d_hi;
    if (!(u * t_hi > 0.0)) {
      d_lo = d_hi = first_ne;  // r <= 0 draws the first candidate
    } else {
      d_lo = max(first_mass_ge(N.cmass, u * t_lo - eps), first_ne);
      d_hi = first_mass_ge(N.cmass, u * t_hi + eps);
      if (d_hi >= kNB) d_hi = kNB - 1;
      if (nr) d_hi = min(d_hi, c_hi);
      d_lo = min(d_lo, d_hi);
    }
    if (nr && d_hi >= c_lo - 1) {  // touches the cut range: one range for both
      pl.lo[0] = min(c_lo, d_lo);
      pl.hi[0] = max(c_hi, d_hi);
      pl.draw_rg = 0;
    } else {
      pl.lo[nr] = d_lo;
      pl.hi[nr] = d_hi;
      pl.draw_rg = nr;
      nr++;
    }
    pl.nr = nr;
    for (int k = 0; k < nr; k++) {
      // without counts the extraction counts the elements above each range
      pl.cnt_above[k] = (counts && pl.lo[k] > 0) ? N.ccnt[pl.lo[k] - 1] : 0;
      pl.mass_above[k] = pl.lo[k] > 0 ? N.cmass[pl.lo[k] - 1] : 0.0;
      if (counts && N.ccnt[pl.hi[k]] - pl.cnt_above[k] > kListCap) flags = kPlanFallback;
      // the extraction tests bins as float bounds, exact below 2^24
      if (fabs((double)b_row + pl.lo[k]) >= 16777216.0 || fabs((double)b_row + pl.hi[k] + 1.0) >= 16777216.0)
        flags = kPlanFallback;
    }
    pl.flags = flags;
    *P = pl;
    if (A.d_row_max) A.d_row_max[r] = (double)Mp;
    if (A.d_row_sum) A.d_row_sum[r] = S;
  }
}

// =============================================================== extract
// The chunk grid in reverse order (the last chunks streamed are first, while
// they are still in L2): every element of the chunk whose row bin lies in one
// of its row's plan ranges goes to that range's list, and the elements above
// each range are counted.  The chunk comes into shared memory by bulk copies,
// as in sample_kernel.  A bin range [b1, b2] is the float interval
// b1 <= -x * a16 < b2 + 1 of the same product nuc_bin floors (exact: the bounds
// are integers below 2^24), so the test is two compares.
template <bool PEN>
__global__ void __launch_bounds__(kThreads, 3) nucleus_extract_kernel(const __grid_constant__ Args A) {
  extern __shared__ __align__(128) unsigned char ext_smem[];
  float* tile = reinterpret_cast<float*>(ext_smem);
  __shared__ __align__(8) uint64_t bar[kSub];
  __shared__ uint32_t penmask[kChunk / 32];
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the plans
  const int r = A.B - 1 - (int)blockIdx.x, c = A.n_chunks - 1 - (int)blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31;
  const NucPlan* P = A.plan + r;
  if (__ldcg(&P->flags)) return;
  const int nr = __ldcg(&P->nr), b_row = __ldcg(&P->b_row);
  float flo[2], fhi[2];
#pragma unroll
  for (int k = 0; k < 2; k++) {
    const bool on = k < nr;
    const int lo = on ? __ldcg(&P->lo[k]) : 0, hi = on ? __ldcg(&P->hi[k]) : -1;
    flo[k] = on ? (float)(b_row + lo) : INFINITY;
    fhi[k] = !on ? -INFINITY : (hi >= kNB - 1 ? INFINITY : (float)(b_row + hi + 1));
  }
  const float a16 = __fmul_rn(A.a, 16.f);
  // every element of the chunk lies at or below its top bin: nothing to do
  // when that is below every range
  if ((float)__ldcg(&A.stats[(int64_t)r * A.n_chunks + c].best_i) >= fmaxf(fhi[0], fhi[1])) return;
  const int c0 = c * kChunk;
  const int n = min(kChunk, A.V - c0);
  const float* g = A.logits + (int64_t)r * A.ld + c0;
  const bool bulk = ((reinterpret_cast<uintptr_t>(g) & 15) == 0) && ((n & 3) == 0);
  if (tid == 0 && bulk) {
    for (int s = 0; s < kSub; s++) mbar_init(&bar[s], 1);
    fence_mbar_init();
  }
  if (PEN) penmask[tid] = 0u;  // kChunk / 32 == kThreads words
  __syncthreads();
  if (bulk) {
    if (tid == 0)
      for (int s = 0; s < kSub; s++) {
        const int b = s * kSubElems, cnt = min(kSubElems, n - b);
        if (cnt > 0) {
          mbar_expect_tx(&bar[s], (uint32_t)cnt * 4u);
          bulk_g2s(tile + b, g + b, (uint32_t)cnt * 4u, &bar[s]);
        }
      }
  } else {
    for (int j = tid; j < n; j += kThreads) tile[j] = __ldg(g + j);
  }
  for (int j = n + tid; j < kChunk; j += kThreads) tile[j] = __int_as_float(0x7fc00000);  // padding fails every test
  if (PEN) pen_bitmap<kThreads>(A, r, c0, n, penmask);  // the chunk's penalty bitmap while the copies fly
  int timed_out = 0;
  if (bulk && tid == 0)
    for (int s = 0; s < kSub; s++)
      if (s * kSubElems < n && !mbar_wait(&bar[s], 0, kWaitCycles)) timed_out = 1;
  if (__syncthreads_or(timed_out)) {
    // the call fails (status word = this call's epoch; the resolve kernel
    // reports -1); let any copy still in flight land (bounded) and stop
    if (tid == 0) {
      atomicExch(A.status, A.epoch);
      for (int s = 0; s < kSub; s++)
        if (s * kSubElems < n) mbar_wait(&bar[s], 0, kWaitCycles);
    }
    __syncthreads();
    return;
  }
  // phase 1: which of this thread's elements fall in each range (bit 4i + l:
  // element l of its float4 i), and how many lie above each range
  const float4* t4 = reinterpret_cast<const float4*>(tile);
  constexpr int kIt = kChunk / 4 / kThreads;  // 8 float4 per thread
  static_assert(4 * kIt <= 32, "hit bits fit one word");
  auto pen_x = [&](float x, int j) {
    return (PEN && ((penmask[j >> 5] >> (j & 31)) & 1u)) ? pen_apply_fast(x, A.pen, A.rpen) : x;
  };
  uint32_t m0 = 0, m1 = 0;
  int above0 = 0, above1 = 0;
  const bool two = nr > 1;
#pragma unroll
  for (int i = 0; i < kIt; i++) {
    const int q = tid + i * kThreads;
    const float4 v = t4[q];
    const float xs[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int l = 0; l < 4; l++) {
      const float w = __fmul_rn(-pen_x(xs[l], 4 * q + l), a16);  // NaN (padding, a NaN row) fails every test
      const bool ge0 = w >= flo[0];
      m0 |= (uint32_t)(ge0 && w < fhi[0]) << (4 * i + l);
      above0 += w < flo[0];
      if (two) {
        m1 |= (uint32_t)(w >= flo[1] && w < fhi[1]) << (4 * i + l);
        above1 += w < flo[1];
      }
    }
  }
  // phase 2: one slot allocation per list per CTA, then each thread writes its hits
  __shared__ int sbase[2];
  const int packed = __popc(m0) | (__popc(m1) << 16);  // at most 32 each: no carry between halves
  int incl = packed;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(kAll, incl, o);
    if (lane >= o) incl += t;
  }
  __shared__ int wtot[kThreads / 32];
  if (lane == 31) wtot[tid >> 5] = incl;
  __syncthreads();
  if (tid < 32) {
    int v = tid < kThreads / 32 ? wtot[tid] : 0;
    int vi = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(kAll, vi, o);
      if (tid >= o) vi += t;
    }
    if (tid < kThreads / 32) wtot[tid] = vi - v;  // exclusive over warps
    if (tid == 31) {
      const int t0 = vi & 0xFFFF, t1 = vi >> 16;
      sbase[0] = t0 ? atomicAdd(&A.list_cnt[4 * r], t0) : 0;
      sbase[1] = t1 ? atomicAdd(&A.list_cnt[4 * r + 1], t1) : 0;
    }
  }
  __syncthreads();
  const int excl = wtot[tid >> 5] + incl - packed;
  int b0 = sbase[0] + (excl & 0xFFFF), b1 = sbase[1] + (excl >> 16);
  Cand* out0 = A.lists + (int64_t)(2 * r) * kListCap;
  Cand* out1 = out0 + kListCap;
  for (uint32_t mm = m0; mm; mm &= mm - 1u) {
    const int bit = __ffs(mm) - 1, j = 4 * (tid + (bit >> 2) * kThreads) + (bit & 3);
    if (b0 < kListCap) out0[b0] = Cand{pen_x(tile[j], j), c0 + j};
    b0++;
  }
  for (uint32_t mm = m1; mm; mm &= mm - 1u) {
    const int bit = __ffs(mm) - 1, j = 4 * (tid + (bit >> 2) * kThreads) + (bit & 3);
    if (b1 < kListCap) out1[b1] = Cand{pen_x(tile[j], j), c0 + j};
    b1++;
  }
  above0 = __reduce_add_sync(kAll, above0);
  above1 = __reduce_add_sync(kAll, above1);
  if (lane == 0) {
    if (above0) atomicAdd(&A.list_cnt[4 * r + 2], above0);
    if (above1) atomicAdd(&A.list_cnt[4 * r + 3], above1);
  }
}

// =============================================================== resolve
constexpr int kListCache = 4096;  // extracted elements a resolve CTA keeps in shared memory

struct ResSmem {
  Cand cache[kListCache];              // the range's elements, when they fit
  int scnt[kNSB];                      // sub-bin counts
  uint32_t smlo[kNSB], smhi[kNSB];     // sub-bin fast masses, 2^-60 units
  unsigned long long key[kExtCap];     // the crossing sub-bin's (prob desc, id asc) keys
  long long red_c[32];
  double red_d[32];
  uint32_t kmin, kmax;
  int sel, n_key, found;
  long long gt_c;
  uint32_t gt_lo, gt_hi;
  float tl, th;
  long long rank_before;
  double mass_before;
  int out_id;
  long long out_rank;
  double out_cum;
};
constexpr double kTwo60 = 1152921504606846976.0;

// A mass in units of 2^-60 (truncated), added to a two-word shared counter.
__device__ __forceinline__ unsigned long long mass60(double mass) { return (unsigned long long)(mass * kTwo60); }
__device__ __forceinline__ void add_u60(uint32_t* lo, uint32_t* hi, unsigned long long u) {
  const uint32_t l = (uint32_t)u, h = (uint32_t)(u >> 32);
  const uint32_t old = atomicAdd(lo, l);
  const uint32_t up = h + ((old + l < old) ? 1u : 0u);
  if (up) atomicAdd(hi, up);
}
__device__ __forceinline__ void add_mass60(uint32_t* lo, uint32_t* hi, double mass) { add_u60(lo, hi, mass60(mass)); }

// In one extracted range (m elements; cnt_above / mass_above the elements and
// fast probability mass of the row above it), the first element in
// (prob desc, id asc) order where rank >= rank_target or the running mass
// >= mass_target (either may be disabled: rank_target <= 0, mass_target NaN).
// Sub-bins of the range's logits (fast masses) find the crossing sub-bin; it
// is widened to whole probability-tie groups, whose elements alone get exact
// probabilities and keys; the mass above them stays fast, as in full_path.
// The range covers -x * a16 in [wlo, whi): a tie group reaching past it holds
// elements that were not extracted, and the row is not settled here.
// One CTA; false when the range or the sub-bin cannot settle it.
__device__ bool select_in_list(const Args& A, const RowInfo& Ri, const Cand* L, int m, float wlo, float whi,
                               long long cnt_above, double mass_above, long long rank_target, double mass_target,
                               ResSmem& R, int* id, long long* rank, double* cum) {
  const int tid = threadIdx.x, nt = (int)blockDim.x, warp = tid >> 5;
  // a target reached before the range, or an empty range, is not settled here
  if (m <= 0 || (rank_target > 0 && cnt_above >= rank_target) || (mass_target == mass_target && mass_above >= mass_target))
    return false;
  auto reached = [&](long long c, double mm) {
    return (rank_target > 0 && c >= rank_target) || (mass_target == mass_target && mm >= mass_target);
  };
  const bool cached = m <= kListCache;  // the first pass copies the range into shared memory
  auto gload = [&](int j) {
    const float2 cv = __ldcg(reinterpret_cast<const float2*>(L + j));
    return Cand{cv.x, __float_as_int(cv.y)};
  };
  auto load = [&](int j) { return cached ? R.cache[j] : gload(j); };
  if (tid == 0) {
    R.kmin = 0xFFFFFFFFu; R.kmax = 0u; R.found = 0; R.n_key = 0; R.sel = kNSB;
    R.gt_c = 0; R.gt_lo = 0u; R.gt_hi = 0u;
  }
  for (int b = tid; b < kNSB; b += nt) { R.scnt[b] = 0; R.smlo[b] = 0u; R.smhi[b] = 0u; }
  __syncthreads();
  uint32_t kmn = 0xFFFFFFFFu, kmx = 0u;
  for (int j = tid; j < m; j += nt) {
    const Cand cd = gload(j);
    if (cached) R.cache[j] = cd;
    const uint32_t k = fkey(cd.x);
    kmn = min(kmn, k);
    kmx = max(kmx, k);
  }
  kmn = __reduce_min_sync(kAll, kmn);
  kmx = __reduce_max_sync(kAll, kmx);
  if ((tid & 31) == 0) { atomicMin(&R.kmin, kmn); atomicMax(&R.kmax, kmx); }
  __syncthreads();
  const uint32_t kmax = R.kmax;
  const unsigned long long span = (unsigned long long)(kmax - R.kmin) + 1ull;
  auto sub = [&](uint32_t k) { return (int)(((unsigned long long)(kmax - k) * kNSB) / span); };  // 0: largest x
  for (int j = tid; j < m; j += nt) {
    const float x = load(j).x;
    const int b = sub(fkey(x));
    atomicAdd(&R.scnt[b], 1);
    add_mass60(&R.smlo[b], &R.smhi[b], mass_fast(Ri, x));
  }
  __syncthreads();
  // prefix over the sub-bins (two per thread: kNSB == 2 * blockDim.x)
  long long c2[2];
  double m2[2];
#pragma unroll
  for (int q = 0; q < 2; q++) {
    const int b = 2 * tid + q;
    c2[q] = R.scnt[b];
    m2[q] = ((double)R.smhi[b] * 4294967296.0 + (double)R.smlo[b]) * (1.0 / kTwo60);
  }
  const long long cs = block_incl_scan<long long>(c2[0] + c2[1], R.red_c);
  const double msum = block_incl_scan<double>(m2[0] + m2[1], R.red_d);
#pragma unroll
  for (int q = 0; q < 2; q++)
    if (reached(cnt_above + cs - (q == 0 ? c2[1] : 0), mass_above + msum - (q == 0 ? m2[1] : 0.0)))
      atomicMin(&R.sel, 2 * tid + q);
  __syncthreads();
  const int sel = R.sel;
  if (sel >= kNSB) return false;  // the targets lie beyond this range
  // the selected sub-bin's key interval, widened to whole probability-tie groups
  if (warp == 0) {
    const unsigned long long d0 = ((unsigned long long)sel * span + kNSB - 1) / kNSB;
    const unsigned long long d1 = ((unsigned long long)(sel + 1) * span + kNSB - 1) / kNSB - 1;
    const float xhi = fkey_inv((uint32_t)(kmax - d0)), xlo = fkey_inv((uint32_t)(kmax - d1));
    const float tl = tie_low(Ri, xlo), th = tie_high(Ri, xhi);
    if ((tid & 31) == 0) { R.tl = tl; R.th = th; }
  }
  __syncthreads();
  const float tl = R.tl, th = R.th;
  const float a16 = __fmul_rn(A.a, 16.f);
  if (!(__fmul_rn(-th, a16) >= wlo) || !(__fmul_rn(-tl, a16) < whi)) return false;
  // the elements above the tie groups: their count and fast mass, summed per
  // thread and per warp (the integer sum is the same in any order), one shared
  // add per warp
  long long gc = 0;
  unsigned long long gm = 0;
  for (int j = tid; j < m; j += nt) {
    const Cand cd = load(j);
    if (cd.x > th) {
      gc++;
      gm += mass60(mass_fast(Ri, cd.x));
    } else if (cd.x >= tl) {
      const int q = atomicAdd(&R.n_key, 1);
      if (q < kExtCap)
        R.key[q] = ((unsigned long long)(0xFFFFFFFFu - __float_as_uint(prob_of(Ri, cd.x))) << 32) | (uint32_t)cd.i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    gc += __shfl_xor_sync(kAll, gc, o);
    gm += __shfl_xor_sync(kAll, gm, o);
  }
  if ((tid & 31) == 0 && gc) atomicAdd(reinterpret_cast<unsigned long long*>(&R.gt_c), (unsigned long long)gc);
  if ((tid & 31) == 0 && gm) add_u60(&R.gt_lo, &R.gt_hi, gm);
  __syncthreads();
  const int nk = R.n_key;
  if (nk > kExtCap) return false;
  int np2 = 1;
  while (np2 < nk) np2 <<= 1;
  for (int j = nk + tid; j < np2; j += nt) R.key[j] = ~0ull;
  __syncthreads();
  for (int kk = 2; kk <= np2; kk <<= 1) {
    for (int jj = kk >> 1; jj > 0; jj >>= 1) {
      for (int i = tid; i < np2; i += nt) {
        const int ixj = i ^ jj;
        if (ixj > i) {
          const unsigned long long x = R.key[i], y = R.key[ixj];
          if ((x > y) == ((i & kk) == 0)) { R.key[i] = y; R.key[ixj] = x; }
        }
      }
      __syncthreads();
    }
  }
  if (tid == 0) {
    long long rk = cnt_above + R.gt_c;
    double acc = mass_above + ((double)R.gt_hi * 4294967296.0 + (double)R.gt_lo) * (1.0 / kTwo60);
    int hit = -1;
    for (int i = 0; i < nk; i++) {
      rk++;
      acc += (double)__uint_as_float(0xFFFFFFFFu - (uint32_t)(R.key[i] >> 32));
      if (reached(rk, acc)) {
        hit = i;
        break;
      }
    }
    R.found = hit >= 0;
    if (hit >= 0) {
      R.out_id = (int)(uint32_t)R.key[hit];
      R.out_rank = rk;
      R.out_cum = acc;
    }
  }
  __syncthreads();
  const bool ok = R.found != 0;
  if (ok) {
    *id = R.out_id;
    *rank = R.out_rank;
    *cum = R.out_cum;
  }
  __syncthreads();
  return ok;
}

// One CTA per row: the cut (rank top_k, running mass top_p) and the draw
// (running mass u * total) from the extracted ranges; the exact whole-row path
// for the rows the plan or the lists cannot settle.
__global__ void __launch_bounds__(kNB, 2) nucleus_resolve_kernel(const __grid_constant__ Args A) {
  extern __shared__ __align__(128) unsigned char nuc_smem[];
  ResSmem& R = *reinterpret_cast<ResSmem*>(nuc_smem);
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the lists
  const int r = blockIdx.x, tid = threadIdx.x, nt = (int)blockDim.x;
  const NucPlan pl = A.plan[r];
  if (pl.flags == kPlanDone) return;
  if (*((volatile int32_t*)A.status) == A.epoch) {  // a wait of this call ran out
    if (tid == 0) {
      A.out_ids[r] = -1;
      if (A.d_row_flags) A.d_row_flags[r] = MS_ROW_TIMEOUT;
    }
    return;
  }
  RowInfo Ri;
  Ri.row = A.logits + (int64_t)r * A.ld;
  Ri.V = A.V;
  Ri.pb = nullptr;
  Ri.pen = A.pen;
  Ri.rpen = A.rpen;
  Ri.M = pl.M;
  Ri.Mp = pl.Mp;
  Ri.S = pl.S;
  Ri.a = A.a;
  Ri.mscale = exp((double)pl.M * A.rT - (double)pl.Mp) / pl.S;
  Ri.T = A.T;
  Ri.temper = A.temper;
  Ri.nat16 = (float)(16.0 / A.T);
  Ri.rT = A.rT;
  Ri.rS = 1.0 / Ri.S;
  const bool use_k = A.k > 0 && A.k < A.V;
  bool ok = pl.flags == 0;
  int out_id = -1;
  long long n = use_k ? A.k : A.V;
  double total = pl.mass_tot;
  int last_id = -1;
  const bool counts = A.h_cnt != nullptr;
  // a list that overflowed cannot settle the row; without histogram counts the
  // extraction counted the elements above each range
  for (int k = 0; k < pl.nr; k++)
    if (__ldcg(&A.list_cnt[4 * r + k]) > kListCap) ok = false;
  long long above[2];
  float wlo[2], whi[2];  // each range as the interval of -x * a16 it covers
  for (int k = 0; k < 2; k++) {
    above[k] = counts ? pl.cnt_above[k] : (long long)__ldcg(&A.list_cnt[4 * r + 2 + k]);
    wlo[k] = (float)(pl.b_row + pl.lo[k]);
    whi[k] = pl.hi[k] >= kNB - 1 ? INFINITY : (float)(pl.b_row + pl.hi[k] + 1);
  }
  if (ok && pl.cut_rg >= 0) {
    const int k = pl.cut_rg;
    const int m = min(__ldcg(&A.list_cnt[4 * r + k]), kListCap);
    const double mt = (A.use_topp && A.top_p >= 0.0) ? A.top_p : __longlong_as_double(0x7ff8000000000000ll);
    const long long rt = A.use_topp && A.top_p < 0.0 ? 1 : (use_k ? (long long)A.k : 0);
    int id;
    long long rk;
    double cum;
    ok = select_in_list(A, Ri, A.lists + (int64_t)(2 * r + k) * kListCap, m, wlo[k], whi[k], above[k], pl.mass_above[k], rt, mt,
                        R, &id, &rk, &cum);
    if (ok) {
      n = rk;
      total = cum;
      last_id = id;
    }
  }
  if (ok) {
    const double u = A.u ? A.u[r] : 0.0;
    const double rr = u * total;
    const int k = pl.draw_rg;
    const int m = min(__ldcg(&A.list_cnt[4 * r + k]), kListCap);
    int id;
    long long rk;
    double cum;
    if (rr <= 0.0 || rr != rr)
      ok = rr == rr && select_in_list(A, Ri, A.lists + (int64_t)(2 * r + k) * kListCap, m, wlo[k], whi[k], above[k],
                                      pl.mass_above[k], 1, __longlong_as_double(0x7ff8000000000000ll), R, &id, &rk,
                                      &cum);
    else
      ok = select_in_list(A, Ri, A.lists + (int64_t)(2 * r + k) * kListCap, m, wlo[k], whi[k], above[k], pl.mass_above[k], 0, rr, R,
                          &id, &rk, &cum);
    if (ok) {
      if (rk > n) {  // past the cut: the reference's loop ends on the last candidate
        ok = last_id >= 0;
        id = last_id;
      }
      out_id = id;
    }
  }
  const bool diag_cands = (A.d_cand_ids || A.d_cand_probs) && A.cand_cap > 0;
  if ((!ok || diag_cands) && A.use_pen && A.penbits) {  // the exact path reads penalised values through a bitmap
    const int W = (A.V + 31) >> 5;
    uint32_t* pb = A.penbits + (int64_t)r * W;
    for (int w = tid; w < W; w += nt) pb[w] = 0u;
    __syncthreads();
    const int64_t h0 = A.hist_off[r], h1 = A.hist_off[r + 1];
    for (int64_t h = h0 + tid; h < h1; h += nt) {
      const int id = A.hist[h];
      if (id >= 0 && id < A.V) atomicOr(&pb[id >> 5], 1u << (id & 31));
    }
    __threadfence_block();
    __syncthreads();
    Ri.pb = pb;
  }
  __syncthreads();
  FullSmem& FS = *reinterpret_cast<FullSmem*>(nuc_smem);
  if (!ok) {
    full_path(A, r, Ri, FS, MS_ROW_SLOWPATH);  // writes the id, n_cand, total, flags and the candidates
    return;
  }
  if (tid == 0) {
    A.out_ids[r] = out_id;
    if (A.d_n_cand) A.d_n_cand[r] = (int32_t)n;
    if (A.d_total) A.d_total[r] = total;
    if (A.d_row_flags) A.d_row_flags[r] = MS_ROW_FULLVOCAB;
  }
  if (diag_cands) {
    block_hist(Ri, FS.h0, [](float) { return true; }, [&](float x) { return bin0(Ri, x); });
    full_emit_cands(A, r, Ri, FS, n);
  }
}

}  // namespace ms
