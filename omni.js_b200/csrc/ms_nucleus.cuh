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
  for (int c = tid; c < A.n_chunks; c += nt)
    if (__ldcg(&st[c].m) != -INFINITY) bmin = min(bmin, __ldcg(&st[c].best_i));
  bmin = __reduce_min_sync(kAll, bmin);
  if (lane == 0) N.red_i[tid >> 5] = bmin;
  __syncthreads();
  int b_row = INT_MAX;
  for (int w = 0; w < (nt >> 5); w++) b_row = min(b_row, N.red_i[w]);
  __syncthreads();
  long long cnt = 0, tcnt = 0;
  double mass = 0.0, tmass = 0.0;
  const int t = tid;  // this thread's row bin, and the chunk bin it moves to the tail
  for (int c = 0; c < A.n_chunks; c++) {
    const float mc = c < kFinChunks ? F.cm[c] : __ldcg(&st[c].m);
    const int64_t hb = ((int64_t)r * A.n_chunks + c) * kNB;
    if (mc == -INFINITY) {  // a chunk of -inf: every element in the tail, mass 0
      if (counts) tcnt += __ldcg(A.h_cnt + hb + t);
      continue;
    }
    const float zc = c < kFinChunks ? F.cz[c] : __ldcg(&st[c].zref);
    const double sc = (c < kFinChunks ? F.cs[c] : chunk_scale(A, mc, zc, Mp)) * rS;
    const long long shift = (long long)__ldcg(&st[c].best_i) - (long long)b_row;
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
// each range are counted.  A bin range [b1, b2] is the float interval
// b1 <= -x * a16 < b2 + 1 of the same product nuc_bin floors (exact: the bounds
// are integers below 2^24), so the test is two compares.
template <bool PEN>
__global__ void __launch_bounds__(256) nucleus_extract_kernel(const __grid_constant__ Args A) {
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
  if (PEN) {
    for (int w = tid; w < kChunk / 32; w += blockDim.x) penmask[w] = 0u;
    __syncthreads();
    const int64_t h0 = A.hist_off[r], h1 = A.hist_off[r + 1];
    for (int64_t h = h0 + tid; h < h1; h += blockDim.x) {
      const uint32_t d = (uint32_t)__ldg(A.hist + h) - (uint32_t)c0;  // ids outside wrap past n
      if (d < (uint32_t)n) atomicOr(&penmask[d >> 5], 1u << (d & 31));
    }
    __syncthreads();
  }
  const float* g = A.logits + (int64_t)r * A.ld + c0;
  Cand* out0 = A.lists + (int64_t)(2 * r) * kListCap;
  Cand* out1 = out0 + kListCap;
  const bool vec = ((reinterpret_cast<uintptr_t>(g) & 15) == 0);
  const int step = 4 * (int)blockDim.x;
  const int rounds = (n + step - 1) / step;  // warp-uniform: every lane runs every round
  auto load4 = [&](int j0, float* xs) {
    if (vec && j0 + 3 < n) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(g + j0));
      xs[0] = v.x; xs[1] = v.y; xs[2] = v.z; xs[3] = v.w;
    } else {
#pragma unroll
      for (int l = 0; l < 4; l++) xs[l] = j0 + l < n ? __ldg(g + j0 + l) : __int_as_float(0x7fc00000);
    }
  };
  float cur[4], nxt[4];
  load4(4 * tid, cur);
  int above0 = 0, above1 = 0;
  for (int rd = 0; rd < rounds; rd++) {
    const int j0 = 4 * (rd * (int)blockDim.x + tid);
    if (rd + 1 < rounds) load4(j0 + step, nxt);  // next round in flight
    uint32_t in0 = 0, in1 = 0;
#pragma unroll
    for (int l = 0; l < 4; l++) {
      float x = cur[l];
      const int j = j0 + l;
      if (PEN && j < n && ((penmask[j >> 5] >> (j & 31)) & 1u)) {
        x = pen_apply_fast(x, A.pen, A.rpen);
        cur[l] = x;
      }
      const float w = __fmul_rn(-x, a16);  // NaN (padding, or a NaN row) fails every test
      in0 |= (uint32_t)(w >= flo[0] && w < fhi[0]) << l;
      in1 |= (uint32_t)(w >= flo[1] && w < fhi[1]) << l;
      above0 += w < flo[0];
      above1 += w < flo[1];
    }
    if (__any_sync(kAll, (in0 | in1) != 0)) {
      // slots for this round's elements: one atomic per list per warp
      const int c0n = __popc(in0), c1n = __popc(in1);
      int s0 = c0n, s1 = c1n;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t0 = __shfl_up_sync(kAll, s0, o), t1 = __shfl_up_sync(kAll, s1, o);
        if (lane >= o) { s0 += t0; s1 += t1; }
      }
      int b0 = 0, b1 = 0;
      if (lane == 31) {
        if (s0) b0 = atomicAdd(&A.list_cnt[4 * r], s0);
        if (s1) b1 = atomicAdd(&A.list_cnt[4 * r + 1], s1);
      }
      b0 = __shfl_sync(kAll, b0, 31) + s0 - c0n;
      b1 = __shfl_sync(kAll, b1, 31) + s1 - c1n;
#pragma unroll
      for (int l = 0; l < 4; l++) {
        if ((in0 >> l) & 1u) { if (b0 < kListCap) out0[b0] = Cand{cur[l], c0 + j0 + l}; b0++; }
        if ((in1 >> l) & 1u) { if (b1 < kListCap) out1[b1] = Cand{cur[l], c0 + j0 + l}; b1++; }
      }
    }
#pragma unroll
    for (int l = 0; l < 4; l++) cur[l] = nxt[l];
  }
  above0 = __reduce_add_sync(kAll, above0);
  above1 = __reduce_add_sync(kAll, above1);
  if (lane == 0) {
    if (above0) atomicAdd(&A.list_cnt[4 * r + 2], above0);
    if (above1) atomicAdd(&A.list_cnt[4 * r + 3], above1);
  }
}

// =============================================================== resolve
struct ResSmem {
  float prob[kListCap];                // exact probabilities of the list
  int scnt[kNSB];                      // sub-bin counts
  uint32_t smlo[kNSB], smhi[kNSB];     // sub-bin masses, 2^-60 units
  unsigned long long key[kExtCap];     // the crossing sub-bin's (prob desc, id asc) keys
  long long red_c[32];
  double red_d[32];
  uint32_t kmin, kmax;
  int sel, n_key, found;
  long long rank_before;
  double mass_before;
  int out_id;
  long long out_rank;
  double out_cum;
};
constexpr double kTwo60 = 1152921504606846976.0;

// In one extracted range (m elements, cnt_above / mass_above the elements and
// fast mass of the bins above it), the first element in (prob desc, id asc)
// order where rank >= rank_target or the running mass >= mass_target (either
// may be disabled: rank_target <= 0, mass_target NaN).  One CTA; returns false
// when the elements or the sub-bin cannot settle it.
__device__ bool select_in_list(const Args& A, const Cand* L, int m, long long cnt_above, double mass_above,
                               long long rank_target, double mass_target, float Mp, double S, ResSmem& R,
                               int* id, long long* rank, double* cum) {
  const int tid = threadIdx.x, nt = (int)blockDim.x;
  // a target reached before the range, or an empty range, is not settled here
  if (m <= 0 || (rank_target > 0 && cnt_above >= rank_target) || (mass_target == mass_target && mass_above >= mass_target))
    return false;
  if (tid == 0) { R.kmin = 0xFFFFFFFFu; R.kmax = 0u; R.found = 0; R.n_key = 0; R.sel = -1; }
  for (int b = tid; b < kNSB; b += nt) { R.scnt[b] = 0; R.smlo[b] = 0u; R.smhi[b] = 0u; }
  __syncthreads();
  uint32_t kmn = 0xFFFFFFFFu, kmx = 0u;
  for (int j = tid; j < m; j += nt) {
    const float2 cv = __ldcg(reinterpret_cast<const float2*>(L + j));
    const Cand cd{cv.x, __float_as_int(cv.y)};
    const float p = prob_exact(term_exact(temper_fast(cd.x, A.T, A.rT, A.temper), Mp), S);
    R.prob[j] = p;
    const uint32_t k = __float_as_uint(p);  // p >= 0: bits grow with p
    kmn = min(kmn, k);
    kmx = max(kmx, k);
  }
  kmn = __reduce_min_sync(kAll, kmn);
  kmx = __reduce_max_sync(kAll, kmx);
  if ((tid & 31) == 0) { atomicMin(&R.kmin, kmn); atomicMax(&R.kmax, kmx); }
  __syncthreads();
  const uint32_t kmin = R.kmin, kmax = R.kmax;
  const unsigned long long span = (unsigned long long)(kmax - kmin) + 1ull;
  auto sub = [&](float p) {  // sub-bin 0 holds the largest probabilities
    return (int)(((unsigned long long)(kmax - __float_as_uint(p)) * kNSB) / span);
  };
  for (int j = tid; j < m; j += nt) {
    const float p = R.prob[j];
    const int b = sub(p);
    atomicAdd(&R.scnt[b], 1);
    const unsigned long long u = (unsigned long long)((double)p * kTwo60);
    const uint32_t lo = (uint32_t)u, hi = (uint32_t)(u >> 32);
    const uint32_t old = atomicAdd(&R.smlo[b], lo);
    const uint32_t up = hi + ((old + lo < old) ? 1u : 0u);
    if (up) atomicAdd(&R.smhi[b], up);
  }
  __syncthreads();
  // prefix over the sub-bins (two per thread with kNB = 512 threads)
  long long c2[2];
  double m2[2];
#pragma unroll
  for (int q = 0; q < 2; q++) {
    const int b = 2 * tid + q;
    c2[q] = b < kNSB ? R.scnt[b] : 0;
    m2[q] = b < kNSB ? ((double)R.smhi[b] * 4294967296.0 + (double)R.smlo[b]) * (1.0 / kTwo60) : 0.0;
  }
  const long long cs = block_incl_scan<long long>(c2[0] + c2[1], R.red_c);
  const double msum = block_incl_scan<double>(m2[0] + m2[1], R.red_d);
  // the first sub-bin whose end reaches a target (it holds the element sought;
  // an empty one means the target lies before this range)
  if (tid == 0) R.sel = kNSB;
  __syncthreads();
  auto reached = [&](long long c, double mm) {
    return (rank_target > 0 && c >= rank_target) || (mass_target == mass_target && mm >= mass_target);
  };
#pragma unroll
  for (int q = 0; q < 2; q++) {
    const int b = 2 * tid + q;
    const long long cend = cnt_above + cs - (q == 0 ? c2[1] : 0);
    const double mend = mass_above + msum - (q == 0 ? m2[1] : 0.0);
    if (b < kNSB && reached(cend, mend)) atomicMin(&R.sel, b);
  }
  __syncthreads();
  const int sel = R.sel;
  if (sel >= kNSB) return false;  // the targets lie beyond this range
  if ((sel >> 1) == tid) {        // the totals before the selected sub-bin
    const int q = sel & 1;
    R.rank_before = cnt_above + cs - c2[1] - (q == 0 ? c2[0] : 0);
    R.mass_before = mass_above + msum - m2[1] - (q == 0 ? m2[0] : 0.0);
  }
  __syncthreads();
  // its elements, ranked exactly
  for (int j = tid; j < m; j += nt) {
    const float p = R.prob[j];
    if (sub(p) == sel) {
      const int q = atomicAdd(&R.n_key, 1);
      if (q < kExtCap)
        R.key[q] = ((unsigned long long)(0xFFFFFFFFu - __float_as_uint(p)) << 32) | (uint32_t)__ldcg(&L[j].i);
    }
  }
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
    long long rk = R.rank_before;
    double acc = R.mass_before;
    int hit = -1;
    for (int i = 0; i < nk; i++) {
      rk++;
      acc += (double)__uint_as_float(0xFFFFFFFFu - (uint32_t)(R.key[i] >> 32));
      if ((rank_target > 0 && rk >= rank_target) || (mass_target == mass_target && acc >= mass_target)) {
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
  for (int k = 0; k < 2; k++) above[k] = counts ? pl.cnt_above[k] : (long long)__ldcg(&A.list_cnt[4 * r + 2 + k]);
  if (ok && pl.cut_rg >= 0) {
    const int k = pl.cut_rg;
    const int m = min(__ldcg(&A.list_cnt[4 * r + k]), kListCap);
    const double mt = (A.use_topp && A.top_p >= 0.0) ? A.top_p : __longlong_as_double(0x7ff8000000000000ll);
    const long long rt = A.use_topp && A.top_p < 0.0 ? 1 : (use_k ? (long long)A.k : 0);
    int id;
    long long rk;
    double cum;
    ok = select_in_list(A, A.lists + (int64_t)(2 * r + k) * kListCap, m, above[k], pl.mass_above[k], rt, mt,
                        pl.Mp, pl.S, R, &id, &rk, &cum);
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
      ok = rr == rr && select_in_list(A, A.lists + (int64_t)(2 * r + k) * kListCap, m, above[k], pl.mass_above[k],
                                      1, __longlong_as_double(0x7ff8000000000000ll), pl.Mp, pl.S, R, &id, &rk,
                                      &cum);
    else
      ok = select_in_list(A, A.lists + (int64_t)(2 * r + k) * kListCap, m, above[k], pl.mass_above[k], 0, rr,
                          pl.Mp, pl.S, R, &id, &rk, &cum);
    if (ok) {
      if (rk > n) {  // past the cut: the reference's loop ends on the last candidate
        ok = last_id >= 0;
        id = last_id;
      }
      out_id = id;
    }
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
