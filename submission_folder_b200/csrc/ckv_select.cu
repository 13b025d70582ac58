// Score finishing, smoothing, rank combination and keep-set selection of the
// CircuitKV prefill path (reference pyramidkv_utils.py):
//   finished scores  PU:2186-2204 (sinks = 1% of the total, divided by the max)
//   smoothing        PU:1884-1937, PU:3131-3160 (zero-padded conv1d)
//   ranks + MAX      PU:1865-1882, PU:3177-3196
//   keep mask        PU:2591-2644;  union keep mask PU:2489-2589
//   compaction       PU:3496-3501 (kept prefix positions in ascending order)
//
// One CTA of 1024 threads per layer.  Ranks are needed only near the top: the
// kept set of MAX(rank a, rank b) over candidates is contained in the union of
// the top-M of a and of b (M = kept + forced), so each vector is reduced to its
// top-M by a 4-pass radix select, the M survivors are bitonic-sorted and get
// ranks n-1, n-2, ...; the threshold of the combined rank is then found with a
// histogram over M bins.  Tie rules follow the reference on CUDA tensors: equal
// scores rank by index (stable argsort), equal combined scores at the k-th value
// are taken lowest index first (topk).
#include <string.h>

#include <mutex>

#include "ckv_common.cuh"
#include "ckv_select.h"

namespace ckv {

constexpr int kSelThreads = 1024;
constexpr int kMaxSort = 8192;   // largest top-M list sorted in shared memory

struct SelShared {
  unsigned long long sortbuf[kMaxSort];
  int hist[256];
  int scan[64];
  int misc[16];
  float fscratch[64];
};

// ---------------------------------------------------------------------------
// helpers
// ---------------------------------------------------------------------------
// Which positions a top-M selection may draw from.
struct Range {
  int n;        // positions [0, n)
  int lo, hi;   // when restricted: only [lo, hi) (the non-forced candidates)
  bool restricted;
  CKV_DEV bool ok(int i) const { return i < n && (!restricted || (i >= lo && i < hi)); }
};

// Radix select of the M largest keys among valid positions.  Returns the boundary
// key (*kstar), the count strictly above it (*above) and how many boundary-key
// elements complete the M (*take).
__device__ void radix_select(const float* v, const Range& rg, int M, SelShared& sh, uint32_t* kstar,
                             int* above, int* take) {
  uint32_t prefix = 0, pmask = 0;
  int remaining = M;
  int gt = 0;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = threadIdx.x; i < 256; i += blockDim.x) sh.hist[i] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < rg.n; i += blockDim.x) {
      if (!rg.ok(i)) continue;
      const uint32_t k = float_key(v[i]);
      if ((k & pmask) == prefix) atomicAdd(&sh.hist[(k >> shift) & 255], 1);
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      const int lane = threadIdx.x;
      // lane l owns digits [8*(31-l), 8*(31-l)+8): lane 0 the highest digits
      int loc[8], s = 0;
#pragma unroll
      for (int d = 0; d < 8; ++d) { loc[d] = sh.hist[8 * (31 - lane) + (7 - d)]; s += loc[d]; }
      int incl = s;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      const int excl = incl - s;
      const bool here = excl < remaining && incl >= remaining;
      const unsigned ball = __ballot_sync(0xffffffffu, here);
      const int owner = ball ? (__ffs(ball) - 1) : 31;
      if (lane == owner) {
        int cum = excl, digit = 8 * (31 - lane);
#pragma unroll
        for (int d = 0; d < 8; ++d) {
          if (cum + loc[d] >= remaining) { digit = 8 * (31 - lane) + (7 - d); break; }
          cum += loc[d];
        }
        sh.misc[0] = digit;
        sh.misc[1] = remaining - cum;   // still needed inside this digit
        sh.misc[2] = cum;               // above, inside the current prefix
      }
    }
    __syncthreads();
    const uint32_t digit = (uint32_t)sh.misc[0];
    gt += sh.misc[2];
    remaining = sh.misc[1];
    prefix |= digit << shift;
    pmask |= 0xFFu << shift;
    __syncthreads();
  }
  *kstar = prefix;
  *above = gt;
  *take = remaining;
}

// Collect the top-M (key, index) composites into sh.sortbuf[0..M) and sort them
// descending.  prefer_high: ties at the boundary keep the highest indices and
// rank higher index higher (stable ascending rank); otherwise lowest indices first.
__device__ void top_sorted(const float* v, const Range& rg, int M, bool prefer_high, SelShared& sh) {
  uint32_t kstar;
  int above, take;
  radix_select(v, rg, M, sh, &kstar, &above, &take);
  if (threadIdx.x == 0) { sh.misc[4] = 0; sh.misc[5] = 0; }
  __syncthreads();
  // strictly above the boundary
  for (int i = threadIdx.x; i < rg.n; i += blockDim.x) {
    if (!rg.ok(i)) continue;
    const uint32_t k = float_key(v[i]);
    if (k > kstar) {
      const int slot = atomicAdd(&sh.misc[4], 1);
      const uint32_t tie = prefer_high ? (uint32_t)i : ~(uint32_t)i;
      sh.sortbuf[slot] = ((unsigned long long)k << 32) | tie;
    }
  }
  // boundary ties: `take` of them, by index order (tiles of blockDim positions)
  const int ntiles = (rg.n + blockDim.x - 1) / blockDim.x;
  int taken = 0;
  for (int tt = 0; tt < ntiles && taken < take; ++tt) {
    const int t = prefer_high ? (ntiles - 1 - tt) : tt;
    const int i = prefer_high ? (t * (int)blockDim.x + (int)(blockDim.x - 1 - threadIdx.x))
                              : (t * (int)blockDim.x + (int)threadIdx.x);
    const bool is_tie = i >= 0 && rg.ok(i) && float_key(v[i]) == kstar;
    int tot;
    const int before = block_exclusive_scan(is_tie ? 1 : 0, sh.scan, &tot);
    if (is_tie && taken + before < take) {
      const int slot = above + taken + before;
      const uint32_t tie = prefer_high ? (uint32_t)i : ~(uint32_t)i;
      sh.sortbuf[slot] = ((unsigned long long)kstar << 32) | tie;
    }
    taken += tot;
  }
  __syncthreads();
  // bitonic sort (descending) of the next power of two >= M
  int P = 1;
  while (P < M) P <<= 1;
  for (int i = M + threadIdx.x; i < P; i += blockDim.x) sh.sortbuf[i] = 0ull;
  __syncthreads();
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < P; i += blockDim.x) {
        const int l = i ^ j;
        if (l > i) {
          const unsigned long long a = sh.sortbuf[i], b = sh.sortbuf[l];
          const bool desc = (i & k) == 0;
          if (desc ? (a < b) : (a > b)) { sh.sortbuf[i] = b; sh.sortbuf[l] = a; }
        }
      }
      __syncthreads();
    }
  }
}

CKV_DEV int sorted_index(unsigned long long e, bool prefer_high) {
  const uint32_t lo = (uint32_t)(e & 0xffffffffull);
  return (int)(prefer_high ? lo : ~lo);
}

// ---------------------------------------------------------------------------
// phase 0: finished scores from the sweep (PU:2186-2204)
// ---------------------------------------------------------------------------
__device__ int early_stop_steps(const Plan& pl, const char* ws, SelShared& sh) {
  const float* cmax = reinterpret_cast<const float*>(ws + pl.off_cmax);
  const float* ymax = reinterpret_cast<const float*>(ws + pl.off_ymax);
  int steps = pl.K;
  for (int k = 1; k <= pl.K; ++k) {
    bool all_small = true;
    for (int ch = 0; ch < pl.nchains; ++ch) {
      float m = 0.f;
      if (pl.n_p > pl.s)
        for (int c = threadIdx.x; c < pl.nscan; c += blockDim.x)
          m = fmaxf(m, __ldcg(cmax + ((size_t)ch * pl.nscan + c) * (kMaxIters + 1) + k));
      m = block_reduce<true>(m, sh.fscratch);
      m = fmaxf(m, __ldcg(ymax + ch * (pl.K + 1) + k));
      if (!(m < 1e-8f)) all_small = false;
    }
    if (all_small) { steps = k; break; }
  }
  return steps;
}

// Raw chain result at transient position j (sum of terms 0..steps).
CKV_DEV float raw_result(const Plan& pl, const char* ws, int ch, int j, int steps) {
  if (j < pl.n_p) {
    const float* cum = reinterpret_cast<const float*>(ws + pl.off_cum) + (size_t)ch * (pl.K + 1) * pl.n_p;
    return __ldcg(cum + (size_t)steps * pl.n_p + j);
  }
  const float* yk = reinterpret_cast<const float*>(ws + pl.off_yk) + (size_t)ch * (pl.K + 1) * pl.W;
  const int c = j - pl.n_p;
  float s = 0.f;
  for (int k = 0; k <= steps; ++k) s += __ldcg(yk + (size_t)k * pl.W + c);
  return s;
}

__device__ void finish_chain(const Plan& pl, const char* ws, int ch, int steps, float* out,
                             SelShared& sh) {
  const int n = pl.n, s = pl.s;
  float tot = 0.f, mx = 0.f;
  for (int j = s + threadIdx.x; j < n; j += blockDim.x) {
    const float v = raw_result(pl, ws, ch, j, steps);
    out[j] = v;
    tot += v;
  }
  tot = block_reduce<false>(tot, sh.fscratch);
  const float sinkv = tot * 0.01f;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const float v = (j < s) ? sinkv : out[j];
    mx = fmaxf(mx, v);
  }
  mx = block_reduce<true>(mx, sh.fscratch);
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    float v = (j < s) ? sinkv : out[j];
    if (mx > 0.f) v = v / mx;
    out[j] = v;
  }
  __syncthreads();
}

// Zero-padded conv1d (PU:1921-1936) from `in` to `out`; copies when k <= 1 or n <= k.
__device__ void smooth(const float* in, float* out, int n, int k, bool gaussian, float sigma) {
  if (k <= 1 || n <= k) {
    for (int j = threadIdx.x; j < n; j += blockDim.x) out[j] = in[j];
    __syncthreads();
    return;
  }
  float w[32];
  float wsum = 0.f;
  const int kk = min(k, 32);
  for (int t = 0; t < kk; ++t) {
    if (gaussian) {
      const float x = (float)t - (float)(k - 1) * 0.5f;
      w[t] = expf(-(x * x) / (2.f * sigma * sigma));
    } else {
      w[t] = 1.f / (float)k;
    }
    wsum += w[t];
  }
  if (gaussian)
    for (int t = 0; t < kk; ++t) w[t] = w[t] / wsum;
  const int pad = k / 2;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    float acc = 0.f;
    for (int t = 0; t < kk; ++t) {
      const int src = j + t - pad;
      if (src >= 0 && src < n) acc = fmaf(w[t], in[src], acc);
    }
    out[j] = acc;
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// phase 2: keep sets
// ---------------------------------------------------------------------------
// Marks kept candidate positions in `keep` (1 byte per position, pre-zeroed).
// Rank-MAX family: vectors vs[0..nv) with their ablation flags.
__device__ void select_rank_max(const Plan& pl, const float* const* vs, const bool* zeroed, int nv,
                                int* combR, uint8_t* keep, SelShared& sh, int32_t* status) {
  const int n = pl.n, kk = pl.kk;
  const int lo = pl.s, hi = pl.n - pl.W;   // candidates [s, n-W)
  if (kk <= 0) return;
  int live = 0;
  for (int v = 0; v < nv; ++v) live += zeroed[v] ? 0 : 1;
  if (live == 0) {
    // every combined score is 0: topk takes the lowest candidate indices
    for (int i = lo + threadIdx.x; i < lo + kk; i += blockDim.x) keep[i] = 1;
    __syncthreads();
    return;
  }
  const int M = min(n, kk + pl.s + pl.W);
  for (int i = threadIdx.x; i < n; i += blockDim.x) combR[i] = -1;
  __syncthreads();
  Range all{n, 0, n, false};
  for (int v = 0; v < nv; ++v) {
    if (zeroed[v]) continue;
    top_sorted(vs[v], all, M, true, sh);
    for (int p = threadIdx.x; p < M; p += blockDim.x) {
      const int idx = sorted_index(sh.sortbuf[p], true);
      atomicMax(&combR[idx], n - 1 - p);
    }
    __syncthreads();
  }
  // histogram of combined ranks >= n-M over the candidates
  int* hist = reinterpret_cast<int*>(sh.sortbuf);   // M ints
  for (int i = threadIdx.x; i < M; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const int r = __ldcg(combR + i);
    if (r >= n - M) atomicAdd(&hist[r - (n - M)], 1);
  }
  __syncthreads();
  {
    // threshold: thread t owns bins from the top, [M - (t+1)c, M - t c)
    const int c = (M + blockDim.x - 1) / blockDim.x;
    const int bhi = M - (int)threadIdx.x * c, blo = max(0, bhi - c);
    int local = 0;
    for (int b = blo; b < bhi; ++b) local += hist[b];
    int tot;
    const int above = block_exclusive_scan(local, sh.scan, &tot);
    if (threadIdx.x == 0) { sh.misc[8] = n; sh.misc[9] = 0; }
    __syncthreads();
    if (above < kk && above + local >= kk) {
      int cum = above;
      for (int b = bhi - 1; b >= blo; --b) {
        if (cum + hist[b] >= kk) { sh.misc[8] = (n - M) + b; sh.misc[9] = kk - cum; break; }
        cum += hist[b];
      }
    }
    __syncthreads();
    if (threadIdx.x == 0 && sh.misc[8] == n) set_status(status, kStatusCount);
  }
  const int t = sh.misc[8], need = sh.misc[9];
  // above the threshold: keep; at the threshold: the lowest `need` indices
  int taken = 0;
  for (int base = lo; base < hi; base += blockDim.x) {
    const int i = base + threadIdx.x;
    const int r = (i < hi) ? __ldcg(combR + i) : -1;
    if (r > t) keep[i] = 1;
    const bool tie = (r == t);
    int tot;
    const int before = block_exclusive_scan(tie ? 1 : 0, sh.scan, &tot);
    if (tie && taken + before < need) keep[i] = 1;
    taken += tot;
  }
  __syncthreads();
}

// Union keep set (PU:2489-2589).
__device__ void select_union(const Plan& pl, const ckv_params& prm, const float* qi, const float* hi,
                             uint8_t* keep, SelShared& sh) {
  const int n = pl.n;
  const int lo = pl.s, hiend = pl.n - pl.W;
  const int cand = hiend - lo;
  const int remaining = pl.kk;   // remaining budget (<= candidates already)
  if (remaining <= 0 || cand <= 0) return;
  const int qb = (int)((float)remaining * prm.qi_ratio);
  const int hb = remaining - qb;
  const int qk = min(qb, cand), hk = min(hb, cand);
  Range rg{n, lo, hiend, true};
  // QI top qk (lowest index among ties)
  if (qk > 0) {
    top_sorted(qi, rg, qk, false, sh);
    for (int p = threadIdx.x; p < qk; p += blockDim.x) keep[sorted_index(sh.sortbuf[p], false)] = 1;
    __syncthreads();
  }
  // HI extended list in topk order; the first hk always join, then fill
  const int ext = min(cand, hb + qb + max(0, remaining));   // upper bound on what the fill can use
  top_sorted(hi, rg, ext, false, sh);
  for (int p = threadIdx.x; p < hk; p += blockDim.x) keep[sorted_index(sh.sortbuf[p], false)] = 1;
  __syncthreads();
  // count the union
  int cnt = 0;
  for (int i = lo + threadIdx.x; i < hiend; i += blockDim.x) cnt += keep[i];
  cnt = (int)block_reduce<false>((float)cnt, sh.fscratch);
  if (cnt < remaining && threadIdx.x < 32) {
    // fill from the HI list in order, skipping members (one warp, 32 at a time)
    int have = cnt;
    for (int base = 0; base < ext && have < remaining; base += 32) {
      const int p = base + threadIdx.x;
      int idx = -1;
      bool add = false;
      if (p < ext) {
        idx = sorted_index(sh.sortbuf[p], false);
        add = keep[idx] == 0;
      }
      const unsigned ball = __ballot_sync(0xffffffffu, add);
      const int rank = __popc(ball & ((1u << threadIdx.x) - 1));
      if (add && have + rank < remaining) keep[idx] = 1;
      have += __popc(ball);
    }
  }
  __syncthreads();
}

// Kept prefix positions (sinks + chosen) in ascending order into out_idx.
__device__ int compact(const Plan& pl, const uint8_t* keep, int32_t* out_idx, SelShared& sh) {
  const int lim = pl.n - pl.W;
  const int cap = pl.s + pl.kk;   // out_idx capacity
  int written = 0;
  for (int base = 0; base < lim; base += blockDim.x) {
    const int i = base + threadIdx.x;
    const bool k = (i < lim) && (i < pl.s || keep[i]);
    int tot;
    const int before = block_exclusive_scan(k ? 1 : 0, sh.scan, &tot);
    if (k && written + before < cap) out_idx[written + before] = i;
    written += tot;
  }
  // a short selection (never expected) leaves valid positions behind: pad with the last sink
  for (int i = written + threadIdx.x; i < cap; i += blockDim.x) out_idx[i] = 0;
  __syncthreads();
  return written;
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kSelThreads) k_select(SelArgs a) {
  extern __shared__ __align__(16) char smraw[];
  SelShared& sh = *reinterpret_cast<SelShared*>(smraw);
  const Plan& pl = a.pl;
  const ckv_params& prm = a.p;
  char* ws = a.ws;
  Header* hdr = reinterpret_cast<Header*>(ws);
  const int n = pl.n;
  float* sc = reinterpret_cast<float*>(ws + pl.off_sel);            // [3][n] finished scores
  float* sm = sc + 3 * (size_t)n;                                   // [3][n] smoothed / weighted
  int* combR = reinterpret_cast<int*>(sm + 3 * (size_t)n);          // [n]
  uint8_t* keep = reinterpret_cast<uint8_t*>(combR + n);            // [n]

  // ---- phase 0: finished scores
  int steps = 0;
  if (a.given) {
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
      sc[j] = a.ga[j];
      sc[n + j] = a.gb ? a.gb[j] : 0.f;
      sc[2 * n + j] = a.gc ? a.gc[j] : 0.f;
    }
    __syncthreads();
  } else {
    steps = early_stop_steps(pl, ws, sh);
    for (int ch = 0; ch < pl.nchains; ++ch) finish_chain(pl, ws, ch, steps, sc + (size_t)ch * n, sh);
    if (threadIdx.x == 0) hdr->steps = steps;
  }
  if (a.finish_only) {
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
      a.out_scores[j] = sc[j];
      if (pl.nchains > 1) a.out_scores[n + j] = sc[n + j];
    }
    return;
  }
  for (int i = threadIdx.x; i < n; i += blockDim.x) keep[i] = 0;
  __syncthreads();

  const int mode = pl.mode;
  if (mode == CKV_COMB_DIS) {
    int qk = prm.qi_kernel_size != 0 ? prm.qi_kernel_size : prm.smoothing_kernel;
    const int hk = prm.hi_kernel_size != 0 ? prm.hi_kernel_size : prm.smoothing_kernel;
    if (prm.smooth_hi_only && qk > 1) qk = 0;
    const float qsig = prm.use_gaussian ? prm.gaussian_sigma * 0.5f : 1.0f;
    smooth(sc, sm, n, qk, prm.use_gaussian, qsig);
    smooth(sc + n, sm + n, n, hk, prm.use_gaussian, prm.gaussian_sigma);
    const bool bridge = prm.use_bridge_importance && (a.given ? a.gc != nullptr : true);
    if (bridge) smooth(sc + 2 * n, sm + 2 * n, n, prm.bi_kernel_size, prm.use_gaussian, prm.gaussian_sigma);
    if (a.out_scores)
      for (int j = threadIdx.x; j < n; j += blockDim.x) {
        a.out_scores[j] = sm[j];
        a.out_scores[n + j] = sm[n + j];
      }
    const float* vs[3] = {sm, sm + n, sm + 2 * n};
    const bool z[3] = {prm.ablate_qi != 0, prm.ablate_hi != 0, false};
    select_rank_max(pl, vs, z, bridge ? 3 : 2, combR, keep, sh, &hdr->status);
  } else if (mode == CKV_COMB_MAX) {
    // a = influence (chain 0), b = H2O column sums
    if (a.out_scores)
      for (int j = threadIdx.x; j < n; j += blockDim.x) {
        a.out_scores[j] = sc[j];
        a.out_scores[n + j] = sc[n + j];
      }
    const float* vs[2] = {sc, sc + n};
    const bool z[2] = {false, false};
    select_rank_max(pl, vs, z, 2, combR, keep, sh, &hdr->status);
  } else {   // union / union_da
    if (mode == CKV_COMB_UNION_DA && !a.given) {
      // DA = column sums of the QI window rows, clamped at 1e-8 (PU:3086-3091)
      const float* colsum = reinterpret_cast<const float*>(ws + pl.off_colsum);
      for (int j = threadIdx.x; j < n; j += blockDim.x) {
        const float da = fmaxf(colsum[j], 1e-8f);
        sc[j] = sc[j] * da;
        sc[n + j] = sc[n + j] * da;
      }
      __syncthreads();
    }
    if (a.out_scores)
      for (int j = threadIdx.x; j < n; j += blockDim.x) {
        a.out_scores[j] = sc[j];
        a.out_scores[n + j] = sc[n + j];
      }
    select_union(pl, prm, sc, sc + n, keep, sh);
  }
  __syncthreads();
  const int written = compact(pl, keep, a.out_idx, sh);
  if (threadIdx.x == 0) {
    hdr->kept = written;
    if (written != pl.s + pl.kk) set_status(&hdr->status, kStatusCount);
  }
}


// ---------------------------------------------------------------------------
// H2O column sums and bridge importance (one CTA)
// ---------------------------------------------------------------------------
// full_attn.sum(dim=0) (PU:3216) for pooled rows R:  colsum_R[j] + h[j] * E[j],
// E[j] = sum_{i=j+1}^{n_p-1} 1 / (C[i-1] + 1e-8), h = max(colsum_R, 1e-6), C = cumsum h.
// Bridge importance (PU:1510-1546) = A^T (A^T 1):
//   bi[j] = sum_r u[n_p + r] R[r, j] + h[j] * sum_{i=j+1}^{n_p-1} u[i] / (C[i-1] + 1e-8),  u = A^T 1.
__global__ void __launch_bounds__(kSelThreads) k_aux(const Plan pl, const ckv_params prm, char* ws) {
  __shared__ int iscan[64];
  __shared__ float fscan[64];
  const int n = pl.n, n_p = pl.n_p;
  const bool bridge = pl.mode == CKV_COMB_DIS && prm.use_bridge_importance;
  const int src = bridge ? (pl.hi_rows ? 1 : 0) : 0;
  const float* colsum = reinterpret_cast<const float*>(ws + pl.off_colsum) + (size_t)src * pl.n_pad;
  const float* rows = reinterpret_cast<const float*>(ws + (src ? pl.off_rows_hi : pl.off_rows_qi));
  float* sc = reinterpret_cast<float*>(ws + pl.off_sel);
  float* sm = sc + 3 * (size_t)n;
  float* inv = sm + 2 * (size_t)n;                       // temp [n]
  float* colA = bridge ? sm + (size_t)n : sc + (size_t)n; // full_attn column sums
  (void)iscan;
  // forward: C and inv
  float carry = 0.f;
  for (int base = 0; base < n_p; base += blockDim.x) {
    const int i = base + threadIdx.x;
    const float h = (i < n_p) ? fmaxf(colsum[i], 1e-6f) : 0.f;
    float tot;
    // exclusive prefix of h within the tile
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    float x = h;
    for (int o = 1; o < 32; o <<= 1) { const float y = __shfl_up_sync(0xffffffffu, x, o); if (lane >= o) x += y; }
    __syncthreads();
    if (lane == 31) fscan[wid] = x;
    __syncthreads();
    if (wid == 0) {
      float s = fscan[lane];
      for (int o = 1; o < 32; o <<= 1) { const float y = __shfl_up_sync(0xffffffffu, s, o); if (lane >= o) s += y; }
      fscan[lane] = s;
    }
    __syncthreads();
    const float excl = carry + ((wid > 0) ? fscan[wid - 1] : 0.f) + x - h;   // C[i-1]
    tot = fscan[31];
    if (i < n_p) inv[i] = (i >= 1) ? 1.0f / (excl + 1e-8f) : 0.f;
    carry += tot;
    __syncthreads();
  }
  // reverse: E and the column sums of full_attn
  for (int p = 0; p < 2; ++p) {
    if (p == 1 && !bridge) break;
    float rc = 0.f;
    const int ntile = (n_p + blockDim.x - 1) / blockDim.x;
    for (int tt = ntile - 1; tt >= 0; --tt) {
      const int i = tt * blockDim.x + threadIdx.x;
      // term summed: inv[i] (pass 0) or colA[i] * inv[i] (pass 1)
      const float v = (i < n_p) ? (p == 0 ? inv[i] : colA[i] * inv[i]) : 0.f;
      // inclusive suffix sum within the tile = total - exclusive prefix
      const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
      float x = v;
      for (int o = 1; o < 32; o <<= 1) { const float y = __shfl_up_sync(0xffffffffu, x, o); if (lane >= o) x += y; }
      __syncthreads();
      if (lane == 31) fscan[wid] = x;
      __syncthreads();
      if (wid == 0) {
        float s = fscan[lane];
        for (int o = 1; o < 32; o <<= 1) { const float y = __shfl_up_sync(0xffffffffu, s, o); if (lane >= o) s += y; }
        fscan[lane] = s;
      }
      __syncthreads();
      const float incl = ((wid > 0) ? fscan[wid - 1] : 0.f) + x;
      const float tot = fscan[31];
      const float after = rc + (tot - incl);    // sum over i' > i
      if (i < n_p) {
        const float h = fmaxf(colsum[i], 1e-6f);
        if (p == 0) colA[i] = colsum[i] + h * after;
        else sc[2 * (size_t)n + i] = h * after;
      }
      rc += tot;
      __syncthreads();
    }
    if (p == 0)
      for (int j = n_p + threadIdx.x; j < n; j += blockDim.x) colA[j] = colsum[j];
    __syncthreads();
  }
  if (bridge) {
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
      float s = 0.f;
      for (int r = 0; r < pl.W; ++r) s = fmaf(colA[n_p + r], rows[(size_t)r * pl.n_pad + j], s);
      sc[2 * (size_t)n + j] = (j < n_p ? sc[2 * (size_t)n + j] : 0.f) + s;
    }
  }
}

cudaError_t launch_aux(const Plan& pl, const ckv_params& p, char* ws, cudaStream_t st) {
  k_aux<<<1, kSelThreads, 0, st>>>(pl, p, ws);
  return cudaGetLastError();
}

size_t select_smem_bytes() { return sizeof(SelShared); }

cudaError_t launch_select(const SelArgs& a, cudaStream_t st) {
  static bool attr = false;
  if (!attr) {
    const cudaError_t e = cudaFuncSetAttribute(k_select, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)sizeof(SelShared));
    if (e != cudaSuccess) return e;
    attr = true;
  }
  k_select<<<1, kSelThreads, sizeof(SelShared), st>>>(a);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Selection with no workspace argument (ckv_select_scores_noalloc)
// ---------------------------------------------------------------------------
// Some callers cannot hand this library device memory: a serving engine that has
// reserved nearly all HBM for its KV-cache pool at start-up (a per-call cudaMalloc
// there either fails or fragments the pool, and cudaMalloc also synchronises the
// device), or plain-C / FFI callers that have no device allocator of their own.
// For them the selection stage keeps its scratch in this file-scope array: header
// (256 B) + the selection area (29 bytes per position) for up to 32768 positions,
// about 0.9 MiB that every GPU which loads the library holds until the process
// exits.  All calls share it and it keeps the last call's contents, so calls that
// overlap on the GPU (different streams, or different host threads on one device)
// race; order them on one stream.
constexpr int kNoAllocMaxN = 32768;
constexpr size_t kNoAllocBytes = 256 + (size_t)29 * kNoAllocMaxN;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

// Device address of g_noalloc_scratch per device, looked up once per device with
// that device current (the host-side symbol is only a stand-in, not a device address).
constexpr int kMaxDevices = 64;
static void* g_noalloc_addr[kMaxDevices] = {};
static std::mutex g_noalloc_mu;

static cudaError_t noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_noalloc_addr[dev] = ptr;
  }
  *out = g_noalloc_addr[dev];
  return cudaSuccess;
}

int select_scores_noalloc(const ckv_params* p, int32_t n, const float* a, const float* b,
                          const float* c, int32_t* out_idx, float* out_scores, cudaStream_t st,
                          const char** why) {
  if (!p || !a || !b || !out_idx) { *why = "null argument"; return CKV_ERR_ARG; }
  if (n > kNoAllocMaxN) {
    *why = "ckv_select_scores_noalloc: n exceeds the static scratch limit of 32768 positions";
    return CKV_ERR_ARG;
  }
  if (n < p->max_capacity_prompt) { *why = "n < max_capacity_prompt: nothing to select"; return CKV_ERR_ARG; }
  Plan pl;
  int rc = make_plan(*p, n, 32, 8, 128, CKV_BF16, &pl, why);
  if (rc) return rc;
  // only the header and the selection area are touched by the given-scores path
  pl.off_sel = 256;
  pl.total = 256 + pl.sel_bytes;
  if (pl.total > kNoAllocBytes) { *why = "selection scratch larger than the static array"; return CKV_ERR_ARG; }
  void* base = nullptr;
  cudaError_t e = noalloc_scratch(&base);
  if (e != cudaSuccess) { *why = cudaGetErrorString(e); return CKV_ERR_CUDA; }
  char* ws = static_cast<char*>(base);
  e = cudaMemsetAsync(ws, 0, sizeof(Header), st);   // status and counters start at zero
  if (e != cudaSuccess) { *why = cudaGetErrorString(e); return CKV_ERR_CUDA; }
  SelArgs sa;
  memset(&sa, 0, sizeof(sa));
  sa.pl = pl; sa.p = *p; sa.ws = ws; sa.out_idx = out_idx; sa.out_scores = out_scores;
  sa.given = 1; sa.ga = a; sa.gb = b; sa.gc = c;
  e = launch_select(sa, st);
  if (e != cudaSuccess) { *why = cudaGetErrorString(e); return CKV_ERR_CUDA; }
  return CKV_OK;
}

}  // namespace ckv
