// Score finishing, smoothing, rank combination and keep-set selection of the
// CircuitKV prefill path (reference pyramidkv_utils.py):
//   finished scores  PU:2186-2204 (sinks = 1% of the total, divided by the max)
//   smoothing        PU:1884-1937, PU:3131-3160 (zero-padded conv1d)
//   ranks + MAX      PU:1865-1882, PU:3177-3196
//   keep mask        PU:2591-2644;  union keep mask PU:2489-2589
//   compaction       PU:3496-3501 (kept prefix positions in ascending order)
//
// One thread-block cluster per layer, one CTA (1024 threads) per score vector
// (QI / HI [/ bridge], or influence / H2O).  Each CTA keeps its vector in shared
// memory (global scratch above 36864 positions), finishes and smooths it, and
// reduces it to its top-M by a 4-pass radix select (per-warp histograms) and a
// bitonic sort of the M survivors: ranks are needed only near the top, since the
// kept set of MAX(rank a, rank b) over the candidates lies in the union of the
// top-M of each vector (M = kept + forced).  CTA 0 reads the other CTAs' lists
// through distributed shared memory, builds the combined ranks, finds the
// threshold with a histogram over M bins and compacts the kept positions.
// Ordered passes (ties by index, compaction) count set predicates per 32-position
// chunk with a warp ballot and do one block scan over the chunk counts.  Tie rules
// follow the reference on CUDA tensors: equal scores rank by index (stable
// argsort); equal combined scores at the k-th value are taken lowest index first.
#include <cooperative_groups.h>
#include <string.h>

#include <mutex>

#include "ckv_common.cuh"
#include "ckv_select.h"

namespace cg = cooperative_groups;

namespace ckv {

constexpr int kSelThreads = 1024;
constexpr int kSelWarps = kSelThreads / 32;
constexpr int kMaxSort = 8192;         // largest top-M list sorted in shared memory
constexpr int kSmemScoresMax = 36864;  // vectors up to this length stay in shared memory

struct SelLayout {
  int n, nchunk;
  bool smem_scores;
  size_t off_x, off_sort, off_cnt_a, off_cnt_b, off_bits, off_misc, total;
};

__host__ __device__ inline SelLayout sel_layout(int n) {
  SelLayout L;
  L.n = n;
  L.nchunk = (n + 31) / 32;
  L.smem_scores = n <= kSmemScoresMax;
  size_t off = 0;
  auto take = [&](size_t b) { const size_t o = off; off = (off + b + 15) & ~(size_t)15; return o; };
  L.off_sort = take(sizeof(unsigned long long) * kMaxSort);   // also the per-warp histograms
  L.off_x = take(L.smem_scores ? sizeof(float) * (size_t)n : 0);
  L.off_cnt_a = take(sizeof(int) * (size_t)L.nchunk);
  L.off_cnt_b = take(sizeof(int) * (size_t)L.nchunk);
  L.off_bits = take(sizeof(uint32_t) * (size_t)L.nchunk);
  L.off_misc = take(sizeof(int) * 256);
  L.total = off;
  return L;
}

struct SelSmem {
  unsigned long long* sortbuf;
  int* hist;        // [kSelWarps][256] (aliases sortbuf)
  float* x;         // score vector (shared or global)
  int* cnt_a;
  int* cnt_b;
  uint32_t* bits;
  int* misc;        // [0..63] scan scratch, [64..] scalars
  float* fmisc;
};

// ---------------------------------------------------------------------------
// block helpers
// ---------------------------------------------------------------------------
CKV_DEV uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// In-place exclusive scan of cnt[0..m); returns the total.  All threads.
__device__ int scan_counts(int* cnt, int m, int* scratch) {
  const int per = (m + blockDim.x - 1) / blockDim.x;
  const int lo = threadIdx.x * per, hi = min(m, lo + per);
  int local = 0;
  for (int i = lo; i < hi; ++i) local += cnt[i];
  int total;
  int run = block_exclusive_scan(local, scratch, &total);
  for (int i = lo; i < hi; ++i) { const int c = cnt[i]; cnt[i] = run; run += c; }
  __syncthreads();
  return total;
}

// Ballot counts of pred(i) per 32-position chunk into cnt (index order).
template <class Pred>
__device__ void chunk_counts(int n, int* cnt, Pred pred) {
  const int lane = threadIdx.x & 31;
  for (int base = threadIdx.x - lane; base < n; base += blockDim.x) {
    const int i = base + lane;
    const unsigned b = __ballot_sync(0xffffffffu, i < n && pred(i));
    if (lane == 0) cnt[base >> 5] = __popc(b);
  }
  __syncthreads();
}

// Rank (in index order) of position i among those with pred true, given the scanned chunk counts.
CKV_DEV int chunk_rank(const int* cnt, int i, unsigned ball) {
  return cnt[i >> 5] + __popc(ball & lanemask_lt());
}

// ---------------------------------------------------------------------------
// top-M of one vector
// ---------------------------------------------------------------------------
struct Range {
  int n, lo, hi;
  bool restricted;
  CKV_DEV bool ok(int i) const { return i < n && (!restricted || (i >= lo && i < hi)); }
};

__device__ void radix_select(const float* v, const Range& rg, int M, SelSmem& sh, uint32_t* kstar,
                             int* above, int* take) {
  uint32_t prefix = 0, pmask = 0;
  int remaining = M, gt = 0;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  int* myhist = sh.hist + wid * 256;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = threadIdx.x; i < kSelWarps * 256; i += blockDim.x) sh.hist[i] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < rg.n; i += blockDim.x) {
      if (!rg.ok(i)) continue;
      const uint32_t k = float_key(v[i]);
      if ((k & pmask) == prefix) atomicAdd(&myhist[(k >> shift) & 255], 1);
    }
    __syncthreads();
    // fold the per-warp histograms into warp 0's row
    if (threadIdx.x < 256) {
      int s = 0;
      for (int w = 0; w < kSelWarps; ++w) s += sh.hist[w * 256 + threadIdx.x];
      sh.hist[threadIdx.x] = s;
    }
    __syncthreads();
    if (wid == 0) {
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
      const unsigned ball = __ballot_sync(0xffffffffu, excl < remaining && incl >= remaining);
      const int owner = ball ? (__ffs(ball) - 1) : 31;
      if (lane == owner) {
        int cum = excl, digit = 8 * (31 - lane);
#pragma unroll
        for (int d = 0; d < 8; ++d) {
          if (cum + loc[d] >= remaining) { digit = 8 * (31 - lane) + (7 - d); break; }
          cum += loc[d];
        }
        sh.misc[64] = digit;
        sh.misc[65] = remaining - cum;
        sh.misc[66] = cum;
      }
    }
    __syncthreads();
    gt += sh.misc[66];
    remaining = sh.misc[65];
    prefix |= (uint32_t)sh.misc[64] << shift;
    pmask |= 0xFFu << shift;
    __syncthreads();
  }
  *kstar = prefix;
  *above = gt;
  *take = remaining;
}

// The top-M (key, index) composites of v over rg, sorted descending, in sh.sortbuf[0..M).
// prefer_high: at the boundary key keep the highest indices and rank a higher index
// higher (stable ascending ranks); otherwise the lowest indices, ranked first (topk).
__device__ void top_sorted(const float* v, const Range& rg, int M, bool prefer_high, SelSmem& sh) {
  uint32_t kstar;
  int above, take;
  radix_select(v, rg, M, sh, &kstar, &above, &take);
  const int lane = threadIdx.x & 31;
  // ties at the boundary key: rank them in index order
  chunk_counts(rg.n, sh.cnt_a, [&](int i) { return rg.ok(i) && float_key(v[i]) == kstar; });
  const int nties = scan_counts(sh.cnt_a, (rg.n + 31) / 32, sh.misc);
  if (threadIdx.x == 0) sh.misc[67] = 0;
  __syncthreads();
  for (int base = threadIdx.x - lane; base < rg.n; base += blockDim.x) {
    const int i = base + lane;
    bool ok = i < rg.n && rg.ok(i);
    const uint32_t k = ok ? float_key(v[i]) : 0u;
    const uint32_t tie = prefer_high ? (uint32_t)i : ~(uint32_t)i;
    // strictly above: warp-aggregated slot allocation
    const unsigned ab = __ballot_sync(0xffffffffu, ok && k > kstar);
    int basepos = 0;
    if (lane == 0 && ab) basepos = atomicAdd(&sh.misc[67], __popc(ab));
    basepos = __shfl_sync(0xffffffffu, basepos, 0);
    if (ok && k > kstar) sh.sortbuf[basepos + __popc(ab & lanemask_lt())] = ((unsigned long long)k << 32) | tie;
    // boundary ties in index order
    const unsigned tb = __ballot_sync(0xffffffffu, ok && k == kstar);
    if (ok && k == kstar) {
      const int r = chunk_rank(sh.cnt_a, i, tb);
      const int ord = prefer_high ? (nties - 1 - r) : r;   // highest index first when prefer_high
      if (ord < take) sh.sortbuf[above + ord] = ((unsigned long long)kstar << 32) | tie;
    }
  }
  __syncthreads();
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
          if (((i & k) == 0) ? (a < b) : (a > b)) { sh.sortbuf[i] = b; sh.sortbuf[l] = a; }
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
// finished chain scores (PU:2186-2204)
// ---------------------------------------------------------------------------
__device__ int early_stop_steps(const Plan& pl, const char* ws, float* scratch) {
  const float* cmax = reinterpret_cast<const float*>(ws + pl.off_cmax);
  const float* ymax = reinterpret_cast<const float*>(ws + pl.off_ymax);
  // max over chunks of every (chain, term) at once: thread t handles (ch, k) pairs by warps
  __shared__ float tmax[2][kMaxIters + 1];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int q = wid; q < pl.nchains * pl.K; q += kSelWarps) {
    const int ch = q / pl.K, k = 1 + q % pl.K;
    float m = 0.f;
    if (pl.n_p > pl.s)
      for (int c = lane; c < pl.nscan; c += 32)
        m = fmaxf(m, __ldcg(cmax + ((size_t)ch * pl.nscan + c) * (kMaxIters + 1) + k));
    m = warp_max(m);
    if (lane == 0) tmax[ch][k] = fmaxf(m, __ldcg(ymax + ch * (pl.K + 1) + k));
  }
  __syncthreads();
  int steps = pl.K;
  for (int k = 1; k <= pl.K; ++k) {
    bool small = true;
    for (int ch = 0; ch < pl.nchains; ++ch) small = small && (tmax[ch][k] < 1e-8f);
    if (small) { steps = k; break; }
  }
  (void)scratch;
  return steps;
}

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

// Writes the finished scores of chain ch into out (global, [n]).
__device__ void finish_chain(const Plan& pl, const char* ws, int ch, int steps, float* out,
                             float* fscratch) {
  const int n = pl.n, s = pl.s;
  float tot = 0.f, mx = 0.f;
  for (int j = s + threadIdx.x; j < n; j += blockDim.x) {
    const float v = raw_result(pl, ws, ch, j, steps);
    out[j] = v;
    tot += v;
    mx = fmaxf(mx, v);
  }
  tot = block_reduce<false>(tot, fscratch);
  mx = block_reduce<true>(mx, fscratch);
  const float sinkv = tot * 0.01f;
  mx = fmaxf(mx, s > 0 ? sinkv : 0.f);
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
// the cluster kernel
// ---------------------------------------------------------------------------
__device__ void set_bit(uint32_t* bits, int i) { atomicOr(bits + (i >> 5), 1u << (i & 31)); }
CKV_DEV bool get_bit(const uint32_t* bits, int i) { return (bits[i >> 5] >> (i & 31)) & 1u; }

__global__ void __launch_bounds__(kSelThreads) k_select(SelArgs a) {
  extern __shared__ __align__(16) char smraw[];
  cg::cluster_group cluster = cg::this_cluster();
  const int v = (int)cluster.block_rank();     // which score vector this CTA owns
  const Plan& pl = a.pl;
  const ckv_params& prm = a.p;
  char* ws = a.ws;
  Header* hdr = reinterpret_cast<Header*>(ws);
  const int n = pl.n;
  const SelLayout L = sel_layout(n);
  SelSmem sh;
  sh.sortbuf = reinterpret_cast<unsigned long long*>(smraw + L.off_sort);
  sh.hist = reinterpret_cast<int*>(sh.sortbuf);
  float* sc = reinterpret_cast<float*>(ws + pl.off_sel);               // [3][n] finished scores
  float* gx = sc + 3 * (size_t)n;                                      // [3][n] global vectors
  int* gcomb = reinterpret_cast<int*>(gx + 3 * (size_t)n);             // [n]
  sh.x = L.smem_scores ? reinterpret_cast<float*>(smraw + L.off_x) : gx + (size_t)v * n;
  sh.cnt_a = reinterpret_cast<int*>(smraw + L.off_cnt_a);
  sh.cnt_b = reinterpret_cast<int*>(smraw + L.off_cnt_b);
  sh.bits = reinterpret_cast<uint32_t*>(smraw + L.off_bits);
  sh.misc = reinterpret_cast<int*>(smraw + L.off_misc);
  sh.fmisc = reinterpret_cast<float*>(sh.misc + 128);
  const int mode = pl.mode;
  const bool dis = mode == CKV_COMB_DIS;

  // ---- phase 0: this CTA's vector into sc[v], then (smoothed) into x
  float* mysc = sc + (size_t)v * n;
  if (a.given) {
    const float* g = v == 0 ? a.ga : (v == 1 ? a.gb : a.gc);
    for (int j = threadIdx.x; j < n; j += blockDim.x) mysc[j] = g[j];
    __syncthreads();
  } else if (v < pl.nchains) {
    const int steps = early_stop_steps(pl, ws, sh.fmisc);
    finish_chain(pl, ws, v, steps, mysc, sh.fmisc);
    if (v == 0 && threadIdx.x == 0) hdr->steps = steps;
    if (mode == CKV_COMB_UNION_DA) {
      const float* colsum = reinterpret_cast<const float*>(ws + pl.off_colsum);
      for (int j = threadIdx.x; j < n; j += blockDim.x) mysc[j] = mysc[j] * fmaxf(colsum[j], 1e-8f);
      __syncthreads();
    }
  }
  if (a.finish_only) {
    if (v < pl.nchains)
      for (int j = threadIdx.x; j < n; j += blockDim.x) a.out_scores[(size_t)v * n + j] = mysc[j];
    return;
  }
  if (dis) {
    int k;
    float sig;
    if (v == 0) {
      k = prm.qi_kernel_size != 0 ? prm.qi_kernel_size : prm.smoothing_kernel;
      if (prm.smooth_hi_only && k > 1) k = 0;
      sig = prm.use_gaussian ? prm.gaussian_sigma * 0.5f : 1.0f;
    } else if (v == 1) {
      k = prm.hi_kernel_size != 0 ? prm.hi_kernel_size : prm.smoothing_kernel;
      sig = prm.gaussian_sigma;
    } else {
      k = prm.bi_kernel_size;
      sig = prm.gaussian_sigma;
    }
    smooth(mysc, sh.x, n, k, prm.use_gaussian, sig);
  } else {
    for (int j = threadIdx.x; j < n; j += blockDim.x) sh.x[j] = mysc[j];
    __syncthreads();
  }
  if (a.out_scores && v < 2)
    for (int j = threadIdx.x; j < n; j += blockDim.x) a.out_scores[(size_t)v * n + j] = sh.x[j];

  // ---- phase 1: this vector's top list
  const int lo = pl.s, hi = pl.n - pl.W;   // candidates [s, n-W)
  const int kk = pl.kk;
  const bool uni = mode == CKV_COMB_UNION || mode == CKV_COMB_UNION_DA;
  int M = 0;
  if (uni) {
    const int remaining = kk, cand = hi - lo;
    const int qb = (int)((float)remaining * prm.qi_ratio), hb = remaining - qb;
    M = (v == 0) ? min(qb, cand) : min(cand, hb + qb + remaining);
    if (threadIdx.x == 0) { sh.misc[70] = min(qb, cand); sh.misc[71] = min(hb, cand); }
    if (M > 0) top_sorted(sh.x, Range{n, lo, hi, true}, M, false, sh);
  } else {
    const bool zeroed = (dis && v == 0 && prm.ablate_qi) || (dis && v == 1 && prm.ablate_hi);
    M = min(n, kk + pl.s + pl.W);
    if (!zeroed && kk > 0) top_sorted(sh.x, Range{n, 0, n, false}, M, true, sh);
  }
  if (threadIdx.x == 0) sh.misc[72] = M;
  cluster.sync();

  // ---- phase 2 (CTA 0): combine, threshold, compact
  if (v == 0) {
    const int nv = cluster.num_blocks();
    for (int i = threadIdx.x; i < L.nchunk; i += blockDim.x) sh.bits[i] = 0u;
    __syncthreads();
    if (kk > 0 && uni) {
      const int qk = sh.misc[70], hk = sh.misc[71];
      const unsigned long long* hl = cluster.map_shared_rank(sh.sortbuf, 1);
      const int ext = *cluster.map_shared_rank(sh.misc + 72, 1);
      for (int p = threadIdx.x; p < qk; p += blockDim.x) set_bit(sh.bits, sorted_index(sh.sortbuf[p], false));
      __syncthreads();
      for (int p = threadIdx.x; p < hk; p += blockDim.x) set_bit(sh.bits, sorted_index(hl[p], false));
      __syncthreads();
      int cnt = 0;
      for (int i = threadIdx.x; i < L.nchunk; i += blockDim.x) cnt += __popc(sh.bits[i]);
      cnt = (int)block_reduce<false>((float)cnt, sh.fmisc);
      if (cnt < kk && threadIdx.x < 32) {
        int have = cnt;
        for (int base = 0; base < ext && have < kk; base += 32) {
          const int p = base + threadIdx.x;
          int idx = -1;
          bool add = false;
          if (p < ext) { idx = sorted_index(hl[p], false); add = !get_bit(sh.bits, idx); }
          const unsigned ball = __ballot_sync(0xffffffffu, add);
          if (add && have + __popc(ball & lanemask_lt()) < kk) set_bit(sh.bits, idx);
          have += __popc(ball);
        }
      }
      __syncthreads();
    } else if (kk > 0) {
      int live = 0;
      for (int u = 0; u < nv; ++u) live += *cluster.map_shared_rank(sh.misc + 72, u) > 0 &&
                                           !((dis && u == 0 && prm.ablate_qi) || (dis && u == 1 && prm.ablate_hi));
      const int Mx = min(n, kk + pl.s + pl.W);
      if (live == 0) {
        for (int i = lo + threadIdx.x; i < lo + kk; i += blockDim.x) set_bit(sh.bits, i);
        __syncthreads();
      } else {
        // combined ranks of the union of the top lists (others: below every kept rank)
        int* comb = L.smem_scores ? reinterpret_cast<int*>(sh.x) : gcomb;
        for (int i = threadIdx.x; i < n; i += blockDim.x) comb[i] = -1;
        __syncthreads();
        for (int u = 0; u < nv; ++u) {
          const bool zeroed = (dis && u == 0 && prm.ablate_qi) || (dis && u == 1 && prm.ablate_hi);
          if (zeroed) continue;
          const unsigned long long* lst = cluster.map_shared_rank(sh.sortbuf, u);
          for (int p = threadIdx.x; p < Mx; p += blockDim.x)
            atomicMax(&comb[sorted_index(lst[p], true)], n - 1 - p);
        }
        __syncthreads();
        // histogram of combined ranks >= n - Mx over the candidates (cnt_b reused as bins)
        // bins over [n - Mx, n): CTA 0's own list has been consumed, its buffer is free
        int* hbuf = sh.hist;
        for (int i = threadIdx.x; i < Mx; i += blockDim.x) hbuf[i] = 0;
        __syncthreads();
        for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
          const int r = comb[i];
          if (r >= n - Mx) atomicAdd(&hbuf[r - (n - Mx)], 1);
        }
        __syncthreads();
        {
          const int c = (Mx + blockDim.x - 1) / blockDim.x;
          const int bhi = Mx - (int)threadIdx.x * c, blo = max(0, bhi - c);
          int local = 0;
          for (int b = blo; b < bhi; ++b) local += hbuf[b];
          int tot;
          const int above = block_exclusive_scan(local, sh.misc, &tot);
          if (threadIdx.x == 0) { sh.misc[80] = n; sh.misc[81] = 0; }
          __syncthreads();
          if (above < kk && above + local >= kk) {
            int cum = above;
            for (int b = bhi - 1; b >= blo; --b) {
              if (cum + hbuf[b] >= kk) { sh.misc[80] = (n - Mx) + b; sh.misc[81] = kk - cum; break; }
              cum += hbuf[b];
            }
          }
          __syncthreads();
          if (threadIdx.x == 0 && sh.misc[80] == n) set_status(&hdr->status, kStatusCount);
        }
        const int t = sh.misc[80], need = sh.misc[81];
        // at the threshold: the lowest `need` candidate indices
        chunk_counts(n, sh.cnt_a, [&](int i) { return i >= lo && i < hi && comb[i] == t; });
        scan_counts(sh.cnt_a, L.nchunk, sh.misc);
        const int lane = threadIdx.x & 31;
        for (int base = threadIdx.x - lane; base < n; base += blockDim.x) {
          const int i = base + lane;
          const bool cand = i < n && i >= lo && i < hi;
          const int r = cand ? comb[i] : -1;
          const unsigned tb = __ballot_sync(0xffffffffu, cand && r == t);
          if (cand && (r > t || (r == t && chunk_rank(sh.cnt_a, i, tb) < need))) set_bit(sh.bits, i);
        }
        __syncthreads();
      }
    }
    // compaction: sinks + chosen, ascending
    const int cap = pl.s + kk;
    chunk_counts(hi, sh.cnt_a, [&](int i) { return i < pl.s || get_bit(sh.bits, i); });
    const int total = scan_counts(sh.cnt_a, (hi + 31) / 32, sh.misc);
    const int lane = threadIdx.x & 31;
    for (int base = threadIdx.x - lane; base < hi; base += blockDim.x) {
      const int i = base + lane;
      const bool kp = i < hi && (i < pl.s || get_bit(sh.bits, i));
      const unsigned b = __ballot_sync(0xffffffffu, kp);
      if (kp) {
        const int r = chunk_rank(sh.cnt_a, i, b);
        if (r < cap) a.out_idx[r] = i;
      }
    }
    for (int i = total + threadIdx.x; i < cap; i += blockDim.x) a.out_idx[i] = 0;
    if (threadIdx.x == 0) {
      hdr->kept = total;
      if (total != cap) set_status(&hdr->status, kStatusCount);
    }
  }
  cluster.sync();   // the other CTAs' lists stay alive until CTA 0 is done
}

size_t select_smem_bytes_n(int n) { return sel_layout(n).total; }

cudaError_t launch_select(const SelArgs& a, cudaStream_t st) {
  const Plan& pl = a.pl;
  const bool bridge = pl.mode == CKV_COMB_DIS && a.p.use_bridge_importance &&
                      (a.given ? a.gc != nullptr : true);
  const int nv = a.finish_only ? pl.nchains : (bridge ? 3 : 2);
  const size_t smem = sel_layout(pl.n).total;
  { const cudaError_t e = ensure_dynamic_smem((const void*)k_select, smem); if (e != cudaSuccess) return e; }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nv, 1, 1);
  cfg.blockDim = dim3(kSelThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = nv;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_select, a);
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
constexpr size_t kNoAllocBytes = sizeof(Header) + (size_t)29 * kNoAllocMaxN;
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
  pl.off_sel = sizeof(Header);
  pl.total = sizeof(Header) + pl.sel_bytes;
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
