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
constexpr int kMaxSort = 8192;          // largest top-M list sorted in shared memory
constexpr int kSliceSmemMax = 16384;    // slice positions kept in shared memory

// Shared memory of one CTA: a sort buffer (used by the vector's leader CTA; the
// per-warp radix histograms alias it), the CTA's slice of its score vector, per
// 32-position chunk counts, scalars, and the histograms / scalars that the other
// CTAs of the cluster read through distributed shared memory.
struct SelLayout {
  int n, P, S, nchunk;
  bool smem_x;
  size_t off_sort, off_x, off_cnt, off_misc, off_hx, off_xch, off_rk, total;
};

__host__ __device__ inline SelLayout sel_layout(int n, int P) {
  SelLayout L;
  L.n = n;
  L.P = P;
  const int per = (n + P - 1) / P;
  L.S = (per + 31) & ~31;
  L.nchunk = L.S / 32;
  L.smem_x = L.S <= kSliceSmemMax;
  size_t off = 0;
  auto take = [&](size_t b) { const size_t o = off; off = (off + b + 15) & ~(size_t)15; return o; };
  L.off_sort = take(sizeof(unsigned long long) * kMaxSort);
  L.off_x = take(L.smem_x ? sizeof(float) * (size_t)L.S : 0);
  L.off_cnt = take(sizeof(int) * (size_t)(L.nchunk > 0 ? L.nchunk : 1));
  L.off_misc = take(sizeof(int) * 256);
  L.off_hx = take(sizeof(int) * 2 * 256);
  L.off_xch = take(sizeof(float) * 16);
  L.off_rk = take(sizeof(int) * 5 * 256);
  L.total = off;
  return L;
}

struct SelSmem {
  unsigned long long* sortbuf;
  int* hist;        // [kSelWarps][256] (aliases sortbuf)
  int* cnt;         // per 32-position chunk counts of a range
  int* misc;        // [0..63] scan scratch, [64..] scalars
  float* fmisc;     // misc + 128: reduction scratch
  int* hx;          // [2][256] this CTA's histogram, read by the vector's other CTAs
  float* xch;       // exchanged scalars: [0] total, [1] max; ints at [2..]
  int* ixch;
  int* rk;          // [5][256] digit totals / below / bases / running / round totals (full ranks)
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

// Ballot counts of pred(i) per 32-position chunk of [b0, b1) into cnt (b0 32-aligned).
template <class Pred>
__device__ void chunk_counts(int b0, int b1, int* cnt, Pred pred) {
  const int lane = threadIdx.x & 31;
  for (int base = b0 + (int)threadIdx.x - lane; base < b1; base += blockDim.x) {
    const int i = base + lane;
    const unsigned b = __ballot_sync(0xffffffffu, i < b1 && pred(i));
    if (lane == 0) cnt[(base - b0) >> 5] = __popc(b);
  }
  __syncthreads();
}

// Rank (in index order) of position i among those with pred true in [b0, ..), given the scanned chunk counts.
CKV_DEV int chunk_rank(const int* cnt, int b0, int i, unsigned ball) {
  return cnt[(i - b0) >> 5] + __popc(ball & lanemask_lt());
}

CKV_DEV int sorted_index(unsigned long long e, bool prefer_high) {
  const uint32_t lo = (uint32_t)(e & 0xffffffffull);
  return (int)(prefer_high ? lo : ~lo);
}

// ---------------------------------------------------------------------------
// top-M of one vector, spread over the P CTAs that hold its slices
// ---------------------------------------------------------------------------
// Radix select (4 passes of 8 bits) of the M-th largest key over positions
// [lo, hi) of the vector; each CTA counts its slice [b0, b1) (values x[i - b0]),
// the P histograms are summed through distributed shared memory, and every CTA of
// the vector takes the same digit.  Called by every CTA of the cluster.
__device__ void radix_select(cg::cluster_group& cl, const float* x, int b0, int b1, int lo, int hi, int M,
                             int vbase, int P, SelSmem& sh, uint32_t* kstar, int* above, int* take) {
  uint32_t prefix = 0, pmask = 0;
  int remaining = M, gt = 0;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  int* myhist = sh.hist + wid * 256;
  const int r0 = max(b0, lo), r1 = min(b1, hi);
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = threadIdx.x; i < kSelWarps * 256; i += blockDim.x) sh.hist[i] = 0;
    __syncthreads();
    for (int i = r0 + threadIdx.x; i < r1; i += blockDim.x) {
      const uint32_t k = float_key(x[i - b0]);
      if ((k & pmask) == prefix) atomicAdd(&myhist[(k >> shift) & 255], 1);
    }
    __syncthreads();
    int* hx = sh.hx + (pass & 1) * 256;
    if (threadIdx.x < 256) {
      int s = 0;
      for (int w = 0; w < kSelWarps; ++w) s += sh.hist[w * 256 + threadIdx.x];
      hx[threadIdx.x] = s;
    }
    cl.sync();
    if (threadIdx.x < 256) {
      int s = 0;
      for (int q = 0; q < P; ++q) s += cl.map_shared_rank(hx, vbase + q)[threadIdx.x];
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

// Bitonic sort (descending) of buf[0, P2), P2 a power of two <= E * blockDim.x, with
// the elements in registers: element i = warp * 32E + 32e + lane.  Compare distances
// below 32 are lane shuffles, 32 .. 32E - 1 swaps inside a thread, and only distances
// of 32E and more go through shared memory (two barriers each).  All threads.
template <int E>
__device__ void bitonic_desc(unsigned long long* buf, int P2) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned long long v[E];
  int idx[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    idx[e] = warp * 32 * E + e * 32 + lane;
    v[e] = idx[e] < P2 ? buf[idx[e]] : 0ull;
  }
  // new value of element i against partner value p at distance j within blocks of k
  auto cmpx = [](unsigned long long own, unsigned long long p, int i, int j, int k) {
    const bool desc = (i & k) == 0, lower = (i & j) == 0;
    const bool take_max = desc == lower;
    const bool own_gt = own > p;
    return (take_max == own_gt) ? own : p;
  };
  for (int k = 2; k <= P2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j >= 32 * E) {
        __syncthreads();   // the previous stage's readers are done
#pragma unroll
        for (int e = 0; e < E; ++e)
          if (idx[e] < P2) buf[idx[e]] = v[e];
        __syncthreads();
#pragma unroll
        for (int e = 0; e < E; ++e)
          if (idx[e] < P2) v[e] = cmpx(v[e], buf[idx[e] ^ j], idx[e], j, k);
      } else if (j >= 32) {
        unsigned long long nv[E];
#pragma unroll
        for (int b = 1; b < E; b <<= 1) {
          if ((j >> 5) == b) {
#pragma unroll
            for (int e = 0; e < E; ++e) nv[e] = cmpx(v[e], v[e ^ b], idx[e], j, k);
#pragma unroll
            for (int e = 0; e < E; ++e) v[e] = nv[e];
          }
        }
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const unsigned long long p = __shfl_xor_sync(0xffffffffu, v[e], j);
          v[e] = cmpx(v[e], p, idx[e], j, k);
        }
      }
    }
  }
  __syncthreads();
#pragma unroll
  for (int e = 0; e < E; ++e)
    if (idx[e] < P2) buf[idx[e]] = v[e];
  __syncthreads();
}

// The top-M (key, index) composites of the vector over [lo, hi), sorted descending,
// in the leader CTA's sort buffer.  prefer_high: at the boundary key keep the highest
// indices and rank a higher index higher (stable ascending ranks); otherwise the
// lowest indices, ranked first (topk).  Called by every CTA of the cluster.
__device__ void top_sorted(cg::cluster_group& cl, const float* x, int b0, int b1, int lo, int hi, int M,
                           bool prefer_high, int vbase, int P, bool leader, SelSmem& sh) {
  uint32_t kstar;
  int above, take;
  radix_select(cl, x, b0, b1, lo, hi, M, vbase, P, sh, &kstar, &above, &take);
  const int lane = threadIdx.x & 31;
  const int r0 = max(b0, lo), r1 = min(b1, hi);
  auto in_range = [&](int i) { return i >= r0 && i < r1; };
  // boundary ties of this slice in index order; slices of lower rank come first
  chunk_counts(b0, b1, sh.cnt, [&](int i) { return in_range(i) && float_key(x[i - b0]) == kstar; });
  const int my_ties = scan_counts(sh.cnt, (b1 - b0 + 31) / 32, sh.misc);
  if (threadIdx.x == 0) {
    sh.ixch[2] = my_ties;
    if (leader) sh.misc[67] = 0;
  }
  cl.sync();
  int tie_base = 0, nties = 0;
  const int part = (int)cl.block_rank() - vbase;
  for (int q = 0; q < P; ++q) {
    const int c = cl.map_shared_rank(sh.ixch, vbase + q)[2];
    if (q < part) tie_base += c;
    nties += c;
  }
  unsigned long long* dst = cl.map_shared_rank(sh.sortbuf, vbase);
  int* dcnt = cl.map_shared_rank(sh.misc + 67, vbase);
  for (int base = b0 + (int)threadIdx.x - lane; base < b1; base += blockDim.x) {
    const int i = base + lane;
    const bool ok = i < b1 && in_range(i);
    const uint32_t k = ok ? float_key(x[i - b0]) : 0u;
    const uint32_t tie = prefer_high ? (uint32_t)i : ~(uint32_t)i;
    // strictly above: warp-aggregated slot allocation in the leader's buffer
    const unsigned ab = __ballot_sync(0xffffffffu, ok && k > kstar);
    int basepos = 0;
    if (lane == 0 && ab) basepos = atomicAdd(dcnt, __popc(ab));
    basepos = __shfl_sync(0xffffffffu, basepos, 0);
    if (ok && k > kstar) dst[basepos + __popc(ab & lanemask_lt())] = ((unsigned long long)k << 32) | tie;
    const unsigned tb = __ballot_sync(0xffffffffu, ok && k == kstar);
    if (ok && k == kstar) {
      const int r = tie_base + chunk_rank(sh.cnt, b0, i, tb);
      const int ord = prefer_high ? (nties - 1 - r) : r;   // highest index first when prefer_high
      if (ord < take) dst[above + ord] = ((unsigned long long)kstar << 32) | tie;
    }
  }
  cl.sync();
  if (leader) {
    int P2 = 1;
    while (P2 < M) P2 <<= 1;
    for (int i = M + threadIdx.x; i < P2; i += blockDim.x) sh.sortbuf[i] = 0ull;
    __syncthreads();
    if (P2 <= kSelThreads) bitonic_desc<1>(sh.sortbuf, P2);
    else if (P2 <= 2 * kSelThreads) bitonic_desc<2>(sh.sortbuf, P2);
    else if (P2 <= 4 * kSelThreads) bitonic_desc<4>(sh.sortbuf, P2);
    else bitonic_desc<8>(sh.sortbuf, P2);
  }
}

// ---------------------------------------------------------------------------
// full stable ranks of one vector (weighted combination, PU:1865-1882)
// ---------------------------------------------------------------------------
// The lanes of the warp whose 9-bit values d (0..256) equal this lane's: one ballot per bit
// (cheaper here than match.any, whose cost dominated the radix passes).
CKV_DEV unsigned warp_peers9(int d) {
  unsigned peers = 0xffffffffu;
#pragma unroll
  for (int b = 0; b < 9; ++b) {
    const bool bit = (d >> b) & 1;
    const unsigned m = __ballot_sync(0xffffffffu, bit);
    peers &= bit ? m : ~m;
  }
  return peers;
}

// argsort(argsort(x)) with a stable sort, over the P CTAs that hold the vector's
// slices: a 4-pass LSD radix sort of the 32-bit keys (float_key) carried with their
// indices through two global buffers (L2-resident).  Each pass: inside a CTA every warp
// owns a contiguous range of the slice and sweeps it in 32-element steps (digit peers from
// ballots), counting its digits (one counting sweep); the per-warp counts give each (digit, warp)
// its offset within the CTA, the per-CTA totals exchanged through distributed shared
// memory give each (digit, CTA) its output base, and a second sweep places the elements
// (within a warp: step order, then lane order).  Stable passes over a sequence that
// starts in index order leave equal keys in index order, so rank[i] = the final
// position of element i.  All CTAs of the cluster call it.
__device__ void full_ranks(cg::cluster_group& cl, const float* x, int b0, int b1, int vbase, int P, int part,
                           unsigned long long* bufA, unsigned long long* bufB, int* rank, SelSmem& sh) {
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, bd = blockDim.x, nwarps = bd >> 5;
  int* tot = sh.rk;              // [256] digit totals over the vector
  int* below = sh.rk + 256;      // [256] digit counts of lower-ranked CTAs
  int* base = sh.rk + 512;       // [256] output base of each digit for this CTA
  int* rtot = sh.rk + 1024;      // [256] scan scratch
  int* wcnt = sh.hist;           // [warps][256] per-warp digit counts, then running offsets
  for (int j = b0 + tid; j < b1; j += bd)
    bufA[j] = ((unsigned long long)float_key(x[j - b0]) << 32) | (uint32_t)j;
  __syncthreads();
  unsigned long long* in = bufA;
  unsigned long long* out = bufB;
  // warp w owns [b0 + w E, b0 + (w + 1) E): E a multiple of 32
  const int E = ((b1 - b0 + 32 * nwarps - 1) / (32 * nwarps)) * 32;
  const int w0 = b0 + wid * E, w1 = min(b1, w0 + E);
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 32 + 8 * pass;
    int* hx = sh.hx + (pass & 1) * 256;
    for (int i = tid; i < nwarps * 256; i += bd) wcnt[i] = 0;
    __syncthreads();
    int* wc = wcnt + wid * 256;
    for (int q0 = w0; q0 < w1; q0 += 4 * 32) {   // counting sweep, 4 steps' loads in flight
      int dg[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int pos = q0 + 32 * u + lane;
        dg[u] = pos < w1 ? (int)((__ldcg(in + pos) >> shift) & 255u) : 256;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int d = dg[u];
        const unsigned peers = warp_peers9(d);
        if (d < 256 && lane == __ffs(peers) - 1) wc[d] += __popc(peers);
        __syncwarp();
      }
    }
    __syncthreads();
    if (tid < 256) {   // per digit: exclusive offsets of the warps, and this CTA's total
      int acc = 0;
      for (int q = 0; q < nwarps; ++q) {
        const int c = wcnt[q * 256 + tid];
        wcnt[q * 256 + tid] = acc;
        acc += c;
      }
      hx[tid] = acc;
    }
    cl.sync();
    if (tid < 256) {
      int t = 0, bl = 0;
      for (int q = 0; q < P; ++q) {
        const int c = cl.map_shared_rank(hx, vbase + q)[tid];
        t += c;
        if (q < part) bl += c;
      }
      tot[tid] = t;
      below[tid] = bl;
    }
    __syncthreads();
    if (wid < 8) {   // exclusive scan of the 256 digit totals
      const int d = wid * 32 + lane;
      int incl = tot[d];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      rtot[d] = incl;   // warp-inclusive; warp offsets below
    }
    __syncthreads();
    if (tid < 256) {
      int off = 0;
      for (int q = 0; q < (tid >> 5); ++q) off += rtot[q * 32 + 31];
      base[tid] = off + rtot[tid] - tot[tid] + below[tid];
    }
    __syncthreads();
    for (int q0 = w0; q0 < w1; q0 += 4 * 32) {   // placing sweep, 4 steps' loads in flight
      unsigned long long ev[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int pos = q0 + 32 * u + lane;
        ev[u] = pos < w1 ? __ldcg(in + pos) : ~0ull;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const bool act = q0 + 32 * u + lane < w1;
        const int d = act ? (int)((ev[u] >> shift) & 255u) : 256;
        const unsigned peers = warp_peers9(d);
        if (act) out[base[d] + wc[d] + __popc(peers & lanemask_lt())] = ev[u];
        __syncwarp();
        if (act && lane == __ffs(peers) - 1) wc[d] += __popc(peers);
        __syncwarp();
      }
    }
    cl.sync();   // every element of the pass is placed
    unsigned long long* t = in;
    in = out;
    out = t;
  }
  for (int j = b0 + tid; j < b1; j += bd) rank[(uint32_t)__ldcg(in + j)] = j;
  cl.sync();
}

// ---------------------------------------------------------------------------
// finished chain scores (PU:2186-2204)
// ---------------------------------------------------------------------------
__device__ int early_stop_steps(const Plan& pl, const char* ws) {
  const float* cmax = reinterpret_cast<const float*>(ws + pl.off_cmax);
  const float* ymax = reinterpret_cast<const float*>(ws + pl.off_ymax);
  // max over chunks of every (chain, term): one warp per pair
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

// Smoothing kernel taps of a zero-padded conv1d (PU:1884-1919).
CKV_DEV int smooth_taps(int k, bool gaussian, float sigma, float (&w)[32]) {
  const int kk = min(k, 32);
  float wsum = 0.f;
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
  return kk;
}

// ---------------------------------------------------------------------------
// the cluster kernel
// ---------------------------------------------------------------------------
// Cluster of nv * P CTAs: CTA rank c owns slice c % P of score vector c / P
// (32-aligned slices of S positions) for the finishing, smoothing and top-M
// phases, and slice c of the positions (T positions) for the combination and
// compaction phases.  Every cluster barrier below is taken by every CTA.
__global__ void __launch_bounds__(kSelThreads, 1) k_select(SelArgs a) {
  extern __shared__ __align__(16) char smraw[];
  cg::cluster_group cl = cg::this_cluster();
  const int C = (int)cl.num_blocks();
  const int rank = (int)cl.block_rank();
  const int P = a.parts;
  const int v = rank / P, part = rank % P, vbase = v * P;
  const bool leader = part == 0;
  const Plan& pl = a.pl;
  const ckv_params& prm = a.p;
  char* ws = a.ws;
  Header* hdr = reinterpret_cast<Header*>(ws);
  const int n = pl.n;
  const SelLayout L = sel_layout(n, P);
  SelSmem sh;
  sh.sortbuf = reinterpret_cast<unsigned long long*>(smraw + L.off_sort);
  sh.hist = reinterpret_cast<int*>(sh.sortbuf);
  sh.cnt = reinterpret_cast<int*>(smraw + L.off_cnt);
  sh.misc = reinterpret_cast<int*>(smraw + L.off_misc);
  sh.fmisc = reinterpret_cast<float*>(sh.misc + 128);
  sh.hx = reinterpret_cast<int*>(smraw + L.off_hx);
  sh.xch = reinterpret_cast<float*>(smraw + L.off_xch);
  sh.ixch = reinterpret_cast<int*>(sh.xch);
  sh.rk = reinterpret_cast<int*>(smraw + L.off_rk);
  float* sc = reinterpret_cast<float*>(ws + pl.off_sel);               // [3][n] finished scores
  float* gx = sc + 3 * (size_t)n;                                      // [3][n] slices not held in smem
  int* gcomb = reinterpret_cast<int*>(gx + 3 * (size_t)n);             // [n] combined ranks
  int* gbins = reinterpret_cast<int*>(gx);                             // [n] rank histogram (after the lists)
  uint32_t* gbits = reinterpret_cast<uint32_t*>(gcomb + n);            // [ceil(n/32)] keep bits
  const int b0 = min(n, part * L.S), b1 = min(n, b0 + L.S);            // vector slice
  float* x = L.smem_x ? reinterpret_cast<float*>(smraw + L.off_x) : gx + (size_t)v * n + b0;
  const int T = (((n + C - 1) / C) + 31) & ~31;
  const int g0 = min(n, rank * T), g1 = min(n, g0 + T);               // position slice
  const int mode = pl.mode;
  const bool dis = mode == CKV_COMB_DIS;
  const bool uni = mode == CKV_COMB_UNION || mode == CKV_COMB_UNION_DA;
  const int lane = threadIdx.x & 31;

  // combined ranks start below every kept rank; keep bits start clear
  for (int i = g0 + threadIdx.x; i < g1; i += blockDim.x) gcomb[i] = -1;
  for (int i = g0 / 32 + threadIdx.x; i < (g1 + 31) / 32; i += blockDim.x) gbits[i] = 0u;

  // ---- phase 0: finished scores of this slice into sc[v] (PU:2186-2204)
  float* mysc = sc + (size_t)v * n;
  const bool chain = !a.given && v < pl.nchains;
  int steps = 0;
  if (a.given) {
    const float* g = v == 0 ? a.ga : (v == 1 ? a.gb : a.gc);
    for (int j = b0 + threadIdx.x; j < b1; j += blockDim.x) mysc[j] = g[j];
  } else if (chain) {
    steps = early_stop_steps(pl, ws);
    // sums of 32-position blocks (the slices are 32-aligned), so that the total below
    // does not depend on how many CTAs share the vector
    float* bsum = gx + (size_t)v * n;   // [ceil(n / 32)]; free until the smoothing phase
    const int wid = threadIdx.x >> 5;
    float mx = 0.f;
    for (int jb = b0 + 32 * wid; jb < b1; jb += 32 * kSelWarps) {
      const int j = jb + lane;
      float r = 0.f;
      if (j < b1 && j >= pl.s) {
        r = raw_result(pl, ws, v, j, steps);
        mysc[j] = r;
        mx = fmaxf(mx, r);
      }
      const float bs = warp_sum(r);
      if (lane == 0) bsum[jb >> 5] = bs;
    }
    mx = block_reduce<true>(mx, sh.fmisc);
    if (threadIdx.x == 0) sh.xch[1] = mx;
  }
  cl.sync();
  if (chain) {
    float mx = 0.f;
    for (int q = 0; q < P; ++q) mx = fmaxf(mx, cl.map_shared_rank(sh.xch, vbase + q)[1]);
    // the total of the block sums in a fixed order (one warp; the same in every CTA)
    if (threadIdx.x < 32) {
      const float* bsum = gx + (size_t)v * n;
      float t = 0.f;
      for (int k = lane; k < (n + 31) / 32; k += 32) t += __ldcg(bsum + k);
      t = warp_sum(t);
      if (lane == 0) sh.fmisc[64] = t;
    }
    __syncthreads();
    const float tot = sh.fmisc[64];
    const float sinkv = tot * 0.01f;
    mx = fmaxf(mx, pl.s > 0 ? sinkv : 0.f);
    const float* colsum = reinterpret_cast<const float*>(ws + pl.off_colsum);
    const float imx = mx > 0.f ? 1.0f / mx : 0.f;
    for (int j = b0 + threadIdx.x; j < b1; j += blockDim.x) {
      float val = (j < pl.s) ? sinkv : mysc[j];
      if (mx > 0.f) val = div_rcp(val, mx, imx);
      if (mode == CKV_COMB_UNION_DA) val = val * fmaxf(__ldcg(colsum + j), 1e-8f);
      mysc[j] = val;
    }
    if (rank == 0 && threadIdx.x == 0) hdr->steps = steps;
  }
  if (a.finish_only) {
    if (chain)
      for (int j = b0 + threadIdx.x; j < b1; j += blockDim.x) a.out_scores[(size_t)v * n + j] = mysc[j];
    cl.sync();   // the exchanged totals stay readable until every CTA has them
    return;
  }
  cl.sync();   // finished vectors complete: smoothing reads the neighbouring slices

  // ---- phase 1: smoothing (PU:1921-1936, PU:3131-3160) of the slice into x
  {
    int k = 0;
    float sig = 1.0f;
    if (dis) {
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
    }
    if (k <= 1 || n <= k) {
      for (int j = b0 + threadIdx.x; j < b1; j += blockDim.x) x[j - b0] = mysc[j];
    } else {
      float w[32];
      const int kk = smooth_taps(k, prm.use_gaussian != 0, sig, w);
      const int pad = k / 2;
      for (int j = b0 + threadIdx.x; j < b1; j += blockDim.x) {
        float acc = 0.f;
        for (int t = 0; t < kk; ++t) {
          const int src = j + t - pad;
          if (src >= 0 && src < n) acc = fmaf(w[t], __ldcg(mysc + src), acc);
        }
        x[j - b0] = acc;
      }
    }
    __syncthreads();
    if (a.out_scores && v < 2)
      for (int j = b0 + threadIdx.x; j < b1; j += blockDim.x) a.out_scores[(size_t)v * n + j] = x[j - b0];
  }

  // ---- phase 2: this vector's top list, sorted, in its leader CTA
  const int lo = pl.s, hi = pl.n - pl.W;   // candidates [s, n-W)
  const int kk = pl.kk;
  const int cand = hi - lo;
  const int qb = (int)((float)kk * prm.qi_ratio), hb = kk - qb;
  const int Mx = min(n, kk + pl.s + pl.W);
  int M;
  if (uni) M = (v == 0) ? min(qb, cand) : min(cand, hb + qb + kk);
  else M = Mx;
  const bool weighted = mode == CKV_COMB_WEIGHTED;
  if (weighted) {
    // full stable ranks of both vectors, then combined = w * rank(H2O) + (1 - w) * rank(influence)
    // (PU:3237-3240); its top kk over the candidates, lowest index first at ties (PU:2616-2644)
    char* wbase = reinterpret_cast<char*>(ws + pl.off_sel) + (((size_t)29 * n + 15) & ~(size_t)15);
    unsigned long long* bufs = reinterpret_cast<unsigned long long*>(wbase);     // [2 vectors][2][n]
    int* ranks = reinterpret_cast<int*>(bufs + (size_t)4 * n);                 // [2][n]
    full_ranks(cl, x, b0, b1, vbase, P, part, bufs + (size_t)v * 2 * n, bufs + (size_t)v * 2 * n + n,
               ranks + (size_t)v * n, sh);
    const float wh = prm.h2o_weight, wi = (float)(1.0 - (double)prm.h2o_weight);
    const float den = (float)(n - 1), iden = n > 1 ? 1.0f / den : 0.f;
    for (int j = b0 + threadIdx.x; j < b1; j += blockDim.x) {
      float ir = 1.f, hr = 1.f;
      if (n > 1) {
        ir = div_rcp((float)__ldcg(ranks + j), den, iden);       // influence (vector 0)
        hr = div_rcp((float)__ldcg(ranks + n + j), den, iden);   // H2O (vector 1)
      }
      x[j - b0] = __fadd_rn(__fmul_rn(wh, hr), __fmul_rn(wi, ir));
    }
    __syncthreads();
    M = max(min(kk, cand), 1);
    top_sorted(cl, x, b0, b1, lo, hi, M, false, vbase, P, leader, sh);
  } else if (uni) {
    top_sorted(cl, x, b0, b1, lo, hi, M, false, vbase, P, leader, sh);
  } else {
    top_sorted(cl, x, b0, b1, 0, n, M, true, vbase, P, leader, sh);
  }
  cl.sync();   // sorted lists ready

  // ---- phase 3: combination (PU:3177-3196 rank MAX; PU:2489-2589 union)
  auto zeroed = [&](int u) { return (dis && u == 0 && prm.ablate_qi) || (dis && u == 1 && prm.ablate_hi); };
  const int nv = C / P;
  int live = 0;
  for (int u = 0; u < nv; ++u) live += zeroed(u) ? 0 : 1;
  const bool rankmax = !uni && !weighted && kk > 0 && live > 0;
  for (int i = g0 + threadIdx.x; i < min(g1, Mx); i += blockDim.x) gbins[i] = 0;
  if (rankmax) {
    // combined rank of every listed position: MAX over the vectors of n - 1 - list position
    for (int u = 0; u < nv; ++u) {
      if (zeroed(u)) continue;
      const unsigned long long* lst = cl.map_shared_rank(sh.sortbuf, u * P);
      for (int p = rank * (int)blockDim.x + threadIdx.x; p < Mx; p += C * (int)blockDim.x)
        atomicMax(&gcomb[sorted_index(lst[p], true)], n - 1 - p);
    }
  }
  cl.sync();
  if (rankmax)
    for (int i = max(g0, lo) + threadIdx.x; i < min(g1, hi); i += blockDim.x) {
      const int r = __ldcg(gcomb + i);
      if (r >= n - Mx) atomicAdd(&gbins[r - (n - Mx)], 1);
    }
  cl.sync();
  int t = n, need = 0;
  if (rankmax) {
    // threshold: the combined rank at which the kept count reaches kk (every CTA alike)
    const int c = (Mx + blockDim.x - 1) / blockDim.x;
    const int bhi = Mx - (int)threadIdx.x * c, blo = max(0, bhi - c);
    int local = 0;
    for (int b = blo; b < bhi; ++b) local += __ldcg(gbins + b);
    int tot;
    const int above = block_exclusive_scan(local, sh.misc, &tot);
    if (threadIdx.x == 0) { sh.misc[80] = n; sh.misc[81] = 0; }
    __syncthreads();
    if (above < kk && above + local >= kk) {
      int cum = above;
      for (int b = bhi - 1; b >= blo; --b) {
        const int hb_ = __ldcg(gbins + b);
        if (cum + hb_ >= kk) { sh.misc[80] = (n - Mx) + b; sh.misc[81] = kk - cum; break; }
        cum += hb_;
      }
    }
    __syncthreads();
    t = sh.misc[80];
    need = sh.misc[81];
    if (rank == 0 && threadIdx.x == 0 && t == n) set_status(&hdr->status, kStatusCount);
    chunk_counts(g0, g1, sh.cnt, [&](int i) { return i >= lo && i < hi && __ldcg(gcomb + i) == t; });
    const int mine = scan_counts(sh.cnt, (g1 - g0 + 31) / 32, sh.misc);
    if (threadIdx.x == 0) sh.ixch[3] = mine;
  }
  cl.sync();
  if (rankmax) {
    // at the threshold: the lowest `need` candidate indices
    int base = 0;
    for (int q = 0; q < rank; ++q) base += cl.map_shared_rank(sh.ixch, q)[3];
    for (int b = g0 + (int)threadIdx.x - lane; b < g1; b += blockDim.x) {
      const int i = b + lane;
      const bool cnd = i < g1 && i >= lo && i < hi;
      const int r = cnd ? __ldcg(gcomb + i) : -1;
      const unsigned tb = __ballot_sync(0xffffffffu, cnd && r == t);
      const bool keep = cnd && (r > t || (r == t && base + chunk_rank(sh.cnt, g0, i, tb) < need));
      const unsigned word = __ballot_sync(0xffffffffu, keep);
      if (lane == 0) gbits[i >> 5] = word;
    }
  } else if (weighted && kk > 0 && rank == 0) {
    // weighted: the kk best combined scores (vector 0's list)
    const int m = min(kk, cand);
    for (int q = threadIdx.x; q < m; q += blockDim.x) {
      const int i = sorted_index(sh.sortbuf[q], false);
      atomicOr(gbits + (i >> 5), 1u << (i & 31));
    }
  } else if (!uni && !weighted && kk > 0) {
    // every vector ablated: the first kk candidates
    for (int b = g0 + (int)threadIdx.x - lane; b < g1; b += blockDim.x) {
      const int i = b + lane;
      const unsigned word = __ballot_sync(0xffffffffu, i < g1 && i >= lo && i < lo + kk);
      if (lane == 0) gbits[i >> 5] = word;
    }
  } else if (uni && kk > 0 && rank == 0) {
    // union: QI top qk, HI top hk, then fill from the HI list in order
    const int qk = min(qb, cand), hk = min(hb, cand);
    const unsigned long long* l0 = sh.sortbuf;
    const unsigned long long* l1 = cl.map_shared_rank(sh.sortbuf, P);
    const int ext = min(cand, hb + qb + kk);
    for (int p = threadIdx.x; p < qk; p += blockDim.x) {
      const int i = sorted_index(l0[p], false);
      atomicOr(gbits + (i >> 5), 1u << (i & 31));
    }
    for (int p = threadIdx.x; p < hk; p += blockDim.x) {
      const int i = sorted_index(l1[p], false);
      atomicOr(gbits + (i >> 5), 1u << (i & 31));
    }
    __syncthreads();
    int cnt = 0;
    for (int i = threadIdx.x; i < (n + 31) / 32; i += blockDim.x) cnt += __popc(__ldcg(gbits + i));
    cnt = (int)block_reduce<false>((float)cnt, sh.fmisc);
    if (cnt < kk && threadIdx.x < 32) {
      int have = cnt;
      for (int base = 0; base < ext && have < kk; base += 32) {
        const int p = base + threadIdx.x;
        int idx = -1;
        bool add = false;
        if (p < ext) {
          idx = sorted_index(l1[p], false);
          add = !((__ldcg(gbits + (idx >> 5)) >> (idx & 31)) & 1u);
        }
        const unsigned ball = __ballot_sync(0xffffffffu, add);
        if (add && have + __popc(ball & lanemask_lt()) < kk) atomicOr(gbits + (idx >> 5), 1u << (idx & 31));
        have += __popc(ball);
      }
    }
  }
  cl.sync();   // keep bits complete

  // ---- phase 4: compaction (PU:3496-3501): sinks + chosen, ascending
  const int cap = pl.s + kk;
  const int h1 = min(g1, hi);
  auto kept = [&](int i) { return i < h1 && (i < pl.s || ((__ldcg(gbits + (i >> 5)) >> (i & 31)) & 1u)); };
  int mine = 0;
  if (g0 < h1) {
    chunk_counts(g0, h1, sh.cnt, kept);
    mine = scan_counts(sh.cnt, (h1 - g0 + 31) / 32, sh.misc);
  }
  if (threadIdx.x == 0) sh.ixch[4] = mine;
  cl.sync();
  int base = 0, total = 0;
  for (int q = 0; q < C; ++q) {
    const int c = cl.map_shared_rank(sh.ixch, q)[4];
    if (q < rank) base += c;
    total += c;
  }
  for (int b = g0 + (int)threadIdx.x - lane; b < h1; b += blockDim.x) {
    const int i = b + lane;
    const bool kp = kept(i);
    const unsigned bb = __ballot_sync(0xffffffffu, kp);
    if (kp) {
      const int r = base + chunk_rank(sh.cnt, g0, i, bb);
      if (r < cap) a.out_idx[r] = i;
    }
  }
  if (rank == C - 1) {
    for (int i = total + threadIdx.x; i < cap; i += blockDim.x) a.out_idx[i] = 0;
    if (threadIdx.x == 0) {
      hdr->kept = total;
      if (total != cap) set_status(&hdr->status, kStatusCount);
    }
  }
  cl.sync();   // shared memory stays readable until every CTA is done with it
}

// CTAs per score vector: up to 16 CTAs per cluster where the device schedules that
// cluster size, else the portable 8.
static int select_parts(int nv, size_t smem, cudaStream_t st, bool narrow) {
  if (narrow) return 8 / nv;
  static std::mutex mu;
  static int cached[64][4] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  std::lock_guard<std::mutex> lock(mu);
  if (cached[dev][nv] != 0) return cached[dev][nv];
  int parts = 8 / nv;
  if (cudaFuncSetAttribute(k_select, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    const int p16 = 16 / nv;
    cfg.gridDim = dim3(nv * p16, 1, 1);
    cfg.blockDim = dim3(kSelThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = nv * p16;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int nclusters = 0;
    if (cudaOccupancyMaxActiveClusters(&nclusters, k_select, &cfg) == cudaSuccess && nclusters >= 1) parts = p16;
    cudaGetLastError();
  }
  cached[dev][nv] = parts;
  return parts;
}

size_t select_smem_bytes_n(int n) { return sel_layout(n, 2).total; }

cudaError_t launch_select(const SelArgs& a0, cudaStream_t st) {
  SelArgs a = a0;
  const Plan& pl = a.pl;
  const bool bridge = pl.mode == CKV_COMB_DIS && a.p.use_bridge_importance &&
                      (a.given ? a.gc != nullptr : true);
  const int nv = a.finish_only ? pl.nchains : (bridge ? 3 : 2);
  const bool uni = pl.mode == CKV_COMB_UNION || pl.mode == CKV_COMB_UNION_DA;
  if (pl.kk + pl.s + pl.W > kMaxSort || (uni && 2 * pl.kk > kMaxSort)) return cudaErrorInvalidValue;   // make_plan rejects these
  // the shared memory layout depends on the slice length, hence on the CTAs per vector
  const size_t s8 = sel_layout(pl.n, 8 / nv).total, s16 = sel_layout(pl.n, 16 / nv).total;
  { const cudaError_t e = ensure_dynamic_smem((const void*)k_select, s8 > s16 ? s8 : s16); if (e != cudaSuccess) return e; }
  a.parts = select_parts(nv, s16, st, a.narrow != 0);
  const size_t smem = sel_layout(pl.n, a.parts).total;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nv * a.parts, 1, 1);
  cfg.blockDim = dim3(kSelThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = nv * a.parts;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_select, a);
}

// ---------------------------------------------------------------------------
// per-head eviction (PU:2208-2382 importance, PU:3296-3464 selection)
// ---------------------------------------------------------------------------
// k_ph_finish, one CTA per (head, vector): QI = query row + eq * two-hop, HI = query
// row * (n_t - pos) / n_t * eh + query row (or the window column sums with
// true_hub_hi) over [s, n); sinks = 0.01 * sum; divided by max(max, 1e-8); cut to
// n - W and smoothed with the Gaussian kernel.  With both ablations the second
// vector is the raw column sum (H2O).  CTA (h, 0) also totals the head's
// query-row entropy.
__global__ void __launch_bounds__(kSelThreads) k_ph_finish(PhArgs a) {
  const Plan& pl = a.pl;
  const ckv_params& prm = a.p;
  const int h = blockIdx.x, v = blockIdx.y;
  const int n = pl.n, s = pl.s, nw = pl.ph_nw;
  const float* qrow = reinterpret_cast<const float*>(a.ws + pl.off_ph_qrow) + (size_t)h * n;
  const float* two = reinterpret_cast<const float*>(a.ws + pl.off_ph_two) + (size_t)h * n;
  const float* col = reinterpret_cast<const float*>(a.ws + pl.off_ph_col) + (size_t)h * n;
  float* vec = reinterpret_cast<float*>(a.ws + pl.off_ph_vec) + ((size_t)h * 2 + v) * nw;
  float* tmp = reinterpret_cast<float*>(a.ws + pl.off_ph_bufs) + (size_t)h * 8 * nw + (size_t)v * n;
  __shared__ float red[64];
  if (v == 0) {   // the head's query-row entropy: -sum_j p ln(p + 1e-10)
    const float* entp = reinterpret_cast<const float*>(a.ws + pl.off_ph_ent);
    float t = 0.f;
    for (int i = threadIdx.x; i < pl.ph_ent_parts; i += blockDim.x) t += __ldcg(entp + (size_t)i * pl.H + h);
    t = block_reduce<false>(t, red);
    if (threadIdx.x == 0)
      reinterpret_cast<float*>(a.ws + pl.off_ph_ent)[(size_t)pl.ph_ent_parts * pl.H + h] = -t;
  }
  if (v == 1 && prm.ablate_qi && prm.ablate_hi) {   // H2O per head: raw column sums
    for (int j = threadIdx.x; j < nw; j += blockDim.x) vec[j] = __ldcg(col + j);
    return;
  }
  const float nt = (float)(n - s), int_ = 1.0f / nt;
  float tot = 0.f, mx = 0.f;
  for (int j = s + threadIdx.x; j < n; j += blockDim.x) {
    float r;
    if (v == 0) {
      r = __fadd_rn(__ldcg(qrow + j), __fmul_rn(a.eq, __ldcg(two + j)));
    } else if (prm.true_hub_hi) {
      r = __ldcg(col + j);
    } else {
      const float qt = __ldcg(qrow + j);
      const float hw = div_rcp(nt - (float)(j - s), nt, int_);
      r = __fadd_rn(__fmul_rn(__fmul_rn(qt, hw), a.eh), qt);
    }
    tmp[j] = r;
    tot += r;
    mx = fmaxf(mx, r);
  }
  tot = block_reduce<false>(tot, red);
  mx = block_reduce<true>(mx, red);
  const float sinkv = __fmul_rn(tot, 0.01f);
  if (s > 0) mx = fmaxf(mx, sinkv);
  mx = fmaxf(mx, 1e-8f);
  const float imx = 1.0f / mx;
  __syncthreads();
  for (int j = threadIdx.x; j < nw; j += blockDim.x) tmp[j] = div_rcp(j < s ? sinkv : tmp[j], mx, imx);
  __syncthreads();
  const int ksz = prm.smoothing_kernel > 0 ? prm.smoothing_kernel : max(prm.qi_kernel_size, prm.hi_kernel_size);
  if (ksz > 1 && nw > ksz) {
    float wt[32];
    const int kk = smooth_taps(ksz, true, prm.gaussian_sigma, wt);
    const int pad = ksz / 2;
    for (int j = threadIdx.x; j < nw; j += blockDim.x) {
      float acc = 0.f;
      for (int t = 0; t < kk; ++t) {
        const int src = j + t - pad;
        if (src >= 0 && src < nw) acc = fmaf(wt[t], __ldcg(tmp + src), acc);
      }
      vec[j] = acc;
    }
  } else {
    for (int j = threadIdx.x; j < nw; j += blockDim.x) vec[j] = __ldcg(tmp + j);
  }
}

// k_ph_ghi, one cluster: the mean over heads of the (smoothed) HI vectors and its
// stable ranks, normalised by n - W - 1 (the global HI of PU:3400-3440).
__global__ void __launch_bounds__(kSelThreads, 1) k_ph_ghi(PhArgs a) {
  extern __shared__ __align__(16) char smraw[];
  cg::cluster_group cl = cg::this_cluster();
  const int P = (int)cl.num_blocks(), part = (int)cl.block_rank();
  const Plan& pl = a.pl;
  const int nw = pl.ph_nw, H = pl.H;
  const SelLayout L = sel_layout(nw, P);
  SelSmem sh;
  sh.sortbuf = reinterpret_cast<unsigned long long*>(smraw + L.off_sort);
  sh.hist = reinterpret_cast<int*>(sh.sortbuf);
  sh.cnt = reinterpret_cast<int*>(smraw + L.off_cnt);
  sh.misc = reinterpret_cast<int*>(smraw + L.off_misc);
  sh.fmisc = reinterpret_cast<float*>(sh.misc + 128);
  sh.hx = reinterpret_cast<int*>(smraw + L.off_hx);
  sh.xch = reinterpret_cast<float*>(smraw + L.off_xch);
  sh.ixch = reinterpret_cast<int*>(sh.xch);
  sh.rk = reinterpret_cast<int*>(smraw + L.off_rk);
  const float* vec = reinterpret_cast<const float*>(a.ws + pl.off_ph_vec);
  unsigned long long* gbuf = reinterpret_cast<unsigned long long*>(a.ws + pl.off_ph_gbuf);
  int* granks = reinterpret_cast<int*>(gbuf + 2 * (size_t)nw);
  float* ghi = reinterpret_cast<float*>(a.ws + pl.off_ph_ghi);
  const int b0 = min(nw, part * L.S), b1 = min(nw, b0 + L.S);
  float* x = L.smem_x ? reinterpret_cast<float*>(smraw + L.off_x) : ghi + b0;   // ghi doubles as scratch
  const float fh = (float)H, ih = 1.0f / fh;
  for (int j = b0 + threadIdx.x; j < b1; j += blockDim.x) {
    float sum = 0.f;
    for (int h = 0; h < H; ++h) sum += __ldcg(vec + ((size_t)h * 2 + 1) * nw + j);
    x[j - b0] = div_rcp(sum, fh, ih);
  }
  __syncthreads();
  full_ranks(cl, x, b0, b1, 0, P, part, gbuf, gbuf + nw, granks, sh);
  const float den = (float)(nw - 1), iden = nw > 1 ? 1.0f / den : 0.f;
  for (int j = b0 + threadIdx.x; j < b1; j += blockDim.x)
    ghi[j] = nw > 1 ? div_rcp((float)__ldcg(granks + j), den, iden) : 1.f;
}

// k_ph_select, one cluster of 8 CTAs per head (4 per vector): stable ranks of the
// head's QI and HI vectors over [0, n - W), the per-head score of PU:3376-3440 (QI
// rank only; global HI rank; H2O rank; entropy-adaptive mix; or MAX(QI rank,
// global HI rank)), its top m over [s, n - W) with the lowest indices first at ties
// (topk), and the kept positions, sinks first, ascending (PU:3442-3452).
__global__ void __launch_bounds__(kSelThreads, 1) k_ph_select(PhArgs a) {
  extern __shared__ __align__(16) char smraw[];
  cg::cluster_group cl = cg::this_cluster();
  const int C = (int)cl.num_blocks(), rank = (int)cl.block_rank();
  const int P = C / 2, v = rank / P, part = rank % P, vbase = v * P;
  const int h = (int)blockIdx.x / C;
  const Plan& pl = a.pl;
  const ckv_params& prm = a.p;
  const int nw = pl.ph_nw, s = pl.s, m = pl.kk, nk = pl.s + pl.kk;
  const SelLayout L = sel_layout(nw, P);
  SelSmem sh;
  sh.sortbuf = reinterpret_cast<unsigned long long*>(smraw + L.off_sort);
  sh.hist = reinterpret_cast<int*>(sh.sortbuf);
  sh.cnt = reinterpret_cast<int*>(smraw + L.off_cnt);
  sh.misc = reinterpret_cast<int*>(smraw + L.off_misc);
  sh.fmisc = reinterpret_cast<float*>(sh.misc + 128);
  sh.hx = reinterpret_cast<int*>(smraw + L.off_hx);
  sh.xch = reinterpret_cast<float*>(smraw + L.off_xch);
  sh.ixch = reinterpret_cast<int*>(sh.xch);
  sh.rk = reinterpret_cast<int*>(smraw + L.off_rk);
  const float* vec = reinterpret_cast<const float*>(a.ws + pl.off_ph_vec) + ((size_t)h * 2 + v) * nw;
  unsigned long long* bufs = reinterpret_cast<unsigned long long*>(a.ws + pl.off_ph_bufs) + (size_t)h * 4 * nw;
  int* ranks = reinterpret_cast<int*>(a.ws + pl.off_ph_ranks) + (size_t)h * 2 * nw;
  const float* ghi = reinterpret_cast<const float*>(a.ws + pl.off_ph_ghi);
  const int nwords = (nw + 31) / 32;
  uint32_t* bits = reinterpret_cast<uint32_t*>(a.ws + pl.off_ph_bits) + (size_t)h * nwords;
  const int b0 = min(nw, part * L.S), b1 = min(nw, b0 + L.S);
  float* x = reinterpret_cast<float*>(smraw + L.off_x);   // the launcher guarantees slices in smem
  const int T = (((nw + C - 1) / C) + 31) & ~31;
  const int g0 = min(nw, rank * T), g1 = min(nw, g0 + T);
  const int lane = threadIdx.x & 31;
  for (int i = g0 / 32 + threadIdx.x; i < (g1 + 31) / 32; i += blockDim.x) bits[i] = 0u;
  for (int j = b0 + threadIdx.x; j < b1; j += blockDim.x) x[j - b0] = __ldcg(vec + j);
  __syncthreads();
  full_ranks(cl, x, b0, b1, vbase, P, part, bufs + (size_t)v * 2 * nw, bufs + (size_t)v * 2 * nw + nw,
             ranks + (size_t)v * nw, sh);
  // per-head combined score weights
  const bool aq = prm.ablate_qi, ah = prm.ablate_hi;
  float wq = 0.5f;
  if (!aq && !ah && prm.entropy_adaptive) {
    const float* ent = reinterpret_cast<const float*>(a.ws + pl.off_ph_ent) + (size_t)pl.ph_ent_parts * pl.H;
    float lo = INFINITY, hi = -INFINITY;
    for (int q = 0; q < pl.H; ++q) { const float e = __ldcg(ent + q); lo = fminf(lo, e); hi = fmaxf(hi, e); }
    if (hi > lo) wq = __fsub_rn(1.0f, __fdiv_rn(__fsub_rn(__ldcg(ent + h), lo), __fsub_rn(hi, lo)));
  }
  // the combined score and its top list over all C CTAs of the cluster (both vectors' CTAs
  // share the work): this CTA's 1/C slice of the positions, ranks read back from global memory
  const float den = (float)(nw - 1), iden = nw > 1 ? 1.0f / den : 0.f;
  const SelLayout LC = sel_layout(nw, C);
  const int c0 = min(nw, rank * LC.S), c1 = min(nw, c0 + LC.S);
  for (int j = c0 + threadIdx.x; j < c1; j += blockDim.x) {
    const float qr = nw > 1 ? div_rcp((float)__ldcg(ranks + j), den, iden) : 1.f;
    const float hr = nw > 1 ? div_rcp((float)__ldcg(ranks + nw + j), den, iden) : 1.f;
    float sc;
    if (ah && !aq) sc = qr;
    else if (aq && !ah) sc = __ldcg(ghi + j);
    else if (aq && ah) sc = hr;
    else if (prm.entropy_adaptive) sc = __fadd_rn(__fmul_rn(wq, qr), __fmul_rn(__fsub_rn(1.0f, wq), hr));
    else sc = fmaxf(qr, __ldcg(ghi + j));
    x[j - c0] = sc;
  }
  __syncthreads();
  top_sorted(cl, x, c0, c1, s, nw, max(m, 1), false, 0, C, rank == 0, sh);
  cl.sync();
  if (rank == 0 && m > 0)
    for (int q = threadIdx.x; q < m; q += blockDim.x) {
      const int i = sorted_index(sh.sortbuf[q], false);
      atomicOr(bits + (i >> 5), 1u << (i & 31));
    }
  cl.sync();
  // kept positions ascending: sinks, then the chosen
  const int h1 = g1;
  auto kept = [&](int i) { return i < h1 && (i < s || ((__ldcg(bits + (i >> 5)) >> (i & 31)) & 1u)); };
  int mine = 0;
  if (g0 < h1) {
    chunk_counts(g0, h1, sh.cnt, kept);
    mine = scan_counts(sh.cnt, (h1 - g0 + 31) / 32, sh.misc);
  }
  if (threadIdx.x == 0) sh.ixch[4] = mine;
  cl.sync();
  int base = 0;
  for (int q = 0; q < rank; ++q) base += cl.map_shared_rank(sh.ixch, q)[4];
  int32_t* out = a.out_idx + (size_t)h * nk;
  for (int b = g0 + (int)threadIdx.x - lane; b < h1; b += blockDim.x) {
    const int i = b + lane;
    const bool kp = kept(i);
    const unsigned bb = __ballot_sync(0xffffffffu, kp);
    if (kp) {
      const int r = base + chunk_rank(sh.cnt, g0, i, bb);
      if (r < nk) out[r] = i;
    }
  }
  cl.sync();
}

size_t ph_select_smem(int nw) { return sel_layout(nw, 4).total; }

cudaError_t launch_ph_select(const PhArgs& a, cudaStream_t st) {
  const Plan& pl = a.pl;
  const int nw = pl.ph_nw;
  if (sel_layout(nw, 4).smem_x == false || sel_layout(nw, 8).smem_x == false) return cudaErrorInvalidValue;
  cudaError_t e = cudaSuccess;
  k_ph_finish<<<dim3(pl.H, 2), kSelThreads, 0, st>>>(a);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  const bool need_ghi = (a.p.ablate_qi && !a.p.ablate_hi) || (!a.p.ablate_qi && !a.p.ablate_hi && !a.p.entropy_adaptive);
  auto cluster_launch = [&](const void* fn, int grid, int cdim, size_t smem) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(kSelThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cdim;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void* args[] = {const_cast<PhArgs*>(&a)};
    return cudaLaunchKernelExC(&cfg, fn, args);
  };
  if (need_ghi) {
    const size_t sm = sel_layout(nw, 8).total;
    if ((e = ensure_dynamic_smem((const void*)k_ph_ghi, sm)) != cudaSuccess) return e;
    if ((e = cluster_launch((const void*)k_ph_ghi, 8, 8, sm)) != cudaSuccess) return e;
  }
  const size_t sm = sel_layout(nw, 4).total;
  if ((e = ensure_dynamic_smem((const void*)k_ph_select, sm)) != cudaSuccess) return e;
  return cluster_launch((const void*)k_ph_select, pl.H * 8, 8, sm);
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
// (512 B, with the device status word) + the selection area (29 bytes per position)
// for up to 32768 positions, about 0.9 MiB that every GPU which loads the library
// holds until the process exits.  All calls share it and it keeps the last call's
// contents, so calls that overlap on the GPU (different streams, or different host
// threads on one device) race; order them on one stream.
constexpr int kNoAllocMaxN = 32768;
constexpr size_t kNoAllocBytes = sizeof(Header) + (size_t)29 * kNoAllocMaxN;
static_assert(sizeof(Header) == 512, "the static scratch starts with the 512-byte header");
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

// Device address of g_noalloc_scratch on the current device.  In host code the array's
// name is only a stand-in for it, so the address is looked up with the device current,
// on every call: the lookup is cheap once the module is loaded, and it stays right after
// the device's primary context is reset.  The first call on a device may load the
// module, which is not allowed while a stream is being captured.
cudaError_t noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  void* ptr = nullptr;
  e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
  if (e != cudaSuccess) return e;
  *out = ptr;
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
  if (p->per_head_eviction) {
    *why = "per-head selection needs the window attention: use ckv_score_evict";
    return CKV_ERR_UNSUPPORTED;
  }
  if (p->combination_mode == CKV_COMB_WEIGHTED) {
    *why = "ckv_select_scores_noalloc: combination_mode 'weighted' needs ckv_select_scores (workspace)";
    return CKV_ERR_UNSUPPORTED;
  }
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
