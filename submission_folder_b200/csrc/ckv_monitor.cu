// Decode-time scoring of circuit_kv's CircuitGraph (reference: CircuitKV/csrc/
// circuit_manager.cpp:433-766 with kernels/graph_update.cu, circuit_walker.cu and
// spectral_power.cu), the methods behind CircuitKVMonitor:
//
//   * graph update: row `current_idx` of a sparse attention graph gets the top_k keys
//     by raw dot product with the query (descending; ties by lower key index), the
//     scores as edge weights, -1 / 0 where fewer than top_k keys exist;
//   * absorbing circuit walker: walkers start at the source, step to a neighbour with
//     probability proportional to its edge weight, count every visit, and stop on
//     reaching the sink tokens [0, 4), a dead end or 1500 steps; PCG states per walker
//     carried across calls;
//   * spectral scores: 10 (or num_iterations) power iterations v <- A v / ||A v||_2
//     from v = 1 / sqrt(n) over the same graph;
//   * combined scores: walker visits and spectral scores each divided by their maximum,
//     then the element-wise maximum.
//
// This file is compiled with --use_fast_math, as the reference's extension is
// (CircuitKV/setup.py), so that its divisions, square roots and reciprocal square roots
// round as the reference's do; the sums keep the reference's order (sequential dot
// products and neighbour sums, the norm's strided partial sums reduced as trees of 256),
// so results are bit-identical to the reference's for the same graph and PCG states.
#include "ckv_common.cuh"
#include "ckv_monitor.h"

namespace ckv {

constexpr int kMonSink = 4;          // absorbing tokens [0, 4)
constexpr int kMonMaxSteps = 1500;   // walk length limit
constexpr int kMonThreads = 1024;

struct MonPcg {
  uint64_t state, inc;
};
CKV_DEV uint32_t mon_pcg_next(MonPcg& r) {
  const uint64_t old = r.state;
  r.state = old * 6364136223846793005ULL + r.inc;
  const uint32_t xs = (uint32_t)(((old >> 18u) ^ old) >> 27u);
  const uint32_t rot = (uint32_t)(old >> 59u);
  return (xs >> rot) | (xs << ((0u - rot) & 31u));
}
CKV_DEV float mon_uniform(MonPcg& r) { return (float)(mon_pcg_next(r) >> 8) * (1.0f / 16777216.0f); }

// ---- graph update -------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) k_graph_scores(const T* __restrict__ q, const T* __restrict__ keys, int n,
                                                      int D, float* __restrict__ scores) {
  extern __shared__ float sq[];
  for (int d = threadIdx.x; d < D; d += blockDim.x) sq[d] = (float)q[d];
  __syncthreads();
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= n) return;
  const T* kr = keys + (size_t)j * D;
  float s = 0.f;
  for (int d = 0; d < D; ++d) s = fmaf(sq[d], (float)kr[d], s);   // the dimensions in order
  scores[j] = s;
}

// (score, index) pairs in descending score, ties by lower index: a before b
CKV_DEV bool mon_before(float sa, int ia, float sb, int ib) { return sa > sb || (sa == sb && ia < ib); }

// One CTA: the top_k entries of scores[0, n) in that order, one block-wide arg-max per
// entry, each below the previous one.
__global__ void __launch_bounds__(kMonThreads) k_graph_topk(const float* __restrict__ scores, int n, int top_k,
                                                            int row, int32_t* __restrict__ adj,
                                                            float* __restrict__ weights) {
  __shared__ float ws[32];
  __shared__ int wi[32];
  __shared__ float last_s;
  __shared__ int last_i;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) { last_s = INFINITY; last_i = -1; }
  __syncthreads();
  for (int k = 0; k < top_k; ++k) {
    const float ps = last_s;
    const int pi = last_i;
    float bs = -INFINITY;
    int bi = -1;
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
      const float s = scores[j];
      if (mon_before(ps, pi, s, j) && (bi < 0 || mon_before(s, j, bs, bi))) { bs = s; bi = j; }
    }
    for (int o = 16; o > 0; o >>= 1) {
      const float os = __shfl_xor_sync(0xffffffffu, bs, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (oi >= 0 && (bi < 0 || mon_before(os, oi, bs, bi))) { bs = os; bi = oi; }
    }
    if (lane == 0) { ws[warp] = bs; wi[warp] = bi; }
    __syncthreads();
    if (warp == 0) {
      bs = lane < (int)(blockDim.x >> 5) ? ws[lane] : -INFINITY;
      bi = lane < (int)(blockDim.x >> 5) ? wi[lane] : -1;
      for (int o = 16; o > 0; o >>= 1) {
        const float os = __shfl_xor_sync(0xffffffffu, bs, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (oi >= 0 && (bi < 0 || mon_before(os, oi, bs, bi))) { bs = os; bi = oi; }
      }
      if (lane == 0) {
        adj[(size_t)row * top_k + k] = bi;        // -1 once the keys run out
        weights[(size_t)row * top_k + k] = bi >= 0 ? bs : 0.f;
        if (bi >= 0) { last_s = bs; last_i = bi; }
      }
    }
    __syncthreads();
  }
}

// ---- absorbing circuit walker -----------------------------------------------------------
__global__ void __launch_bounds__(256) k_circuit_walk(const int32_t* __restrict__ adj, const float* __restrict__ w,
                                                      int32_t* __restrict__ visits, uint64_t* __restrict__ states,
                                                      int source, int n, int top_k, int num_walkers) {
  const int wk = blockIdx.x * blockDim.x + threadIdx.x;
  if (wk >= num_walkers) return;
  MonPcg r{states[2 * wk], states[2 * wk + 1]};
  int pos = source;
  for (int step = 0; step < kMonMaxSteps; ++step) {
    atomicAdd(&visits[pos], 1);
    if (pos < kMonSink) break;   // absorbed
    const int32_t* nb = adj + (size_t)pos * top_k;
    const float* ww = w + (size_t)pos * top_k;
    float total = 0.f;
    int valid = 0;
    for (int k = 0; k < top_k; ++k) {
      const int j = nb[k];
      if (j >= 0 && j < n) { total += ww[k]; ++valid; }
    }
    if (valid == 0 || total <= 0.f) break;   // dead end
    const float target = mon_uniform(r) * total;
    float cum = 0.f;
    int next = -1;
    for (int k = 0; k < top_k && next < 0; ++k) {
      const int j = nb[k];
      if (j >= 0 && j < n) {
        cum += ww[k];
        if (cum >= target) next = j;
      }
    }
    if (next < 0) break;
    pos = next;
  }
  states[2 * wk] = r.state;
  states[2 * wk + 1] = r.inc;
}

__global__ void k_pcg_init(uint64_t* __restrict__ states, uint64_t seed, int num_walkers) {
  const int wk = blockIdx.x * blockDim.x + threadIdx.x;
  if (wk >= num_walkers) return;
  MonPcg r{0u, ((uint64_t)wk << 1u) | 1u};
  mon_pcg_next(r);
  r.state += seed;
  mon_pcg_next(r);
  states[2 * wk] = r.state;
  states[2 * wk + 1] = r.inc;
}

// ---- spectral power iteration (one CTA) ----------------------------------------------
// The squared norm as the reference forms it: nb = min(ceil(n / 256), 256) strided
// partial sums (block b, thread t: i = b 256 + t, b 256 + t + 256 nb, ...), each block's
// 256 reduced as a halving tree, then the nb partials reduced the same way.  1024
// threads work on four such blocks at a time.
CKV_DEV float mon_norm(const float* __restrict__ v, int n, float* sred, float* spart) {
  const int nb = min((n + 255) / 256, 256);
  const int t = threadIdx.x & 255, grp = threadIdx.x >> 8;
  for (int b0 = 0; b0 < nb; b0 += 4) {
    const int b = b0 + grp;
    float s = 0.f;
    if (b < nb)
      for (int i = b * 256 + t; i < n; i += 256 * nb) s = fmaf(v[i], v[i], s);
    sred[threadIdx.x] = s;
    __syncthreads();
    for (int stride = 128; stride > 0; stride >>= 1) {
      if (t < stride) sred[threadIdx.x] += sred[threadIdx.x + stride];
      __syncthreads();
    }
    if (t == 0 && b < nb) spart[b] = sred[threadIdx.x];
    __syncthreads();
  }
  if (threadIdx.x < 256) sred[threadIdx.x] = threadIdx.x < nb ? spart[threadIdx.x] : 0.f;
  __syncthreads();
  for (int stride = 128; stride > 0; stride >>= 1) {
    if (threadIdx.x < stride) sred[threadIdx.x] += sred[threadIdx.x + stride];
    __syncthreads();
  }
  const float total = sred[0];
  __syncthreads();
  return sqrtf(total);
}

__global__ void __launch_bounds__(kMonThreads) k_spectral(const int32_t* __restrict__ adj, const float* __restrict__ w,
                                                          int n, int top_k, int iters, float* __restrict__ v,
                                                          float* __restrict__ vtmp) {
  __shared__ float sred[kMonThreads];
  __shared__ float spart[256];
  const float u = rsqrtf((float)n);
  for (int i = threadIdx.x; i < n; i += blockDim.x) v[i] = u;
  __syncthreads();
  for (int it = 0; it < iters; ++it) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) {   // v_tmp = A v over the adjacency rows
      const int32_t* nb = adj + (size_t)i * top_k;
      const float* ww = w + (size_t)i * top_k;
      float s = 0.f;
      for (int k = 0; k < top_k; ++k) {
        const int j = nb[k];
        if (j >= 0 && j < n) s = fmaf(ww[k], v[j], s);
      }
      vtmp[i] = s;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) v[i] = vtmp[i];
    __syncthreads();
    const float nrm = mon_norm(v, n, sred, spart);
    if (nrm > 1e-8f)
      for (int i = threadIdx.x; i < n; i += blockDim.x) v[i] = v[i] / nrm;
    __syncthreads();
  }
}

// ---- combined scores (one CTA) ---------------------------------------------------------
CKV_DEV float mon_max(const float* __restrict__ v, int n, float* sred) {
  float m = -1e30f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, v[i]);
  sred[threadIdx.x] = m;
  __syncthreads();
  for (int stride = blockDim.x / 2; stride > 0; stride >>= 1) {
    if (threadIdx.x < stride) sred[threadIdx.x] = fmaxf(sred[threadIdx.x], sred[threadIdx.x + stride]);
    __syncthreads();
  }
  const float r = sred[0];
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kMonThreads) k_combine(const int32_t* __restrict__ visits, float* __restrict__ spectral,
                                                         float* __restrict__ walker, float* __restrict__ combined,
                                                         int n) {
  __shared__ float sred[kMonThreads];
  for (int i = threadIdx.x; i < n; i += blockDim.x) walker[i] = (float)visits[i];
  __syncthreads();
  const float ms = mon_max(spectral, n, sred);
  if (ms > 1e-8f)
    for (int i = threadIdx.x; i < n; i += blockDim.x) spectral[i] = spectral[i] / ms;
  const float mw = mon_max(walker, n, sred);
  if (mw > 1e-8f)
    for (int i = threadIdx.x; i < n; i += blockDim.x) walker[i] = walker[i] / mw;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) combined[i] = fmaxf(spectral[i], walker[i]);
}

// ---- landmark walkers ------------------------------------------------------------------
// CircuitGraph::update_and_step_landmark_walker / _absorbing_walker (circuit_manager.cpp:
// 768-1164; landmark_walker.cu, landmark_absorbing_walker.cu) over a dense fp32 attention
// matrix.  Every sum the reference forms by a sequential scan over a row (a source's start
// distribution over [4, source), a transition's total over [0, pos), the running cumsum of
// its sampling scan) is an fp32 prefix sum of that row taken in the same order.  So each
// row's prefix array is built once, sequentially, and a walker step reads its total from it
// and finds the first position whose running sum reaches the target by binary search: the
// same additions and comparisons as the reference's O(n) scans, in O(log n) per step.
// Where a row holds a negative or NaN value (the running sums are then not monotone) the
// walker scans that row's prefix array linearly instead.

constexpr int kLmMaxLandmarks = 32;   // landmarks per call
constexpr int kLmSinkBuffer = 20;     // landmark range starts at sink + 20 ...
constexpr int kLmWindow = 64;         // ... and ends 64 tokens before the end
constexpr int kLmRows = 3 + 2 * kLmMaxLandmarks;   // prefix rows: H2O, query x2, landmarks x2

// Column sums over the causal rows (H2O scores, landmark_walker.cu:476-505) in the
// reference's order: the partial of residue t (t < 256) sums rows i = t, t + 256, ... with
// i >= column, in increasing i; the 256 partials reduce as a halving tree.  A CTA owns 128
// adjacent columns: a lane reads 4 of them as one float4, so a warp reads 512 contiguous
// bytes of a row; warp w keeps the partials of residues w, w + 16, ..., w + 240 for its 4
// columns in registers (4 row loads in flight per warp at a time).  The partials
// meet in shared memory for the tree.  VEC = 0 (n not a multiple of 4): scalar loads.
constexpr int kH2oCols = 128;
constexpr int kH2oWarps = 16;
template <bool VEC>
__global__ void __launch_bounds__(32 * kH2oWarps) k_lm_h2o(const float* __restrict__ a, int n,
                                                            float* __restrict__ h2o) {
  extern __shared__ float part[];   // [256][kH2oCols]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c0 = blockIdx.x * kH2oCols, cl = c0 + 4 * lane;   // this lane's first column
  float acc[16][4];
#pragma unroll
  for (int m = 0; m < 16; ++m)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[m][e] = 0.f;
  for (int b = (c0 / 256) * 256; b < n; b += 256) {
#pragma unroll
    for (int h = 0; h < 16; h += 4) {   // groups of 4 rows in flight
      float4 x[4];
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int i = b + warp + 16 * (h + m);
        const float* row = a + (size_t)i * n;
        if (VEC) {
          x[m] = (i < n && cl < n) ? __ldg(reinterpret_cast<const float4*>(row + cl)) : make_float4(0.f, 0.f, 0.f, 0.f);
        } else {
          x[m].x = (i < n && cl < n) ? __ldg(row + cl) : 0.f;
          x[m].y = (i < n && cl + 1 < n) ? __ldg(row + cl + 1) : 0.f;
          x[m].z = (i < n && cl + 2 < n) ? __ldg(row + cl + 2) : 0.f;
          x[m].w = (i < n && cl + 3 < n) ? __ldg(row + cl + 3) : 0.f;
        }
      }
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int i = b + warp + 16 * (h + m);
        if (i < n) {   // rows at or below the diagonal of each column (i >= c)
          if (i >= cl) acc[h + m][0] += x[m].x;
          if (i >= cl + 1) acc[h + m][1] += x[m].y;
          if (i >= cl + 2) acc[h + m][2] += x[m].z;
          if (i >= cl + 3) acc[h + m][3] += x[m].w;
        }
      }
    }
  }
#pragma unroll
  for (int m = 0; m < 16; ++m)
    *reinterpret_cast<float4*>(part + (warp + 16 * m) * kH2oCols + 4 * lane) =
        make_float4(acc[m][0], acc[m][1], acc[m][2], acc[m][3]);
  __syncthreads();
  for (int stride = 128; stride > 0; stride >>= 1) {
    for (int e = threadIdx.x; e < stride * kH2oCols; e += blockDim.x)
      part[e] += part[e + stride * kH2oCols];   // residue e / 128 += residue e / 128 + stride
    __syncthreads();
  }
  if (threadIdx.x < kH2oCols && c0 + threadIdx.x < n) h2o[c0 + threadIdx.x] = part[threadIdx.x];
}

// Stratified landmarks (landmark_walker.cu:404-464): [24, n - 64) in num_landmarks equal
// segments (fewer, of at least min_spacing, when a segment would be shorter), the highest
// H2O score of each (first index among equals; NaN and values <= -1e30 never chosen), in
// segment order.  One warp per segment.
__global__ void __launch_bounds__(1024) k_lm_select(const float* __restrict__ h2o, int n, int max_landmarks,
                                                    int min_spacing, int32_t* __restrict__ positions,
                                                    int32_t* __restrict__ count) {
  __shared__ int best[kLmMaxLandmarks];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int valid_start = kMonSink + kLmSinkBuffer, valid_end = n - kLmWindow;
  const int range = valid_end - valid_start;
  if (range <= 0) {
    if (threadIdx.x == 0) *count = 0;
    return;
  }
  int segs = max_landmarks, seg = range / segs;
  if (seg < min_spacing && min_spacing > 0) {
    segs = max(range / min_spacing, 1);
    seg = range / segs;
  }
  if (warp < segs) {
    const int s0 = valid_start + warp * seg, s1 = warp == segs - 1 ? valid_end : s0 + seg;
    float bv = -1e30f;
    int bi = -1;
    for (int i = s0 + lane; i < s1; i += 32) {
      const float x = h2o[i];
      if (x > bv) { bv = x; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
    }
    if (lane == 0) best[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int cnt = 0;
    for (int w = 0; w < segs; ++w)
      if (best[w] >= 0) positions[cnt++] = best[w];
    *count = cnt;
  }
}

// Prefix rows, each of `stride` floats: P[m] = src[start] + ... + src[m - 1] summed left
// to right (0 for m <= start), for m <= len.  Row 0: H2O from 0; rows 1 / 2: the query's
// attention row from 0 / from the sink end; rows 3 + 2 l / 4 + 2 l: landmark l's row from 0 /
// from the sink end, up to its position.  mono[r] = 1 when every summed value is >= 0.
// One CTA per row: chunks staged in shared memory, summed in order by one thread.
__global__ void __launch_bounds__(1024) k_lm_prefix(const float* __restrict__ a, int n, int current_idx,
                                                    const float* __restrict__ h2o,
                                                    const int32_t* __restrict__ positions,
                                                    const int32_t* __restrict__ count, float* __restrict__ pref,
                                                    int stride, int32_t* __restrict__ mono) {
  __shared__ float buf[1024];
  __shared__ float carry;
  const int r = blockIdx.x;
  const float* src;
  int start = 0, len = n;
  if (r == 0) {
    src = h2o;
  } else if (r <= 2) {
    src = a + (size_t)current_idx * n;
    start = r == 2 ? kMonSink : 0;
  } else {
    const int l = (r - 3) >> 1;
    if (l >= *count) return;
    const int pos = positions[l];
    src = a + (size_t)pos * n;
    start = ((r - 3) & 1) ? kMonSink : 0;
    len = pos;
  }
  float* P = pref + (size_t)r * stride;
  for (int m = threadIdx.x; m <= min(start, len); m += blockDim.x) P[m] = 0.f;
  if (threadIdx.x == 0) carry = 0.f;
  bool ok = true;
  for (int j0 = start; j0 < len; j0 += 1024) {
    const int j = j0 + threadIdx.x;
    const int cnt = min(1024, len - j0);
    __syncthreads();
    if (j < len) {
      const float x = src[j];
      ok = ok && (x >= 0.f);
      buf[threadIdx.x] = x;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float run = carry;
      for (int t = 0; t < cnt; ++t) {
        run += buf[t];
        buf[t] = run;
      }
      carry = run;
    }
    __syncthreads();
    if (j < len) P[j + 1] = buf[threadIdx.x];
  }
  ok = __syncthreads_and(ok);
  if (threadIdx.x == 0) mono[r] = ok ? 1 : 0;
}

// The first j in [lo, hi) whose running sum P[j + 1] reaches target, else dflt.
CKV_DEV int lm_first_reach(const float* __restrict__ P, int lo, int hi, float target, bool mono, int dflt) {
  if (mono) {
    int x = lo, y = hi;
    while (x < y) {
      const int m = (x + y) >> 1;
      if (P[m + 1] >= target) y = m;
      else x = m + 1;
    }
    return x < hi ? x : dflt;
  }
  for (int j = lo; j < hi; ++j)
    if (P[j + 1] >= target) return j;
  return dflt;
}

// One thread per walker (landmark_walker.cu:59-236, landmark_absorbing_walker.cu:66-238):
// walkers_per_source walkers from every landmark and from the query (the last token, its
// row the attention row of current_idx), a start drawn from the source's row over
// [4, source); then at each position a visit of weight 1 (landmark walkers) or
// (int)query_boost (query walkers), absorption at [0, 4) (and, absorbing form, with
// probability 0.1 at another source's landmark), and a step to an earlier position drawn
// from the query's row (last 64 tokens), the landmark's row (at a landmark) or the H2O
// scores (elsewhere); a row with no mass jumps a random 2-10 % of the way to the sink.
__global__ void __launch_bounds__(256) k_lm_walk(const float* __restrict__ pref, int stride,
                                                 const int32_t* __restrict__ mono,
                                                 const int32_t* __restrict__ positions,
                                                 const int32_t* __restrict__ count, int n, int walkers_per_source,
                                                 float query_boost, int absorbing, int absorb_at_landmarks,
                                                 uint64_t* __restrict__ states, int32_t* __restrict__ visits) {
  __shared__ int32_t lm[kLmMaxLandmarks];
  const int L = *count;
  if (threadIdx.x < L) lm[threadIdx.x] = positions[threadIdx.x];
  __syncthreads();
  const int wk = blockIdx.x * blockDim.x + threadIdx.x;
  if (wk >= (L + 1) * walkers_per_source) return;
  const int src = wk / walkers_per_source;
  const bool is_q = src == L;
  const int src_lm = is_q ? -1 : src;
  const int source_pos = is_q ? n - 1 : lm[src];
  const int32_t weight = (int32_t)(is_q ? query_boost : 1.0f);
  const int srow = is_q ? 2 : 4 + 2 * src;
  const float* S = pref + (size_t)srow * stride;
  MonPcg r{states[2 * wk], states[2 * wk + 1]};
  float total = source_pos > kMonSink ? S[source_pos] : 0.f;
  if (total <= 1e-8f) {
    states[2 * wk] = r.state;
    states[2 * wk + 1] = r.inc;
    return;
  }
  float target = mon_uniform(r) * total;
  int pos = lm_first_reach(S, kMonSink, source_pos, target, mono[srow] != 0, kMonSink);
  const int window_start = max(0, n - kLmWindow);
  for (int step = 0; step < kMonMaxSteps; ++step) {
    atomicAdd(&visits[pos], weight);
    if (pos < kMonSink) break;
    if (absorbing && absorb_at_landmarks && L > 0) {
      bool absorbed = false;
      for (int l = 0; l < L; ++l)
        if (lm[l] == pos && l != src_lm) {
          absorbed = mon_uniform(r) < 0.1f;
          break;
        }
      if (absorbed) break;
    }
    int row = 0;   // H2O
    if (pos >= window_start) {
      row = 1;
    } else {
      for (int l = 0; l < L; ++l)
        if (lm[l] == pos) { row = 3 + 2 * l; break; }
    }
    const float* P = pref + (size_t)row * stride;
    total = P[pos];
    if (total <= 1e-8f) {
      const int distance = pos - kMonSink;
      const int jump = max(1, (int)((float)distance * fmaf(mon_uniform(r), 0.08f, 0.02f)));
      pos = max(kMonSink, pos - jump);
      continue;
    }
    target = mon_uniform(r) * total;
    pos = lm_first_reach(P, 0, pos, target, mono[row] != 0, 0);
  }
  states[2 * wk] = r.state;
  states[2 * wk + 1] = r.inc;
}

// Scores from the visits: mode 0 positional (visits / (1 / d^alpha + 1e-8), d = p - 3;
// landmark_walker.cu:305-341), 1 reachability (visits / the walkers able to reach p;
// :255-296), 2 reachability with 0.9 pass-through per landmark (absorbing form;
// landmark_absorbing_walker.cu:254-309).  [0, 4) scores 0.
__global__ void __launch_bounds__(256) k_lm_normalize(const int32_t* __restrict__ visits,
                                                      const int32_t* __restrict__ positions,
                                                      const int32_t* __restrict__ count, int n, int mode,
                                                      int walkers_per_source, float query_boost, float alpha,
                                                      float* __restrict__ scores) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n) return;
  if (idx < kMonSink) {
    scores[idx] = 0.f;
    return;
  }
  const int L = *count;
  const float v = (float)visits[idx];
  const float wps = (float)walkers_per_source;
  if (mode == 0) {
    const float distance = (float)(idx - kMonSink + 1);
    const float expected = 1.0f / powf(distance, alpha);
    scores[idx] = v / (expected + 1e-8f);
    return;
  }
  float reach = 0.f;
  if (mode == 1) {
    for (int l = 0; l < L; ++l)
      if (positions[l] > idx) reach += wps;
    if (n - 1 > idx) reach = fmaf(wps, query_boost, reach);
    scores[idx] = reach > 1e-8f ? v / reach : 0.f;
    return;
  }
  int after = 0;
  for (int l = 0; l < L; ++l)
    if (positions[l] > idx) ++after;
  if (after > 0) reach = wps * (float)after * 0.9f;
  if (n - 1 > idx) {
    float p;
    if (after == 0) p = 1.0f;
    else if (after <= 8) {
      const float decay[9] = {1.0f, 0.9f, 0.81f, 0.729f, 0.656f, 0.590f, 0.531f, 0.478f, 0.430f};
      p = decay[after];
    } else {
      p = fmaxf(0.1f, powf(0.9f, (float)after));
    }
    reach = fmaf(wps * query_boost, p, reach);
  }
  scores[idx] = reach > 1e-8f ? v / reach : v / ((float)(L + 1) * wps);
}

// ---- launchers -------------------------------------------------------------------------
cudaError_t launch_graph_update(const void* q, const void* keys, int dtype, int n, int D, int row, int top_k,
                                float* scores, int32_t* adj, float* weights, cudaStream_t st) {
  const int blocks = (n + 255) / 256;
  const size_t smem = (size_t)D * sizeof(float);
  if (dtype == CKV_FP16)
    k_graph_scores<__half><<<blocks, 256, smem, st>>>(static_cast<const __half*>(q), static_cast<const __half*>(keys),
                                                      n, D, scores);
  else if (dtype == CKV_BF16)
    k_graph_scores<__nv_bfloat16><<<blocks, 256, smem, st>>>(static_cast<const __nv_bfloat16*>(q),
                                                             static_cast<const __nv_bfloat16*>(keys), n, D, scores);
  else
    k_graph_scores<float><<<blocks, 256, smem, st>>>(static_cast<const float*>(q), static_cast<const float*>(keys), n,
                                                     D, scores);
  k_graph_topk<<<1, kMonThreads, 0, st>>>(scores, n, top_k, row, adj, weights);
  return cudaGetLastError();
}

cudaError_t launch_circuit_walk(const int32_t* adj, const float* w, int32_t* visits, uint64_t* states, int source,
                                int n, int top_k, int num_walkers, cudaStream_t st) {
  k_circuit_walk<<<(num_walkers + 255) / 256, 256, 0, st>>>(adj, w, visits, states, source, n, top_k, num_walkers);
  return cudaGetLastError();
}

cudaError_t launch_pcg_init(uint64_t* states, uint64_t seed, int num_walkers, cudaStream_t st) {
  k_pcg_init<<<(num_walkers + 255) / 256, 256, 0, st>>>(states, seed, num_walkers);
  return cudaGetLastError();
}

cudaError_t launch_spectral(const int32_t* adj, const float* w, int n, int top_k, int iters, float* v, float* vtmp,
                            cudaStream_t st) {
  k_spectral<<<1, kMonThreads, 0, st>>>(adj, w, n, top_k, iters, v, vtmp);
  return cudaGetLastError();
}

cudaError_t launch_combine(const int32_t* visits, float* spectral, float* walker, float* combined, int n,
                           cudaStream_t st) {
  k_combine<<<1, kMonThreads, 0, st>>>(visits, spectral, walker, combined, n);
  return cudaGetLastError();
}


size_t landmark_workspace_floats(int n) {
  const size_t stride = ((size_t)n + 1 + 3) & ~(size_t)3;
  return ((size_t)n + 3) / 4 * 4 + kLmRows * stride + 128;
}

cudaError_t launch_landmark_walk(const float* attn, int n, int current_idx, int mode, int num_landmarks,
                                 int walkers_per_source, float query_boost, int min_spacing, float alpha,
                                 int absorb_at_landmarks, uint64_t* states, int32_t* visits, float* scores,
                                 int32_t* positions, int32_t* count, float* ws, cudaStream_t st) {
  const int stride = (int)(((size_t)n + 1 + 3) & ~(size_t)3);
  float* h2o = ws;
  float* pref = ws + ((size_t)n + 3) / 4 * 4;
  int32_t* mono = reinterpret_cast<int32_t*>(pref + (size_t)kLmRows * stride);
  cudaError_t e = cudaMemsetAsync(visits, 0, (size_t)n * sizeof(int32_t), st);
  if (e != cudaSuccess) return e;
  {
    const size_t sm = (size_t)256 * kH2oCols * sizeof(float);
    const unsigned blocks = (unsigned)((n + kH2oCols - 1) / kH2oCols);
    if (n % 4 == 0 && (reinterpret_cast<uintptr_t>(attn) & 15u) == 0) {   // 16-byte row segments
      e = cudaFuncSetAttribute(k_lm_h2o<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
      if (e != cudaSuccess) return e;
      k_lm_h2o<true><<<blocks, 32 * kH2oWarps, sm, st>>>(attn, n, h2o);
    } else {
      e = cudaFuncSetAttribute(k_lm_h2o<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
      if (e != cudaSuccess) return e;
      k_lm_h2o<false><<<blocks, 32 * kH2oWarps, sm, st>>>(attn, n, h2o);
    }
  }
  k_lm_select<<<1, 1024, 0, st>>>(h2o, n, num_landmarks, min_spacing, positions, count);
  k_lm_prefix<<<3 + 2 * num_landmarks, 1024, 0, st>>>(attn, n, current_idx, h2o, positions, count, pref, stride,
                                                      mono);
  const long long walkers = (long long)(num_landmarks + 1) * walkers_per_source;
  if (walkers > 0)
    k_lm_walk<<<(unsigned)((walkers + 255) / 256), 256, 0, st>>>(pref, stride, mono, positions, count, n,
                                                                walkers_per_source, query_boost, mode == 2 ? 1 : 0,
                                                                absorb_at_landmarks, states, visits);
  k_lm_normalize<<<(n + 255) / 256, 256, 0, st>>>(visits, positions, count, n, mode, walkers_per_source, query_boost,
                                                  alpha, scores);
  return cudaGetLastError();
}

}  // namespace ckv
