// Influence walker of the legacy use_neumann=False path (reference:
// CircuitKV/csrc/kernels/influence_walker.cu:66-456, circuit_manager.cpp:1190-1311,
// called from PU:3244-3263).
//
// Walkers step along full_attn rows (row i: how much position i attends to j),
// sampling the next position among the non-sink positions [sink, pos] with
// probability proportional to max(A[pos, j], 1e-10)^(1/T): the first (1 - ratio) of
// the walkers use the base temperature, the rest the exploratory one; the first
// half start at the query, the others at a uniform position in [sink, query].
// Every step's landing position is counted; the counts are divided by
// sqrt(n - p + 1), normalised by their maximum and the sinks set to 1.
//
// The reference's extension is built with --use_fast_math, so its powf is the
// __powf intrinsic; the walkers here call the same intrinsic.  Generators:
//   * PCG-XSH-RR (M. E. O'Neill, "PCG: A Family of Simple Fast Space-Efficient
//     Statistically Good Algorithms for Random Number Generation", 2014; the
//     pcg32 seeding of its reference implementation), one state per walker, seeded
//     with (seed, walker) like the reference's init_rng_kernel
//     (circuit_walker.cu:157-171, the initialiser CircuitGraph uses), so that with the
//     same dense matrix the visit counts match the reference's walker;
//   * Philox4x64-10 (J. K. Salmon et al., "Parallel random numbers: as easy as
//     1, 2, 3", SC'11), counter based: key (seed, 0), counter (draw / 4, walker,
//     call, 0).
#include "ckv_common.cuh"
#include "ckv_walker.h"

namespace ckv {

// ---- generators --------------------------------------------------------------
struct Pcg {
  uint64_t state, inc;
};
CKV_DEV uint32_t pcg_next(Pcg& r) {
  const uint64_t old = r.state;
  r.state = old * 6364136223846793005ULL + r.inc;
  const uint32_t xs = (uint32_t)(((old >> 18u) ^ old) >> 27u);
  const uint32_t rot = (uint32_t)(old >> 59u);
  return (xs >> rot) | (xs << ((0u - rot) & 31u));
}
CKV_DEV void pcg_seed(Pcg& r, uint64_t initstate, uint64_t initseq) {
  r.state = 0u;
  r.inc = (initseq << 1u) | 1u;
  pcg_next(r);
  r.state += initstate;
  pcg_next(r);
}

CKV_DEV void philox4x64_10(uint64_t (&c)[4], uint64_t k0, uint64_t k1) {
  constexpr uint64_t kM0 = 0xD2E7470EE14C6C93ULL, kM1 = 0xCA5A826395121157ULL;
  constexpr uint64_t kW0 = 0x9E3779B97F4A7C15ULL, kW1 = 0xBB67AE8584CAA73BULL;
#pragma unroll
  for (int round = 0; round < 10; ++round) {
    if (round > 0) { k0 += kW0; k1 += kW1; }
    const uint64_t hi0 = __umul64hi(kM0, c[0]), lo0 = kM0 * c[0];
    const uint64_t hi1 = __umul64hi(kM1, c[2]), lo1 = kM1 * c[2];
    const uint64_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
    c[0] = n0; c[1] = lo1; c[2] = n2; c[3] = lo0;
  }
}

// A walker's uniform floats in [0, 1): 24 random bits times 2^-24.
struct WalkRng {
  int mode;
  Pcg pcg;
  uint64_t key, walker, call, draw;
  uint64_t blk[4];
  CKV_DEV float uniform() {
    uint32_t bits;
    if (mode == 1) {
      bits = pcg_next(pcg) >> 8;
    } else {
      const int lane = (int)(draw & 3u);
      if (lane == 0) {
        blk[0] = draw >> 2; blk[1] = walker; blk[2] = call; blk[3] = 0;
        philox4x64_10(blk, key, 0);
      }
      bits = (uint32_t)(blk[lane] >> 40);
      ++draw;
    }
    return (float)bits * (1.0f / 16777216.0f);
  }
};

CKV_DEV WalkRng walker_rng(const WalkArgs& a, int w) {
  WalkRng g;
  g.mode = a.rng_mode;
  g.key = a.seed;
  g.walker = (uint64_t)w;
  g.draw = 0;
  g.call = 0;
  const bool init = a.init_state || !a.rng_state;   // no state buffer: seeded on every call
  if (a.rng_mode == 1) {
    if (init) pcg_seed(g.pcg, a.seed, (uint64_t)w);
    else { g.pcg.state = a.rng_state[2 * w]; g.pcg.inc = a.rng_state[2 * w + 1]; }
  } else {
    g.call = init ? 0 : a.rng_state[0];
  }
  return g;
}

CKV_DEV void walker_store(const WalkArgs& a, int w, const WalkRng& g) {
  if (a.rng_mode == 1 && a.rng_state) { a.rng_state[2 * w] = g.pcg.state; a.rng_state[2 * w + 1] = g.pcg.inc; }
}

// Start position and inverse temperature of walker w (influence_walker.cu:92-121).
CKV_DEV int walker_start(const WalkArgs& a, int w, WalkRng& g, float* inv_t) {
  const int explore_start = (int)((1.0f - a.explore_ratio) * (float)a.num_walkers);
  *inv_t = (w >= explore_start) ? a.inv_explore_temp : a.inv_temp;
  if (w < a.num_walkers / 2) return a.current_idx;
  const int nvs = a.current_idx - a.sink + 1;
  if (nvs <= 0) return a.current_idx;
  int off = (int)(g.uniform() * (float)nvs);
  if (off >= nvs) off = nvs - 1;
  return a.sink + off;
}

// ---- dense walker -------------------------------------------------------------
__global__ void __launch_bounds__(256) k_walk_dense(const WalkArgs a) {
  const int w = blockIdx.x * blockDim.x + threadIdx.x;
  if (w >= a.num_walkers) return;
  WalkRng g = walker_rng(a, w);
  float it;
  int pos = walker_start(a, w, g, &it);
  for (int step = 0; step < a.max_steps; ++step) {
    if (pos < a.sink) break;
    const float* row = a.attn + (size_t)pos * a.n;
    float sum = 0.f;
    for (int j = a.sink; j <= pos; ++j) sum += __powf(fmaxf(row[j], 1e-10f), it);
    if (sum < 1e-10f) break;
    const float r = g.uniform() * sum;
    float cs = 0.f;
    int next = a.sink;
    for (int j = a.sink; j <= pos; ++j) {
      cs += __powf(fmaxf(row[j], 1e-10f), it);
      next = j;
      if (r < cs) break;
    }
    atomicAdd(&a.visits[next], 1.0f);
    pos = next;
  }
  walker_store(a, w, g);
}

// ---- dense walker, one warp per walker (Philox mode) ----------------------------
// The same walk with the row work spread over the warp: lanes read 32 consecutive weights
// at a time (coalesced), the row total is a warp sum, and the sampled position is found by
// a warp prefix scan per 32-position block with a ballot on the first crossing.  The
// random draws are the thread-per-walker kernel's (lane 0 holds the counter-based
// generator, so the draw sequence of each walker is the same); only the order of the fp32
// additions differs, so a step can land one position over where a running sum crosses the
// target within its rounding.  PCG mode keeps k_walk_dense: there the visit counts must be
// the reference's bit for bit, which needs its sequential sums.
constexpr int kWalkWarps = 8;
__global__ void __launch_bounds__(32 * kWalkWarps) k_walk_dense_warp(const WalkArgs a) {
  const int lane = threadIdx.x & 31;
  const int w = blockIdx.x * kWalkWarps + (threadIdx.x >> 5);
  if (w >= a.num_walkers) return;   // warp-uniform
  WalkRng g = walker_rng(a, w);
  float it = 0.f;
  int pos = 0;
  if (lane == 0) pos = walker_start(a, w, g, &it);
  pos = __shfl_sync(0xffffffffu, pos, 0);
  it = __shfl_sync(0xffffffffu, it, 0);
  for (int step = 0; step < a.max_steps; ++step) {
    if (pos < a.sink) break;
    const float* row = a.attn + (size_t)pos * a.n;
    float part = 0.f;
    for (int j = a.sink + lane; j <= pos; j += 32) part += __powf(fmaxf(__ldg(row + j), 1e-10f), it);
    const float sum = warp_sum(part);
    if (sum < 1e-10f) break;
    float r = 0.f;
    if (lane == 0) r = g.uniform() * sum;
    r = __shfl_sync(0xffffffffu, r, 0);
    float base = 0.f;
    int next = pos;   // no crossing within rounding: the last position, as the scan ends there
    for (int j0 = a.sink; j0 <= pos; j0 += 32) {
      const int j = j0 + lane;
      float v = j <= pos ? __powf(fmaxf(__ldg(row + j), 1e-10f), it) : 0.f;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {   // inclusive prefix sum over the block
        const float t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
      }
      const unsigned hit = __ballot_sync(0xffffffffu, j <= pos && r < base + v);
      if (hit) { next = j0 + __ffs(hit) - 1; break; }
      base += __shfl_sync(0xffffffffu, v, 31);
    }
    if (lane == 0) atomicAdd(&a.visits[next], 1.0f);
    pos = next;
  }
  if (lane == 0) walker_store(a, w, g);
}

// ---- structured walker --------------------------------------------------------
// Prefix row pos < n_p: A[pos, j] = h[j] * cinv[pos] for j < pos, 0 at j = pos, so the
// weights are h[j]^(1/T) * cinv^(1/T) (the 1e-10 floor never binds: h >= 1e-6 and the
// row denominators stay far below 1e4) plus 1e-10^(1/T) at j = pos: the sampled
// position comes from a binary search on the prefix sums of h^(1/T).  Window row
// pos = n_p + r: the pooled row r, scanned as in the dense walker.
__global__ void __launch_bounds__(256) k_walk_rows(const WalkArgs a) {
  const int w = blockIdx.x * blockDim.x + threadIdx.x;
  if (w >= a.num_walkers) return;
  WalkRng g = walker_rng(a, w);
  float it;
  int pos = walker_start(a, w, g, &it);
  const int n_p = a.n - a.W;
  const double* pre = a.pre + (it == a.inv_temp ? 0 : (size_t)(n_p + 1));
  const double wfloor = (double)__powf(1e-10f, it);
  for (int step = 0; step < a.max_steps; ++step) {
    if (pos < a.sink) break;
    int next = a.sink;
    if (pos < n_p) {
      const double ct = (double)__powf(a.cinv[pos], it);
      const double body = pos > a.sink ? ct * (pre[pos] - pre[a.sink]) : 0.0;
      const double total = body + wfloor;
      if (total < 1e-10) break;
      const double r = (double)g.uniform() * total;
      if (r >= body) {
        next = pos;
      } else {
        const double target = pre[a.sink] + r / ct;   // first j with pre[j + 1] > target
        int lo = a.sink, hi = pos - 1;
        while (lo < hi) {
          const int mid = (lo + hi) >> 1;
          if (pre[mid + 1] > target) hi = mid;
          else lo = mid + 1;
        }
        next = lo;
      }
    } else {
      const float* row = a.rows + (size_t)(pos - n_p) * a.ld;
      float sum = 0.f;
      for (int j = a.sink; j <= pos; ++j) sum += __powf(fmaxf(row[j], 1e-10f), it);
      if (sum < 1e-10f) break;
      const float r = g.uniform() * sum;
      float cs = 0.f;
      for (int j = a.sink; j <= pos; ++j) {
        cs += __powf(fmaxf(row[j], 1e-10f), it);
        next = j;
        if (r < cs) break;
      }
    }
    atomicAdd(&a.visits[next], 1.0f);
    pos = next;
  }
  walker_store(a, w, g);
}

// h = max(column sums of the pooled rows over the prefix, 1e-6), cinv[i] = 1 / (C[i-1] +
// 1e-8) with C the running sum (accumulated in double), the prefix sums of h^(1/T) for
// both temperatures, and the column sums of full_attn (PU:3253: window rows plus
// h[j] * sum_{i>j} cinv[i]).  One CTA.
__global__ void __launch_bounds__(1024) k_walk_prep(const WalkArgs a, float* hbuf, float* cinv, double* pre) {
  float* h2o = a.h2o;
  const int n = a.n, n_p = n - a.W;
  __shared__ double sc[32];
  __shared__ double carry_c, carry_a, carry_b;
  if (threadIdx.x == 0) { carry_c = 0.0; carry_a = 0.0; carry_b = 0.0; }
  __syncthreads();
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  auto block_scan = [&](double v, double* tot) {   // inclusive scan in double
    double x = v;
    for (int o = 1; o < 32; o <<= 1) { const double y = __shfl_up_sync(0xffffffffu, x, o); if (lane >= o) x += y; }
    if (lane == 31) sc[wid] = x;
    __syncthreads();
    if (wid == 0) {
      double s = sc[lane];
      for (int o = 1; o < 32; o <<= 1) { const double y = __shfl_up_sync(0xffffffffu, s, o); if (lane >= o) s += y; }
      sc[lane] = s;
    }
    __syncthreads();
    const double r = x + (wid > 0 ? sc[wid - 1] : 0.0);
    *tot = sc[31];
    __syncthreads();
    return r;
  };
  for (int base = 0; base < n_p; base += blockDim.x) {
    const int j = base + threadIdx.x;
    float hj = 0.f;
    if (j < n_p) {
      float c = 0.f;
      for (int r = 0; r < a.W; ++r) c += a.rows[(size_t)r * a.ld + j];
      hj = fmaxf(c, 1e-6f);
      hbuf[j] = hj;
    }
    double tc, ta, tb;
    const double ic = block_scan((double)hj, &tc);                              // C[j] (inclusive)
    const double ia = block_scan(j < n_p ? (double)__powf(hj, a.inv_temp) : 0.0, &ta);
    const double ib = block_scan(j < n_p ? (double)__powf(hj, a.inv_explore_temp) : 0.0, &tb);
    if (j < n_p) {
      const double cprev = carry_c + ic - (double)hj;                           // C[j - 1]
      cinv[j] = j >= 1 ? 1.0f / ((float)cprev + 1e-8f) : 0.f;
      pre[j + 1] = carry_a + ia;
      pre[(size_t)(n_p + 1) + j + 1] = carry_b + ib;
    }
    __syncthreads();
    if (threadIdx.x == 0) { carry_c += tc; carry_a += ta; carry_b += tb; }
    __syncthreads();
  }
  if (threadIdx.x == 0) { pre[0] = 0.0; pre[(size_t)(n_p + 1)] = 0.0; }
  __syncthreads();
  // H2O: full_attn column sums = window rows + h[j] * sum_{i = j+1}^{n_p-1} cinv[i]
  double rcarry = 0.0;
  const int ntile = (n_p + blockDim.x - 1) / blockDim.x;
  for (int t = ntile - 1; t >= 0; --t) {
    const int i = t * blockDim.x + threadIdx.x;
    const double v = i < n_p ? (double)cinv[i] : 0.0;
    double tot;
    const double incl = block_scan(v, &tot);
    const double after = rcarry + (tot - incl);   // sum over i' > i in [0, n_p)
    if (i < n_p) {
      float c = 0.f;
      for (int r = 0; r < a.W; ++r) c += a.rows[(size_t)r * a.ld + i];
      h2o[i] = c + hbuf[i] * (float)after;
    }
    rcarry += tot;
  }
  for (int j = n_p + threadIdx.x; j < n; j += blockDim.x) {
    float c = 0.f;
    for (int r = 0; r < a.W; ++r) c += a.rows[(size_t)r * a.ld + j];
    h2o[j] = c;
  }
}

// visits / sqrt(n - p + 1), divided by the maximum over [sink, min(n, 256 * 256)) (the
// reference reduces at most 256 blocks of 256), sinks = 1 (influence_walker.cu:296-456).
__global__ void __launch_bounds__(1024) k_walk_normalize(const WalkArgs a) {
  __shared__ float red[32];
  const int n = a.n, s = a.sink;
  const int nb = min(256, (n + 255) / 256);
  const int lim = min(n, nb * 256);
  float mx = 0.f;
  for (int p = threadIdx.x; p < n; p += blockDim.x) {
    const float adj = p < s ? 0.f : a.visits[p] / sqrtf((float)(n - p + 1));
    a.scores[p] = adj;
    if (p >= s && p < lim) mx = fmaxf(mx, adj);
  }
  mx = block_reduce<true>(mx, red);
  for (int p = threadIdx.x; p < n; p += blockDim.x)
    a.scores[p] = p < s ? 1.f : (mx > 1e-10f ? a.scores[p] / mx : 0.f);
  if (threadIdx.x == 0 && a.rng_mode == 0 && a.rng_state)   // Philox: next call's counter
    a.rng_state[0] = (a.init_state ? 0 : a.rng_state[0]) + 1;
}

cudaError_t launch_walk_dense(const WalkArgs& a, cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(a.visits, 0, (size_t)a.n * sizeof(float), st);
  if (e != cudaSuccess) return e;
  if (a.rng_mode == 0)
    k_walk_dense_warp<<<(a.num_walkers + kWalkWarps - 1) / kWalkWarps, 32 * kWalkWarps, 0, st>>>(a);
  else
    k_walk_dense<<<(a.num_walkers + 255) / 256, 256, 0, st>>>(a);
  k_walk_normalize<<<1, 1024, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_walk_prep(const WalkArgs& a, float* hbuf, float* cinv, double* pre, cudaStream_t st) {
  k_walk_prep<<<1, 1024, 0, st>>>(a, hbuf, cinv, pre);
  return cudaGetLastError();
}

cudaError_t launch_walk_rows(const WalkArgs& a, cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(a.visits, 0, (size_t)a.n * sizeof(float), st);
  if (e != cudaSuccess) return e;
  k_walk_rows<<<(a.num_walkers + 255) / 256, 256, 0, st>>>(a);
  k_walk_normalize<<<1, 1024, 0, st>>>(a);
  return cudaGetLastError();
}

__global__ void k_rng_fill(int mode, uint64_t seed, uint64_t stream, int count, uint64_t* out) {
  if (mode == 1) {   // one sequential pcg32 stream
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    Pcg r;
    pcg_seed(r, seed, stream);
    for (int i = 0; i < count; ++i) out[i] = pcg_next(r);
    return;
  }
  const int b = blockIdx.x * blockDim.x + threadIdx.x;   // one Philox block of 4 outputs
  if (4 * b >= count) return;
  uint64_t c[4] = {(uint64_t)b, stream, 0, 0};
  philox4x64_10(c, seed, 0);
  for (int l = 0; l < 4 && 4 * b + l < count; ++l) out[4 * b + l] = c[l];
}

cudaError_t launch_rng_fill(int mode, uint64_t seed, uint64_t stream, int count, uint64_t* out,
                            cudaStream_t st) {
  const int blocks = mode == 1 ? 1 : ((count + 3) / 4 + 255) / 256;
  k_rng_fill<<<blocks > 0 ? blocks : 1, mode == 1 ? 32 : 256, 0, st>>>(mode, seed, stream, count, out);
  return cudaGetLastError();
}

}  // namespace ckv
