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

}  // namespace ckv
