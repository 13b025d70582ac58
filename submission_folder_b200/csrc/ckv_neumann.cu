// Structured absorbing-chain (Neumann) solve of the CircuitKV prefill path
// (reference: pyramidkv_utils.py PU:2060-2206 dual chains, PU:1939-2058 single
// chain) without the n x n matrix the reference materialises (PU:3003-3034).
//
// Prefix rows of the transition matrix have rank-one structure:
// P[i, j] = g[j] / G[i-1] for j < i < n - W (g = clamped column sums of the
// pooled window rows raised to 1/T, G = cumsum g).  With c_i = 1 / G[i-1] one
// Neumann step on the prefix is x_{k+1}[j] = gamma g_j S_k[j] + b_k[j], where
// S_k[j] = sum_{i > j} c_i x_k[i] and b_k = gamma (window rows)^T (y_k / rowsum)
// (the window chain y_k is the W x W part, computed by the pooling pass).
// All K steps are carried together in ONE reverse sweep over positions: the
// per-position update of the carry S = (S_0..S_{K-1}) is the affine map
//     S' = (I + c_j gamma g_j N) S + c_j (x0_j, b_0[j], ..., b_{K-2}[j]),
// N the shift; these maps are polynomials in N, so a chunk of positions
// composes into one (K coefficients, K offsets) map and chunks combine in a
// tree.  k_sweep_chunks builds b_k, c, g and the chunk maps; k_sweep_apply
// folds the maps of all later chunks into its incoming carry, scans its own
// positions and writes the running sums of x_0..x_K plus per-chunk maxima (the
// early stop of PU:2183 needs the max of every term).
#include "ckv_common.cuh"
#include "ckv_neumann.h"

namespace ckv {

void stage_mark(cudaStream_t st);

template <int KM> struct Map {
  float a[KM];   // polynomial coefficients in the shift N (a[0] == 1)
  float u[KM];   // offset
};

template <int KM> CKV_DEV void map_identity(Map<KM>& m) {
#pragma unroll
  for (int i = 0; i < KM; ++i) { m.a[i] = (i == 0) ? 1.f : 0.f; m.u[i] = 0.f; }
}

// (L o R)(S) = L(R(S)): R is applied first (R covers the higher positions).
template <int KM> CKV_DEV Map<KM> compose(const Map<KM>& L, const Map<KM>& R) {
  Map<KM> o;
#pragma unroll
  for (int m = 0; m < KM; ++m) {
    float sa = 0.f, su = L.u[m];
#pragma unroll
    for (int i = 0; i <= m; ++i) {
      sa = fmaf(L.a[i], R.a[m - i], sa);
      su = fmaf(L.a[i], R.u[m - i], su);
    }
    o.a[m] = sa;
    o.u[m] = su;
  }
  return o;
}

template <int KM> CKV_DEV void apply(const Map<KM>& M, const float* S, float* out) {
#pragma unroll
  for (int k = 0; k < KM; ++k) {
    float s = M.u[k];
#pragma unroll
    for (int i = 0; i <= k; ++i) s = fmaf(M.a[i], S[k - i], s);
    out[k] = s;
  }
}

// Maps live in shared memory with a stride of 2*KM+1 floats (odd: no bank conflicts).
template <int KM> __host__ __device__ constexpr int map_stride() { return 2 * KM + 1; }

template <int KM> CKV_DEV void store_map(float* dst, const Map<KM>& m) {
#pragma unroll
  for (int i = 0; i < KM; ++i) { dst[i] = m.a[i]; dst[KM + i] = m.u[i]; }
}
template <int KM> CKV_DEV Map<KM> load_map(const float* src) {
  Map<KM> m;
#pragma unroll
  for (int i = 0; i < KM; ++i) { m.a[i] = src[i]; m.u[i] = src[KM + i]; }
  return m;
}

// Exclusive block scan of floats (sum); returns the exclusive prefix, *total = block sum.
__device__ float block_exclusive_scan_f(float v, float* scratch, float* total) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  float x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  __syncthreads();
  if (lane == 31) scratch[wid] = x;
  __syncthreads();
  if (wid == 0) {
    float s = (lane < nw) ? scratch[lane] : 0.f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    if (lane < nw) scratch[lane] = s;
  }
  __syncthreads();
  const float base = (wid > 0) ? scratch[wid - 1] : 0.f;
  const float t = scratch[nw - 1];
  __syncthreads();
  if (total) *total = t;
  return base + x - v;
}

// Which pooled rows chain `ch` reads (the HI chain reuses the QI rows when the
// reference's attention_for_hi is None, PU:2135-2146).
CKV_DEV int row_source(const Plan& pl, int ch) { return (ch == 1 && pl.hi_rows) ? 1 : 0; }

// Per-position map of position j (identity outside the transient prefix).
template <int KM>
CKV_DEV Map<KM> position_map(const Plan& pl, int ch, int j, float c, float g, const float* bk,
                             float gamma, float x0) {
  Map<KM> m;
  map_identity(m);
  if (j < pl.s || j >= pl.n_p) return m;
  if (KM > 1) m.a[1] = c * gamma * g;
  m.u[0] = c * x0;
#pragma unroll
  for (int k = 1; k < KM; ++k) m.u[k] = (k < pl.K) ? c * bk[k - 1] : 0.f;
  return m;
}

CKV_DEV float start_value(const Plan& pl, int ch, int j) {
  // HI chain starts uniform over the transient states, QI from the query one-hot (a window position)
  return (ch == 1 && j >= pl.s && j < pl.n_p) ? 1.0f / (float)(pl.n - pl.s) : 0.f;
}

// ---------------------------------------------------------------------------
// kernel 1: b_k, c, g and the chunk maps
// ---------------------------------------------------------------------------
template <int KM>
__global__ void __launch_bounds__(kScanChunk) k_sweep_chunks(const Plan pl, const ckv_params prm,
                                                             char* ws) {
  extern __shared__ __align__(16) float sm[];
  const int chunk = blockIdx.x, ch = blockIdx.y;
  const int src = row_source(pl, ch);
  const int j = chunk * kScanChunk + threadIdx.x;
  const int K = pl.K;
  const bool tempered = prm.neumann_temperature != 1.0f && prm.neumann_temperature > 0.f;
  const float invT = tempered ? 1.0f / prm.neumann_temperature : 1.0f;
  const float gamma = prm.neumann_gamma;
  const float* rows = reinterpret_cast<const float*>(ws + (src ? pl.off_rows_hi : pl.off_rows_qi));
  const float* colsum = reinterpret_cast<const float*>(ws + pl.off_colsum) + (size_t)src * pl.n_pad;
  const float* gtile = reinterpret_cast<const float*>(ws + pl.off_gtile) + (size_t)src * pl.ncol_tiles * 8;
  const float* wk = reinterpret_cast<const float*>(ws + pl.off_wk) + (size_t)ch * K * pl.W;
  float* bk_out = reinterpret_cast<float*>(ws + pl.off_bk) + (size_t)ch * K * pl.n_p;
  float2* cg_out = reinterpret_cast<float2*>(ws + pl.off_cg) + (size_t)ch * pl.n_p;
  float* agg = reinterpret_cast<float*>(ws + pl.off_agg) + ((size_t)ch * pl.nscan) * 2 * KM;

  float* sW = sm;                            // [K][W]
  float* sMaps = sW + K * pl.W;              // [kScanChunk][2*KM+1]
  float* scratch = sMaps + kScanChunk * map_stride<KM>();   // 32 floats
  for (int i = threadIdx.x; i < K * pl.W; i += blockDim.x) sW[i] = wk[i];

  // G offset of this chunk: sum of g over all earlier positions (partial totals of
  // g_slice columns each)
  const int tiles_before = (chunk * kScanChunk) / pl.g_slice;
  float off = 0.f;
  for (int t = threadIdx.x; t < tiles_before; t += blockDim.x) off += gtile[t];
  off = block_reduce<false>(off, scratch);

  float g = 0.f;
  if (j < pl.n_p) {
    g = fmaxf(colsum[j], 1e-6f);
    if (tempered) g = powf(g, invT);
  }
  const float excl = block_exclusive_scan_f(g, scratch, nullptr);
  const float Gprev = off + excl;              // G[j-1]
  const float c = (j >= 1 && Gprev > 0.f) ? 1.0f / Gprev : 0.f;

  float bk[KM];
#pragma unroll
  for (int k = 0; k < KM; ++k) bk[k] = 0.f;
  if (j < pl.n_p && j >= pl.s) {
    // 16 independent row loads in flight per batch (the rows are L2-resident)
    for (int r0 = 0; r0 < pl.W; r0 += 16) {
      float v[16];
#pragma unroll
      for (int u = 0; u < 16; ++u) v[u] = __ldcg(rows + (size_t)(r0 + u) * pl.n_pad + j);
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        float x = v[u];
        if (tempered) x = x > 0.f ? powf(x, invT) : 0.f;
#pragma unroll
        for (int k = 0; k < KM; ++k)
          if (k < K) bk[k] = fmaf(x, sW[k * pl.W + r0 + u], bk[k]);
      }
    }
  }
  if (j < pl.n_p) {
#pragma unroll
    for (int k = 0; k < KM; ++k)
      if (k < K) bk_out[(size_t)k * pl.n_p + j] = bk[k];
    cg_out[j] = make_float2(c, g);
  }
  Map<KM> m = position_map<KM>(pl, ch, j, c, g, bk, gamma, start_value(pl, ch, j));
  store_map(sMaps + threadIdx.x * map_stride<KM>(), m);
  __syncthreads();
  for (int d = 1; d < kScanChunk; d <<= 1) {
    if ((threadIdx.x % (2 * d)) == 0) {
      const Map<KM> L = load_map<KM>(sMaps + threadIdx.x * map_stride<KM>());
      const Map<KM> R = load_map<KM>(sMaps + (threadIdx.x + d) * map_stride<KM>());
      store_map(sMaps + threadIdx.x * map_stride<KM>(), compose(L, R));
    }
    __syncthreads();
  }
  if (threadIdx.x < 2 * KM) agg[(size_t)chunk * 2 * KM + threadIdx.x] = sMaps[threadIdx.x];
}

// ---------------------------------------------------------------------------
// kernel 2: incoming carry, in-chunk suffix scan, terms x_0..x_K
// ---------------------------------------------------------------------------
template <int KM>
__global__ void __launch_bounds__(kScanChunk) k_sweep_apply(const Plan pl, const ckv_params prm,
                                                            char* ws) {
  extern __shared__ __align__(16) float sm[];
  const int chunk = blockIdx.x, ch = blockIdx.y;
  const int j = chunk * kScanChunk + threadIdx.x;
  const int K = pl.K;
  const float gamma = prm.neumann_gamma;
  const float* agg = reinterpret_cast<const float*>(ws + pl.off_agg) + ((size_t)ch * pl.nscan) * 2 * KM;
  const float* bk_in = reinterpret_cast<const float*>(ws + pl.off_bk) + (size_t)ch * K * pl.n_p;
  const float2* cg_in = reinterpret_cast<const float2*>(ws + pl.off_cg) + (size_t)ch * pl.n_p;
  float* cum = reinterpret_cast<float*>(ws + pl.off_cum) + (size_t)ch * (K + 1) * pl.n_p;
  float* cmax = reinterpret_cast<float*>(ws + pl.off_cmax) + ((size_t)ch * pl.nscan + chunk) * (kMaxIters + 1);

  float* bufA = sm;                               // [kScanChunk][2*KM+1]
  float* bufB = bufA + kScanChunk * map_stride<KM>();   // [kScanChunk][2*KM+1]
  float* scratch = bufB + kScanChunk * map_stride<KM>();   // (kScanChunk/32) * (kMaxIters+1) floats

  // 1) fold the maps of all later chunks (tree over at most kScanChunk maps per round)
  float Sin[KM];
#pragma unroll
  for (int k = 0; k < KM; ++k) Sin[k] = 0.f;
  {
    // process later chunks from the far end in rounds of kScanChunk maps
    Map<KM> acc;   // composition of the chunks already folded (they are higher)
    map_identity(acc);
    const int first = chunk + 1, last = pl.nscan;   // [first, last)
    for (int hi = last; hi > first; hi -= kScanChunk) {
      const int lo = max(first, hi - kScanChunk);
      const int cnt = hi - lo;
      Map<KM> m;
      if ((int)threadIdx.x < cnt) m = load_map<KM>(agg + (size_t)(lo + threadIdx.x) * 2 * KM);
      else map_identity(m);
      store_map(bufA + threadIdx.x * map_stride<KM>(), m);
      __syncthreads();
      for (int d = 1; d < kScanChunk; d <<= 1) {
        if ((threadIdx.x % (2 * d)) == 0) {
          const Map<KM> L = load_map<KM>(bufA + threadIdx.x * map_stride<KM>());
          const Map<KM> R = load_map<KM>(bufA + (threadIdx.x + d) * map_stride<KM>());
          store_map(bufA + threadIdx.x * map_stride<KM>(), compose(L, R));
        }
        __syncthreads();
      }
      acc = compose(load_map<KM>(bufA), acc);
      __syncthreads();
    }
    const float zero[KM] = {};
    apply(acc, zero, Sin);
  }

  // 2) per-position maps of this chunk, inclusive suffix scan (Hillis-Steele)
  float c = 0.f, g = 0.f, bk[KM];
#pragma unroll
  for (int k = 0; k < KM; ++k) bk[k] = 0.f;
  if (j < pl.n_p) {
    const float2 v = cg_in[j];
    c = v.x; g = v.y;
#pragma unroll
    for (int k = 0; k < KM; ++k)
      if (k < K) bk[k] = bk_in[(size_t)k * pl.n_p + j];
  }
  const float x0 = start_value(pl, ch, j);
  store_map(bufA + threadIdx.x * map_stride<KM>(), position_map<KM>(pl, ch, j, c, g, bk, gamma, x0));
  __syncthreads();
  float* src = bufA;
  float* dst = bufB;
  for (int d = 1; d < kScanChunk; d <<= 1) {
    Map<KM> m = load_map<KM>(src + threadIdx.x * map_stride<KM>());
    if (threadIdx.x + d < kScanChunk) m = compose(m, load_map<KM>(src + (threadIdx.x + d) * map_stride<KM>()));
    store_map(dst + threadIdx.x * map_stride<KM>(), m);
    __syncthreads();
    float* t = src; src = dst; dst = t;
  }
  // carry after all positions > j
  float S[KM];
  if (threadIdx.x + 1 < kScanChunk) apply(load_map<KM>(src + (threadIdx.x + 1) * map_stride<KM>()), Sin, S);
  else {
#pragma unroll
    for (int k = 0; k < KM; ++k) S[k] = Sin[k];
  }

  // 3) terms x_0..x_K of this position, running sums and per-chunk maxima
  const bool valid = (j >= pl.s && j < pl.n_p);
  float x = x0, run = x0;
  float mx[kMaxIters + 1];
#pragma unroll
  for (int k = 0; k <= kMaxIters; ++k) mx[k] = 0.f;
  if (valid) cum[j] = run;
#pragma unroll
  for (int k = 0; k < KM; ++k) {
    if (k < K) {
      x = fmaf(gamma * g, S[k], bk[k]);
      run += x;
      if (valid) {
        cum[(size_t)(k + 1) * pl.n_p + j] = run;
        mx[k + 1] = fabsf(x);
      }
    }
  }
  // block max of every term index: warp shuffles, one barrier
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int k = 1; k <= KM; ++k) {
    float v = (valid && k <= K) ? mx[k] : 0.f;
    v = warp_max(v);
    if (lane == 0) scratch[wid * (kMaxIters + 1) + k] = v;
  }
  __syncthreads();
  if (threadIdx.x >= 1 && threadIdx.x <= K) {
    float v = 0.f;
    for (int w = 0; w < kScanChunk / 32; ++w) v = fmaxf(v, scratch[w * (kMaxIters + 1) + threadIdx.x]);
    cmax[threadIdx.x] = v;
  }
}

template <int KM>
static cudaError_t launch_sweep_t(const Plan& pl, const ckv_params& prm, char* ws, cudaStream_t st) {
  const size_t s1 = sizeof(float) * ((size_t)pl.K * pl.W + kScanChunk * map_stride<KM>() + 64);
  const size_t s2 = sizeof(float) * (2 * (size_t)kScanChunk * map_stride<KM>() + (kScanChunk / 32) * (kMaxIters + 1) + 64);
  {
    cudaError_t e = ensure_dynamic_smem((const void*)k_sweep_chunks<KM>, s1);
    if (e == cudaSuccess) e = ensure_dynamic_smem((const void*)k_sweep_apply<KM>, s2);
    if (e != cudaSuccess) return e;
  }
  const dim3 grid(pl.nscan, pl.nchains);
  k_sweep_chunks<KM><<<grid, kScanChunk, s1, st>>>(pl, prm, ws);
  stage_mark(st);
  k_sweep_apply<KM><<<grid, kScanChunk, s2, st>>>(pl, prm, ws);
  return cudaGetLastError();
}

cudaError_t launch_sweep(const Plan& pl, const ckv_params& prm, char* ws, cudaStream_t st) {
  if (pl.n_p <= pl.s) return cudaSuccess;   // no transient prefix
  if (pl.K <= 4) return launch_sweep_t<4>(pl, prm, ws, st);
  if (pl.K <= 8) return launch_sweep_t<8>(pl, prm, ws, st);
  if (pl.K <= 10) return launch_sweep_t<10>(pl, prm, ws, st);
  if (pl.K <= 12) return launch_sweep_t<12>(pl, prm, ws, st);
  return launch_sweep_t<16>(pl, prm, ws, st);
}

}  // namespace ckv
