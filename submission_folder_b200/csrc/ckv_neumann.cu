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
// N the shift; these maps are polynomials in N, so a run of positions
// composes into one (K coefficients, K offsets) map.  Applying or composing a
// single position's map costs O(K) (it is 1 + alpha N plus an offset); two
// composed runs cost O(K^2).  So each thread sweeps a run of kSweepRun
// consecutive positions in O(K) per position, and only run / warp / chunk
// aggregates are composed densely (warp shuffles, then across warps).
// k_sweep_chunks builds b_k, c, g and each chunk's map; its last CTA per chain
// composes the chunk maps from the top and stores every chunk's incoming carry.
// k_sweep_apply turns that carry into each run's incoming carry, sweeps its
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

CKV_DEV float start_value(const Plan& pl, int ch, int j) {
  // HI chain starts uniform over the transient states, QI from the query one-hot (a window position)
  return (ch == 1 && j >= pl.s && j < pl.n_p) ? 1.0f / (float)(pl.n - pl.s) : 0.f;
}

// Position j's map composed onto M (M covers higher positions and is applied first):
// a <- (1 + alpha N) a, u <- (1 + alpha N) u + u_j, truncated at degree KM - 1.
template <int KM>
CKV_DEV void push_position(Map<KM>& M, float alpha, const float* uj) {
#pragma unroll
  for (int k = KM - 1; k >= 1; --k) {
    M.a[k] = fmaf(alpha, M.a[k - 1], M.a[k]);
    M.u[k] = fmaf(alpha, M.u[k - 1], M.u[k]) + uj[k];
  }
  M.u[0] += uj[0];
}

// Inclusive suffix composition within a warp: lane l ends with A_l o A_{l+1} o ... o A_31.
template <int KM>
CKV_DEV Map<KM> warp_suffix_compose(Map<KM> A) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    Map<KM> B;
#pragma unroll
    for (int i = 0; i < KM; ++i) {
      B.a[i] = __shfl_down_sync(0xffffffffu, A.a[i], d);
      B.u[i] = __shfl_down_sync(0xffffffffu, A.u[i], d);
    }
    if (lane + d < 32) A = compose(A, B);
  }
  return A;
}

// The map of lane l + 1's inclusive suffix (identity for the last lane).
template <int KM>
CKV_DEV Map<KM> next_lane_map(const Map<KM>& A) {
  Map<KM> B;
#pragma unroll
  for (int i = 0; i < KM; ++i) {
    B.a[i] = __shfl_down_sync(0xffffffffu, A.a[i], 1);
    B.u[i] = __shfl_down_sync(0xffffffffu, A.u[i], 1);
  }
  if ((threadIdx.x & 31) == 31) map_identity(B);
  return B;
}

// c, g and the per-position offsets u_j of thread's run (positions j0 .. j0 + kSweepRun - 1).
static_assert(kSweepRun == 4, "the row loads below read one float4 per run");

struct RunIn {
  float c[kSweepRun], g[kSweepRun];
};

// ---------------------------------------------------------------------------
// kernel 1: b_k, c, g and the chunk maps; the last CTA of a chain stores the
// incoming carry of every chunk
// ---------------------------------------------------------------------------
template <int KM>
__global__ void __launch_bounds__(kSweepThreads) k_sweep_chunks(const Plan pl, const ckv_params prm,
                                                                char* ws) {
  constexpr int KW = (KM + 3) / 4 * 4;       // w_k padded to whole float4s
  extern __shared__ __align__(16) float sm[];
  const int chunk = blockIdx.x, ch = blockIdx.y;
  const int src = row_source(pl, ch);
  const int K = pl.K;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int j0 = chunk * kScanChunk + threadIdx.x * kSweepRun;
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

  float* sW = sm;                                        // [W][KW]: w_k of window row r
  float* sWarp = sW + pl.W * KW;                         // [8 warps][2*KM+1]
  float* scratch = sWarp + (kSweepThreads / 32) * map_stride<KM>();   // 32 floats
  for (int i = threadIdx.x; i < pl.W * KW; i += blockDim.x) {
    const int r = i / KW, k = i % KW;
    sW[i] = k < K ? wk[k * pl.W + r] : 0.f;
  }

  // G offset of this chunk: sum of g over all earlier positions (partial totals of
  // g_slice columns each)
  const int tiles_before = (chunk * kScanChunk) / pl.g_slice;
  float off = 0.f;
  for (int t = threadIdx.x; t < tiles_before; t += blockDim.x) off += gtile[t];
  off = block_reduce<false>(off, scratch);

  RunIn ri;
  float run_tot = 0.f, pre[kSweepRun];
#pragma unroll
  for (int p = 0; p < kSweepRun; ++p) {
    const int j = j0 + p;
    float g = 0.f;
    if (j < pl.n_p) {
      g = fmaxf(colsum[j], 1e-6f);
      if (tempered) g = powf(g, invT);
    }
    ri.g[p] = g;
    pre[p] = run_tot;
    run_tot += g;
  }
  const float excl = block_exclusive_scan_f(run_tot, scratch, nullptr);
#pragma unroll
  for (int p = 0; p < kSweepRun; ++p) {
    const int j = j0 + p;
    const float Gprev = off + excl + pre[p];           // G[j-1]
    ri.c[p] = (j >= 1 && Gprev > 0.f) ? 1.0f / Gprev : 0.f;
  }
  __syncthreads();   // sW is complete

  // b_k[j] = sum_r rows[r][j] w_k[r] for the run (rows are L2-resident)
  float bk[kSweepRun][KM];
#pragma unroll
  for (int p = 0; p < kSweepRun; ++p)
#pragma unroll
    for (int k = 0; k < KM; ++k) bk[p][k] = 0.f;
  if (j0 < pl.n_p && j0 + kSweepRun > pl.s) {
    const bool full = j0 + kSweepRun <= pl.n_p;
    constexpr int kRowBatch = 8;   // rows in flight per thread (W is a multiple of 8)
    for (int r0 = 0; r0 < pl.W; r0 += kRowBatch) {
      float4 xb[kRowBatch];
#pragma unroll
      for (int u = 0; u < kRowBatch; ++u) {
        const float* rr = rows + (size_t)(r0 + u) * pl.n_pad + j0;
        if (full) {
          xb[u] = __ldcg(reinterpret_cast<const float4*>(rr));
        } else {
          xb[u].x = (j0 < pl.n_p) ? __ldcg(rr) : 0.f;
          xb[u].y = (j0 + 1 < pl.n_p) ? __ldcg(rr + 1) : 0.f;
          xb[u].z = (j0 + 2 < pl.n_p) ? __ldcg(rr + 2) : 0.f;
          xb[u].w = (j0 + 3 < pl.n_p) ? __ldcg(rr + 3) : 0.f;
        }
      }
#pragma unroll
      for (int u = 0; u < kRowBatch; ++u) {
        float x[kSweepRun] = {xb[u].x, xb[u].y, xb[u].z, xb[u].w};
        if (tempered) {
#pragma unroll
          for (int p = 0; p < kSweepRun; ++p) x[p] = x[p] > 0.f ? powf(x[p], invT) : 0.f;
        }
        float w[KW];
#pragma unroll
        for (int q = 0; q < KW; q += 4) {
          const float4 v = *reinterpret_cast<const float4*>(sW + (r0 + u) * KW + q);
          w[q] = v.x; w[q + 1] = v.y; w[q + 2] = v.z; w[q + 3] = v.w;
        }
#pragma unroll
        for (int p = 0; p < kSweepRun; ++p)
#pragma unroll
          for (int k = 0; k < KM; ++k) bk[p][k] = fmaf(x[p], w[k], bk[p][k]);
      }
    }
  }
  // outside the transient prefix the position map is the identity
#pragma unroll
  for (int p = 0; p < kSweepRun; ++p) {
    const int j = j0 + p;
    if (j < pl.s || j >= pl.n_p)
#pragma unroll
      for (int k = 0; k < KM; ++k) bk[p][k] = 0.f;
  }
  if ((pl.n_p & 3) == 0 && j0 + kSweepRun <= pl.n_p) {   // whole run, 16-byte aligned: vector stores
#pragma unroll
    for (int k = 0; k < KM; ++k)
      if (k < K)
        *reinterpret_cast<float4*>(bk_out + (size_t)k * pl.n_p + j0) = make_float4(bk[0][k], bk[1][k], bk[2][k], bk[3][k]);
    float4* cg4 = reinterpret_cast<float4*>(cg_out + j0);
    cg4[0] = make_float4(ri.c[0], ri.g[0], ri.c[1], ri.g[1]);
    cg4[1] = make_float4(ri.c[2], ri.g[2], ri.c[3], ri.g[3]);
  } else {
#pragma unroll
    for (int p = 0; p < kSweepRun; ++p) {
      const int j = j0 + p;
      if (j < pl.n_p) {
#pragma unroll
        for (int k = 0; k < KM; ++k)
          if (k < K) bk_out[(size_t)k * pl.n_p + j] = bk[p][k];
        cg_out[j] = make_float2(ri.c[p], ri.g[p]);
      }
    }
  }

  // this run's map (positions from the top of the run down), then the chunk's
  Map<KM> A;
  map_identity(A);
#pragma unroll
  for (int p = kSweepRun - 1; p >= 0; --p) {
    const int j = j0 + p;
    if (j < pl.s || j >= pl.n_p) continue;
    float uj[KM];
    uj[0] = ri.c[p] * start_value(pl, ch, j);
#pragma unroll
    for (int k = 1; k < KM; ++k) uj[k] = (k < K) ? ri.c[p] * bk[p][k - 1] : 0.f;
    push_position(A, KM > 1 ? ri.c[p] * gamma * ri.g[p] : 0.f, uj);
  }
  A = warp_suffix_compose(A);
  if (lane == 0) store_map(sWarp + wid * map_stride<KM>(), A);
  __syncthreads();
  if (threadIdx.x == 0) {
    Map<KM> M = load_map<KM>(sWarp + (kSweepThreads / 32 - 1) * map_stride<KM>());
    for (int w = kSweepThreads / 32 - 2; w >= 0; --w) M = compose(load_map<KM>(sWarp + w * map_stride<KM>()), M);
    store_map(agg + (size_t)chunk * 2 * KM, M);
  }

  // the last CTA of this chain: incoming carry of every chunk = u of (A_{c+1} o ... o A_top)
  Header* hdr = reinterpret_cast<Header*>(ws);
  __shared__ bool last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(&hdr->cnt_sweep[ch], 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last || wid != 0) return;
  __threadfence();
  float* sin = reinterpret_cast<float*>(ws + pl.off_sin) + ((size_t)ch * pl.nscan) * kMaxIters;
  Map<KM> acc;   // composition of the chunks above the current group of 32
  map_identity(acc);
  for (int hi = pl.nscan; hi > 0; hi -= 32) {
    const int lo = hi - 32;
    const int c = lo + lane;
    Map<KM> m;
    if (c >= 0) {
#pragma unroll
      for (int i = 0; i < KM; ++i) {
        m.a[i] = __ldcg(agg + (size_t)c * 2 * KM + i);
        m.u[i] = __ldcg(agg + (size_t)c * 2 * KM + KM + i);
      }
    } else {
      map_identity(m);
    }
    const Map<KM> incl = warp_suffix_compose(m);
    const Map<KM> excl = compose(next_lane_map(incl), acc);   // chunks c+1 .. top
    if (c >= 0)
#pragma unroll
      for (int k = 0; k < KM; ++k) sin[(size_t)c * kMaxIters + k] = excl.u[k];
    Map<KM> top;
#pragma unroll
    for (int i = 0; i < KM; ++i) {
      top.a[i] = __shfl_sync(0xffffffffu, incl.a[i], 0);
      top.u[i] = __shfl_sync(0xffffffffu, incl.u[i], 0);
    }
    acc = compose(top, acc);
  }
  if (lane == 0) hdr->cnt_sweep[ch] = 0;
}

// ---------------------------------------------------------------------------
// kernel 2: incoming carry of each run, the run's sweep, terms x_0..x_K
// ---------------------------------------------------------------------------
template <int KM>
__global__ void __launch_bounds__(kSweepThreads) k_sweep_apply(const Plan pl, const ckv_params prm,
                                                               char* ws) {
  const int chunk = blockIdx.x, ch = blockIdx.y;
  const int K = pl.K;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int j0 = chunk * kScanChunk + threadIdx.x * kSweepRun;
  const float gamma = prm.neumann_gamma;
  const float* sin = reinterpret_cast<const float*>(ws + pl.off_sin) + ((size_t)ch * pl.nscan + chunk) * kMaxIters;
  const float* bk_in = reinterpret_cast<const float*>(ws + pl.off_bk) + (size_t)ch * K * pl.n_p;
  const float2* cg_in = reinterpret_cast<const float2*>(ws + pl.off_cg) + (size_t)ch * pl.n_p;
  float* cum = reinterpret_cast<float*>(ws + pl.off_cum) + (size_t)ch * (K + 1) * pl.n_p;
  float* cmax = reinterpret_cast<float*>(ws + pl.off_cmax) + ((size_t)ch * pl.nscan + chunk) * (kMaxIters + 1);
  __shared__ float sWarp[kSweepThreads / 32][2 * KM + 1];
  __shared__ float sCarry[kSweepThreads / 32][KM];
  __shared__ float sMax[kSweepThreads / 32][kMaxIters + 1];

  float c[kSweepRun], g[kSweepRun], bk[kSweepRun][KM];
#pragma unroll
  for (int p = 0; p < kSweepRun; ++p) {
    const int j = j0 + p;
    const bool in = j < pl.n_p;
    const float2 v = in ? cg_in[j] : make_float2(0.f, 0.f);
    c[p] = v.x; g[p] = v.y;
#pragma unroll
    for (int k = 0; k < KM; ++k) bk[p][k] = (in && k < K && j >= pl.s) ? bk_in[(size_t)k * pl.n_p + j] : 0.f;
  }
  auto offsets = [&](int p, float* uj) {
    const int j = j0 + p;
    uj[0] = c[p] * start_value(pl, ch, j);
#pragma unroll
    for (int k = 1; k < KM; ++k) uj[k] = (k < K) ? c[p] * bk[p][k - 1] : 0.f;
  };
  // this run's map, the suffix within the warp, the carry into each warp
  Map<KM> A;
  map_identity(A);
#pragma unroll
  for (int p = kSweepRun - 1; p >= 0; --p) {
    const int j = j0 + p;
    if (j < pl.s || j >= pl.n_p) continue;
    float uj[KM];
    offsets(p, uj);
    push_position(A, KM > 1 ? c[p] * gamma * g[p] : 0.f, uj);
  }
  const Map<KM> incl = warp_suffix_compose(A);
  if (lane == 0) store_map(&sWarp[wid][0], incl);
  __syncthreads();
  if (threadIdx.x == 0) {
    float S[KM], T[KM];
#pragma unroll
    for (int k = 0; k < KM; ++k) S[k] = sin[k];
    for (int w = kSweepThreads / 32 - 1; w >= 0; --w) {
#pragma unroll
      for (int k = 0; k < KM; ++k) sCarry[w][k] = S[k];
      apply(load_map<KM>(&sWarp[w][0]), S, T);
#pragma unroll
      for (int k = 0; k < KM; ++k) S[k] = T[k];
    }
  }
  __syncthreads();
  float S[KM];
  {
    float Cw[KM];
#pragma unroll
    for (int k = 0; k < KM; ++k) Cw[k] = sCarry[wid][k];
    apply(next_lane_map(incl), Cw, S);   // carry after every position above this run
  }

  // the run's positions from the top: terms from the incoming carry, then the update
  float mx[KM + 1];
#pragma unroll
  for (int k = 0; k <= KM; ++k) mx[k] = 0.f;
#pragma unroll
  for (int p = kSweepRun - 1; p >= 0; --p) {
    const int j = j0 + p;
    if (j >= pl.n_p) continue;
    const bool valid = j >= pl.s;
    const float x0 = start_value(pl, ch, j);
    float xs[KM];
#pragma unroll
    for (int k = 0; k < KM; ++k) xs[k] = 0.f;
    float run = x0;
    if (valid) cum[j] = run;
#pragma unroll
    for (int k = 0; k < KM; ++k) {
      if (k < K) {
        const float x = fmaf(gamma * g[p], S[k], bk[p][k]);
        xs[k] = x;
        run += x;
        if (valid) {
          cum[(size_t)(k + 1) * pl.n_p + j] = run;
          mx[k + 1] = fmaxf(mx[k + 1], fabsf(x));
        }
      }
    }
    if (valid) {   // S_k += c_j x_k[j] (x_0 = start, x_k for k >= 1 from the old carry)
#pragma unroll
      for (int k = KM - 1; k >= 1; --k) S[k] = fmaf(c[p], xs[k - 1], S[k]);
      S[0] = fmaf(c[p], x0, S[0]);
    }
  }
  // block max of every term index
#pragma unroll
  for (int k = 1; k <= KM; ++k) {
    const float v = warp_max(k <= K ? mx[k] : 0.f);
    if (lane == 0) sMax[wid][k] = v;
  }
  __syncthreads();
  if (threadIdx.x >= 1 && threadIdx.x <= K) {
    float v = 0.f;
    for (int w = 0; w < kSweepThreads / 32; ++w) v = fmaxf(v, sMax[w][threadIdx.x]);
    cmax[threadIdx.x] = v;
  }
}

template <int KM>
static cudaError_t launch_sweep_t(const Plan& pl, const ckv_params& prm, char* ws, cudaStream_t st) {
  constexpr int KW = (KM + 3) / 4 * 4;
  const size_t s1 = sizeof(float) * ((size_t)pl.W * KW + (kSweepThreads / 32) * map_stride<KM>() + 64);
  {
    const cudaError_t e = ensure_dynamic_smem((const void*)k_sweep_chunks<KM>, s1);
    if (e != cudaSuccess) return e;
  }
  const dim3 grid(pl.nscan, pl.nchains);
  k_sweep_chunks<KM><<<grid, kSweepThreads, s1, st>>>(pl, prm, ws);
  stage_mark(st);
  k_sweep_apply<KM><<<grid, kSweepThreads, 0, st>>>(pl, prm, ws);
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
