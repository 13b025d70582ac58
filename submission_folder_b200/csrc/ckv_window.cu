// Window attention of the CircuitKV prefill path (reference: pyramidkv_utils.py
// PU:2874-2999): window logits against every key, causal fp32 softmax, per-head
// entropy / transient mass, entropy-aware head selection, QI / HI pooling.
//
// Two passes over K (the softmax normaliser and the head sets are needed before
// the pooled rows can be formed):
//   k_window_stats : per row running (max, sum, entropy moment, sink mass) over a
//                    column chunk; the last CTA merges the chunks, derives the
//                    log-sum-exp of every row and a speculative head selection
//                    from the unclamped entropy.
//   k_window_pool  : recomputes the logits, forms exact probabilities, the exact
//                    clamped entropy / mass (PU:1452-1508), and pools the rows of
//                    the speculated head sets; the last CTA checks the exact head
//                    selection against the speculation (a mismatch re-runs the
//                    pass with the exact sets), reduces the row sums and runs the
//                    W x W window chain of the absorption solve.
// Logits are rounded exactly as the reference rounds them: the fp32 product is
// rounded to the input dtype, divided by sqrt(D) in fp32 and rounded again
// (PU:2874-2877).
#include <math.h>

#include "ckv_common.cuh"
#include "ckv_plan.h"
#include "ckv_window.h"

namespace ckv {

__device__ void window_pool_finish(const WinArgs& a, char* smem);
__device__ void run_window_chains(const Plan& pl, const ckv_params& prm, char* ws, float* smem);

constexpr float kGeps = 1.8420680743952367e-07f;   // -1e-8 * ln(1e-8): a clamped entry

// ---------------------------------------------------------------------------
// shared-memory staging
// ---------------------------------------------------------------------------
CKV_DEV uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

CKV_DEV void cp_async16(void* smem, const void* gmem, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(src_bytes));
}
CKV_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N> CKV_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// Bytes of one staged row of D=128 elements.
template <int DT> __host__ __device__ constexpr int row_bytes() { return DT == CKV_FP32 ? 512 : 256; }

// 16-byte chunk position inside a staged row (XOR swizzle for the 16-bit ldmatrix path).
template <int DT> CKV_DEV int chunk_off(int row, int chunk) {
  if (DT == CKV_FP32) return chunk << 4;
  return ((chunk ^ (row & 7)) << 4);
}

// Stage `rows` rows of 128 elements; row i comes from base + row_src(i) (nullptr -> zeros).
template <int DT>
CKV_DEV void stage_rows(char* smem, const char* const* srcs, int rows) {
  constexpr int kChunks = row_bytes<DT>() / 16;
  for (int i = threadIdx.x; i < rows * kChunks; i += blockDim.x) {
    const int row = i / kChunks, ch = i % kChunks;
    const char* src = srcs[row];
    char* dst = smem + row * row_bytes<DT>() + chunk_off<DT>(row, ch);
    if (src) cp_async16(dst, src + ch * 16, 16);
    else cp_async16(dst, srcs[-1], 0);   // zero fill; srcs[-1] is any valid address
  }
}

// ---------------------------------------------------------------------------
// 32 x 64 (16-bit MMA) or 16 x 64 (fp32 SIMT) logits tile of one warp.
// acc[mt][nt][e]: row = mt*16 + (lane>>2) + 8*(e>>1), col = nt*8 + 2*(lane&3) + (e&1).
// ---------------------------------------------------------------------------
template <int DT> struct MmaOp;
template <> struct MmaOp<CKV_BF16> {
  static CKV_DEV void run(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};
template <> struct MmaOp<CKV_FP16> {
  static CKV_DEV void run(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};

CKV_DEV void ldsm_x4(uint32_t* r, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

template <int DT> struct WarpTile {
  static constexpr int MT = (DT == CKV_FP32) ? 1 : 2;   // m16 tiles per warp
  static CKV_DEV void compute(const char* sQ, const char* sK, int row0, float (&acc)[MT][8][4]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[mt][nt][e] = 0.f;
    if constexpr (DT == CKV_FP32) {
      const int g = lane >> 2, t = lane & 3;
      const float* qa = reinterpret_cast<const float*>(sQ + (row0 + g) * 512);
      const float* qb = reinterpret_cast<const float*>(sQ + (row0 + g + 8) * 512);
      for (int k = 0; k < kHeadDim; k += 4) {
        const float4 a = *reinterpret_cast<const float4*>(qa + k);
        const float4 b = *reinterpret_cast<const float4*>(qb + k);
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float4 kv =
                *reinterpret_cast<const float4*>(sK + (nt * 8 + 2 * t + e) * 512 + k * 4);
            float s0 = acc[0][nt][e], s1 = acc[0][nt][2 + e];
            s0 = fmaf(a.x, kv.x, s0); s0 = fmaf(a.y, kv.y, s0);
            s0 = fmaf(a.z, kv.z, s0); s0 = fmaf(a.w, kv.w, s0);
            s1 = fmaf(b.x, kv.x, s1); s1 = fmaf(b.y, kv.y, s1);
            s1 = fmaf(b.z, kv.z, s1); s1 = fmaf(b.w, kv.w, s1);
            acc[0][nt][e] = s0;
            acc[0][nt][2 + e] = s1;
          }
      }
    } else {
#pragma unroll
      for (int ks = 0; ks < kHeadDim / 16; ++ks) {
        uint32_t a[MT][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const int row = row0 + mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int ch = ks * 2 + (lane >> 4);
          ldsm_x4(a[mt], sQ + row * 256 + chunk_off<DT>(row, ch));
        }
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t b[4];
          const int row = np * 16 + (lane & 7) + ((lane >> 4) & 1) * 8;
          const int ch = ks * 2 + ((lane >> 3) & 1);
          ldsm_x4(b, sK + row * 256 + chunk_off<DT>(row, ch));
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            MmaOp<DT>::run(acc[mt][2 * np], a[mt], b[0], b[1]);
            MmaOp<DT>::run(acc[mt][2 * np + 1], a[mt], b[2], b[3]);
          }
        }
      }
    }
  }
};

// Reference rounding of a logit: dtype(dtype(acc) / sqrt(D)) for 16-bit inputs, acc / sqrt(D) for fp32.
template <int DT> CKV_DEV float logit_of(float acc, float scale) {
  if constexpr (DT == CKV_FP32) return __fdiv_rn(acc, scale);
  return round_dt<DT>(__fdiv_rn(round_dt<DT>(acc), scale));
}

// ---------------------------------------------------------------------------
// online softmax moments
// ---------------------------------------------------------------------------
struct Moments {
  float m, z, t, s;   // max (log2 units), sum 2^(y-m), sum 2^(y-m)(y-m), sink part of z
};

CKV_DEV Moments merge(const Moments& a, const Moments& b) {
  Moments r;
  r.m = fmaxf(a.m, b.m);
  if (r.m == -INFINITY) { r.z = r.t = r.s = 0.f; return r; }
  float sa = 0.f, sb = 0.f, ta = 0.f, tb = 0.f;
  if (a.m != -INFINITY) { const float d = a.m - r.m; sa = ex2(d); ta = sa * (a.t + d * a.z); }
  if (b.m != -INFINITY) { const float d = b.m - r.m; sb = ex2(d); tb = sb * (b.t + d * b.z); }
  r.z = sa * a.z + sb * b.z;
  r.t = ta + tb;
  r.s = sa * a.s + sb * b.s;
  return r;
}

// ---------------------------------------------------------------------------
// head selection (PU:2905-2999) from per-head entropy and transient mass
// ---------------------------------------------------------------------------
__device__ void select_heads(const ckv_params& p, int H, const float* ent, const float* mass,
                             uint64_t* qi_set, uint64_t* hi_set, int* hi_mode, int* n_hi) {
  const uint64_t all = (H >= 64) ? ~0ull : ((1ull << H) - 1);
  if (!p.entropy_aware) {
    *qi_set = all; *hi_set = all; *hi_mode = 2; *n_hi = H;
    return;
  }
  // QI: the k lowest entropies (or highest masses); ties resolved by head index.
  const int k = min(p.top_k_heads, H);
  uint64_t q = 0;
  for (int h = 0; h < H; ++h) {
    int better = 0;
    for (int o = 0; o < H; ++o) {
      bool b;
      if (p.head_selection_mode == 1) b = mass[o] > mass[h] || (mass[o] == mass[h] && o < h);
      else b = ent[o] < ent[h] || (ent[o] == ent[h] && o < h);
      better += b ? 1 : 0;
    }
    if (better < k) q |= 1ull << h;
  }
  *qi_set = q;
  if (p.hi_pooling_mode == 1) { *hi_set = all; *hi_mode = 1; *n_hi = H; return; }
  uint64_t hs = all;
  if (p.hi_mass_cdf > 0.f) {
    float total = 0.f;
    for (int h = 0; h < H; ++h) total += mass[h];
    if (total > 0.f) {
      // heads in descending mass order until the cumulative share reaches the threshold
      int need = 1;
      float cum = 0.f;
      int order[kMaxHeads];
      for (int h = 0; h < H; ++h) {
        int pos = 0;
        for (int o = 0; o < H; ++o)
          pos += (mass[o] > mass[h] || (mass[o] == mass[h] && o < h)) ? 1 : 0;
        order[pos] = h;
      }
      int below = 0;
      for (int i = 0; i < H; ++i) { cum += mass[order[i]]; if (cum / total < p.hi_mass_cdf) ++below; }
      need = min(below + 1, H);
      hs = 0;
      for (int i = 0; i < need; ++i) hs |= 1ull << order[i];
    }
  } else if (p.hi_top_k_heads > 0) {
    const int kh = min(p.hi_top_k_heads, H);
    hs = 0;
    for (int h = 0; h < H; ++h) {
      int better = 0;
      for (int o = 0; o < H; ++o)
        better += (mass[o] > mass[h] || (mass[o] == mass[h] && o < h)) ? 1 : 0;
      if (better < kh) hs |= 1ull << h;
    }
  } else if (p.hi_mass_threshold > 0.f) {
    hs = 0;
    for (int h = 0; h < H; ++h)
      if (mass[h] >= p.hi_mass_threshold) hs |= 1ull << h;
    if (hs == 0) hs = all;
  }
  *hi_set = hs; *hi_mode = 0; *n_hi = __popcll(hs);
}

// ---------------------------------------------------------------------------
// common per-CTA setup of the window kernels
// ---------------------------------------------------------------------------
struct BatchGeom {
  int h0;        // first head of the batch
  int g0;        // first KV head touched by the batch
  int ng;        // KV heads touched
};

CKV_DEV BatchGeom batch_geom(const Plan& pl, int b) {
  BatchGeom bg;
  bg.h0 = b * pl.heads_per_batch;
  bg.g0 = bg.h0 / pl.G;
  bg.ng = (bg.h0 + pl.heads_per_batch - 1) / pl.G - bg.g0 + 1;
  return bg;
}

template <int DT>
CKV_DEV void stage_q(const WinArgs& a, const BatchGeom& bg, char* sQ, const char** srcs) {
  using T = typename Elem<DT>::T;
  const Plan& pl = a.pl;
  // row i of the batch: head h0 + i / W, window row i % W
  for (int i = threadIdx.x; i < pl.rows_per_batch; i += blockDim.x) {
    const int h = bg.h0 + i / pl.W, r = i % pl.W;
    srcs[i] = reinterpret_cast<const char*>(static_cast<const T*>(a.q) + h * a.qhs +
                                            (int64_t)(pl.n - pl.W + r) * a.qts);
  }
  if (threadIdx.x == 0) srcs[-1] = reinterpret_cast<const char*>(a.q);
  __syncthreads();
  stage_rows<DT>(sQ, srcs, pl.rows_per_batch);
  __syncthreads();
}

template <int DT>
CKV_DEV void stage_k(const WinArgs& a, const BatchGeom& bg, int j0, char* sK, const char** srcs) {
  using T = typename Elem<DT>::T;
  const Plan& pl = a.pl;
  const int rows = bg.ng * kColTile;
  for (int i = threadIdx.x; i < rows; i += blockDim.x) {
    const int gk = bg.g0 + i / kColTile, j = j0 + i % kColTile;
    srcs[i] = (j < pl.n) ? reinterpret_cast<const char*>(static_cast<const T*>(a.k) + gk * a.khs +
                                                         (int64_t)j * a.kts)
                         : nullptr;
  }
  if (threadIdx.x == 0) srcs[-1] = reinterpret_cast<const char*>(a.k);
  __syncthreads();
  stage_rows<DT>(sK, srcs, rows);
}

// ---------------------------------------------------------------------------
// pass 1: row moments
// ---------------------------------------------------------------------------
template <int DT>
__global__ void __launch_bounds__(256) k_window_stats(WinArgs a) {
  using WT = WarpTile<DT>;
  constexpr int MT = WT::MT;
  extern __shared__ __align__(128) char smem[];
  const Plan& pl = a.pl;
  const int chunk = blockIdx.x, b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const BatchGeom bg = batch_geom(pl, b);
  char* sQ = smem;
  char* sK0 = sQ + pl.rows_per_batch * row_bytes<DT>();
  const int kbytes = pl.ktiles_per_batch * kColTile * row_bytes<DT>();
  char* sK1 = sK0 + kbytes;
  const char** srcs = reinterpret_cast<const char**>(sK1 + kbytes) + 1;

  stage_q<DT>(a, bg, sQ, srcs);
  cp_async_commit();

  const int row0 = warp * pl.rows_per_warp;          // batch-local first row of this warp
  const int hl = row0 / pl.W;                        // batch-local head (W is a multiple of rows/warp)
  const int kt = (bg.h0 + hl) / pl.G - bg.g0;        // K tile of this warp's KV head
  const float scale = sqrtf((float)pl.D);
  const int t0 = chunk * pl.tiles_per_chunk;
  const int t1 = min(t0 + pl.tiles_per_chunk, pl.ncol_tiles);

  Moments mom[MT][2];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) mom[mt][hf] = Moments{-INFINITY, 0.f, 0.f, 0.f};

  if (t0 < t1) {
    __syncthreads();
    stage_k<DT>(a, bg, t0 * kColTile, sK0, srcs);
    cp_async_commit();
  }
  for (int t = t0; t < t1; ++t) {
    char* cur = ((t - t0) & 1) ? sK1 : sK0;
    char* nxt = ((t - t0) & 1) ? sK0 : sK1;
    __syncthreads();
    if (t + 1 < t1) {
      stage_k<DT>(a, bg, (t + 1) * kColTile, nxt, srcs);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    float acc[MT][8][4];
    WT::compute(sQ, cur + kt * kColTile * row_bytes<DT>(), row0, acc);
    const int j0 = t * kColTile;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int rl = row0 + mt * 16 + (lane >> 2) + 8 * hf;   // batch-local row
        const int r = rl % pl.W;
        const int lim = pl.n - pl.W + r;                          // last visible key
        float y[16];
        float tmax = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int j = j0 + nt * 8 + 2 * (lane & 3) + e;
            float v = -INFINITY;
            if (j <= lim) v = logit_of<DT>(acc[mt][nt][2 * hf + e], scale) * kLog2e;
            y[nt * 2 + e] = v;
            tmax = fmaxf(tmax, v);
          }
        Moments& M = mom[mt][hf];
        if (tmax > M.m) {
          if (M.m == -INFINITY) {
            M.m = tmax;
          } else {
            const float d = tmax - M.m;
            const float sc = ex2(-d);
            M.t = sc * (M.t - d * M.z);
            M.z *= sc;
            M.s *= sc;
            M.m = tmax;
          }
        }
        if (M.m != -INFINITY) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            if (y[i] != -INFINITY) {
              const float d = y[i] - M.m;
              const float e = ex2(d);
              M.z += e;
              M.t = fmaf(e, d, M.t);
              const int j = j0 + (i >> 1) * 8 + 2 * (lane & 3) + (i & 1);
              if (j < pl.s) M.s += e;
            }
          }
        }
      }
  }
  // merge the four lanes of a quad, then write this chunk's partial moments
  float4* part = reinterpret_cast<float4*>(a.ws + pl.off_stats);
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      Moments M = mom[mt][hf];
#pragma unroll
      for (int o = 1; o <= 2; o <<= 1) {
        Moments O;
        O.m = __shfl_xor_sync(0xffffffffu, M.m, o);
        O.z = __shfl_xor_sync(0xffffffffu, M.z, o);
        O.t = __shfl_xor_sync(0xffffffffu, M.t, o);
        O.s = __shfl_xor_sync(0xffffffffu, M.s, o);
        M = merge(M, O);
      }
      if ((lane & 3) == 0) {
        const int rl = row0 + mt * 16 + (lane >> 2) + 8 * hf;
        const int h = bg.h0 + rl / pl.W, r = rl % pl.W;
        part[((size_t)chunk * pl.H + h) * pl.W + r] = make_float4(M.m, M.z, M.t, M.s);
      }
    }

  // ---- the last CTA merges the chunks and speculates the head sets ----
  __shared__ bool last;
  __threadfence();
  __syncthreads();
  Header* hdr = reinterpret_cast<Header*>(a.ws);
  if (threadIdx.x == 0) {
    const uint32_t total = gridDim.x * gridDim.y;
    last = atomicAdd(&hdr->cnt_stats, 1u) == total - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  float* lse = reinterpret_cast<float*>(a.ws + pl.off_lse);
  float* spec = reinterpret_cast<float*>(a.ws + pl.off_spec);   // [H] entropy, [H] mass
  float* rowE = reinterpret_cast<float*>(smem);                  // [H*W]
  float* rowM = rowE + pl.H * pl.W;
  for (int i = threadIdx.x; i < pl.H * pl.W; i += blockDim.x) {
    Moments M{-INFINITY, 0.f, 0.f, 0.f};
    for (int c = 0; c < pl.nstat_chunks; ++c) {
      const float4 v = __ldcg(part + (size_t)c * pl.H * pl.W + i);
      M = merge(M, Moments{v.x, v.y, v.z, v.w});
    }
    const float l2z = log2f(M.z);
    lse[i] = M.m + l2z;
    const int r = i % pl.W;
    rowE[i] = l2z * kLn2 - kLn2 * (M.t / M.z) + (float)(pl.W - 1 - r) * kGeps;
    rowM[i] = 1.f - M.s / M.z;
  }
  __syncthreads();
  for (int h = threadIdx.x; h < pl.H; h += blockDim.x) {
    float e = 0.f, m = 0.f;
    for (int r = 0; r < pl.W; ++r) { e += rowE[h * pl.W + r]; m += rowM[h * pl.W + r]; }
    spec[h] = e / (float)pl.W;
    spec[pl.H + h] = m / (float)pl.W;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    uint64_t qs, hs;
    int hm, nh;
    select_heads(a.p, pl.H, spec, spec + pl.H, &qs, &hs, &hm, &nh);
    hdr->qi_heads = qs;
    hdr->hi_heads = hs;
    hdr->hi_mode = hm;
    hdr->n_hi = nh;
    hdr->fixup = 0;
    hdr->cnt_stats = 0;
  }
}

// ---------------------------------------------------------------------------
// pass 2: exact probabilities, exact entropy / mass, pooled rows
// ---------------------------------------------------------------------------
constexpr int kStageStride = kColTile + 8;   // floats per staged probability row

template <int DT>
__global__ void __launch_bounds__(256) k_window_pool(WinArgs a) {
  using WT = WarpTile<DT>;
  constexpr int MT = WT::MT;
  extern __shared__ __align__(128) char smem[];
  const Plan& pl = a.pl;
  Header* hdr = reinterpret_cast<Header*>(a.ws);
  if (a.fixup_pass && *reinterpret_cast<volatile int32_t*>(&hdr->fixup) == 0) return;

  const int tile = blockIdx.x;
  const int j0 = tile * kColTile;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  char* sQ = smem;
  char* sK = sQ + pl.rows_per_batch * row_bytes<DT>();
  float* sP = reinterpret_cast<float*>(sK + pl.ktiles_per_batch * kColTile * row_bytes<DT>());
  const char** srcs =
      reinterpret_cast<const char**>(sP + pl.rows_per_batch * kStageStride) + 1;
  __shared__ float red[64];
  __shared__ float colpart[4][kColTile];

  const uint64_t qset = hdr->qi_heads, hset = hdr->hi_heads;
  const int hmode = hdr->hi_mode, nhi = hdr->n_hi;
  const float* lse = reinterpret_cast<const float*>(a.ws + pl.off_lse);
  float* epart = reinterpret_cast<float*>(a.ws + pl.off_epart);
  float* mpart = reinterpret_cast<float*>(a.ws + pl.off_mpart);
  const float scale = sqrtf((float)pl.D);

  // pooling-pass mapping: column c = tid % 64, rows r = tid / 64 + 4 i
  const int pc = threadIdx.x % kColTile;
  const int pr0 = threadIdx.x / kColTile;
  constexpr int kRowsPerThread = kMaxWindow / 4;
  float qacc[kRowsPerThread], hacc[kRowsPerThread];
#pragma unroll
  for (int i = 0; i < kRowsPerThread; ++i) { qacc[i] = 0.f; hacc[i] = 0.f; }

  for (int b = 0; b < pl.nbatch; ++b) {
    const BatchGeom bg = batch_geom(pl, b);
    __syncthreads();
    stage_q<DT>(a, bg, sQ, srcs);       // (syncs inside)
    stage_k<DT>(a, bg, j0, sK, srcs);
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    const int row0 = warp * pl.rows_per_warp;
    const int hl = row0 / pl.W;
    const int kt = (bg.h0 + hl) / pl.G - bg.g0;
    float acc[MT][8][4];
    WT::compute(sQ, sK + kt * kColTile * row_bytes<DT>(), row0, acc);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int rl = row0 + mt * 16 + (lane >> 2) + 8 * hf;
        const int h = bg.h0 + rl / pl.W, r = rl % pl.W;
        const int lim = pl.n - pl.W + r;
        const float L = lse[h * pl.W + r];
        float ent = 0.f, mass = 0.f;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          float pv[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int j = j0 + nt * 8 + 2 * (lane & 3) + e;
            float p = 0.f;
            if (j <= lim) {
              const float y = logit_of<DT>(acc[mt][nt][2 * hf + e], scale) * kLog2e;
              const float d = y - L;
              p = ex2(d);
              ent += (p >= 1e-8f) ? -p * d * kLn2 : kGeps;
              if (j >= pl.s) mass += p;
            } else if (j < pl.n) {
              ent += kGeps;   // masked entry: probability 0, clamped to 1e-8
            }
            pv[e] = p;
          }
          *reinterpret_cast<float2*>(sP + rl * kStageStride + nt * 8 + 2 * (lane & 3)) =
              make_float2(pv[0], pv[1]);
        }
        ent += __shfl_xor_sync(0xffffffffu, ent, 1);
        ent += __shfl_xor_sync(0xffffffffu, ent, 2);
        mass += __shfl_xor_sync(0xffffffffu, mass, 1);
        mass += __shfl_xor_sync(0xffffffffu, mass, 2);
        if ((lane & 3) == 0) {
          epart[((size_t)tile * pl.H + h) * pl.W + r] = ent;
          mpart[((size_t)tile * pl.H + h) * pl.W + r] = mass;
        }
      }
    __syncthreads();
    // pool the batch's heads in ascending head order
    for (int hl2 = 0; hl2 < pl.heads_per_batch; ++hl2) {
      const int h = bg.h0 + hl2;
      const bool inq = (qset >> h) & 1ull, inh = (hset >> h) & 1ull;
      if (!inq && !inh) continue;
#pragma unroll
      for (int i = 0; i < kRowsPerThread; ++i) {
        const int r = pr0 + 4 * i;
        if (r < pl.W) {
          const float p = sP[(hl2 * pl.W + r) * kStageStride + pc];
          if (inq) qacc[i] = fmaxf(qacc[i], p);
          if (inh) hacc[i] = (hmode == 1) ? fmaxf(hacc[i], p) : hacc[i] + p;
        }
      }
    }
  }

  // ---- finalize the pooled rows of this column tile ----
  const int j = j0 + pc;
  const bool tempered = a.p.neumann_temperature != 1.0f && a.p.neumann_temperature > 0.f;
  const float invT = tempered ? 1.0f / a.p.neumann_temperature : 1.0f;
  float* rows_qi = reinterpret_cast<float*>(a.ws + pl.off_rows_qi);
  float* rows_hi = reinterpret_cast<float*>(a.ws + pl.off_rows_hi);
  float* colsum = reinterpret_cast<float*>(a.ws + pl.off_colsum);     // [2][n_pad]
  float* gtile = reinterpret_cast<float*>(a.ws + pl.off_gtile);       // [2][ncol_tiles]
  float* rspart = reinterpret_cast<float*>(a.ws + pl.off_rspart);     // [2][ncol_tiles][W]
  __shared__ float sRed[kRowsPerThread][kWarps];
  const int nch = pl.hi_rows ? 2 : 1;
  for (int ch = 0; ch < nch; ++ch) {
    float* rows = ch == 0 ? rows_qi : rows_hi;
    float cs = 0.f;
#pragma unroll
    for (int i = 0; i < kRowsPerThread; ++i) {
      const int r = pr0 + 4 * i;
      if (r < pl.W) {   // uniform per warp: a warp's 32 threads share r
        float v = ch == 0 ? qacc[i] : (hmode == 1 ? hacc[i] : hacc[i] / (float)nhi);
        if (j >= pl.n) v = 0.f;
        rows[(size_t)r * pl.n_pad + j] = v;
        cs += v;
        // row-sum partial over this tile's columns (tempered for the transition rows)
        float rv = tempered ? (v > 0.f ? powf(v, invT) : 0.f) : v;
        rv = warp_sum(rv);
        if (lane == 0) sRed[i][warp] = rv;
      }
    }
    colpart[pr0][pc] = cs;
    __syncthreads();
    for (int r = threadIdx.x; r < pl.W; r += blockDim.x) {
      const int i = r / 4, w = 2 * (r % 4);
      rspart[((size_t)ch * pl.ncol_tiles + tile) * pl.W + r] = sRed[i][w] + sRed[i][w + 1];
    }
    if (threadIdx.x < kColTile) {
      const int jj = j0 + threadIdx.x;
      const float c = colpart[0][threadIdx.x] + colpart[1][threadIdx.x] + colpart[2][threadIdx.x] +
                      colpart[3][threadIdx.x];
      colsum[(size_t)ch * pl.n_pad + jj] = c;
      float g = 0.f;
      if (jj < pl.n_p) {
        g = fmaxf(c, 1e-6f);
        if (tempered) g = powf(g, invT);
      }
      g = warp_sum(g);
      if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = g;
    }
    __syncthreads();
    if (threadIdx.x == 0) gtile[(size_t)ch * pl.ncol_tiles + tile] = red[0] + red[1];
    __syncthreads();
  }

  // ---- the last CTA verifies the head sets and runs the window chain ----
  __shared__ bool last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    last = atomicAdd(&hdr->cnt_pool, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  window_pool_finish(a, smem);
}

// ---------------------------------------------------------------------------
// last-CTA work of the pooling pass
// ---------------------------------------------------------------------------
__device__ void window_pool_finish(const WinArgs& a, char* smem) {
  const Plan& pl = a.pl;
  Header* hdr = reinterpret_cast<Header*>(a.ws);
  const float* epart = reinterpret_cast<const float*>(a.ws + pl.off_epart);
  const float* mpart = reinterpret_cast<const float*>(a.ws + pl.off_mpart);
  float* exact = reinterpret_cast<float*>(a.ws + pl.off_spec) + 2 * pl.H;   // [H] ent, [H] mass
  float* rowE = reinterpret_cast<float*>(smem);
  float* rowM = rowE + pl.H * pl.W;
  for (int i = threadIdx.x; i < pl.H * pl.W; i += blockDim.x) {
    float e = 0.f, m = 0.f;
    for (int t = 0; t < pl.ncol_tiles; ++t) {
      e += __ldcg(epart + (size_t)t * pl.H * pl.W + i);
      m += __ldcg(mpart + (size_t)t * pl.H * pl.W + i);
    }
    rowE[i] = e;
    rowM[i] = m;
  }
  __syncthreads();
  for (int h = threadIdx.x; h < pl.H; h += blockDim.x) {
    float e = 0.f, m = 0.f;
    for (int r = 0; r < pl.W; ++r) { e += rowE[h * pl.W + r]; m += rowM[h * pl.W + r]; }
    exact[h] = e / (float)pl.W;
    exact[pl.H + h] = m / (float)pl.W;
  }
  __syncthreads();
  __shared__ int redo;
  if (threadIdx.x == 0) {
    uint64_t qs, hs;
    int hm, nh;
    select_heads(a.p, pl.H, exact, exact + pl.H, &qs, &hs, &hm, &nh);
    redo = (qs != hdr->qi_heads || hs != hdr->hi_heads || hm != hdr->hi_mode) ? 1 : 0;
    if (redo && !a.fixup_pass) {
      hdr->qi_heads = qs;
      hdr->hi_heads = hs;
      hdr->hi_mode = hm;
      hdr->n_hi = nh;
      hdr->fixup = 1;
    } else {
      redo = 0;
    }
    hdr->cnt_pool = 0;
  }
  __syncthreads();
  if (redo) return;   // the fixup launch redoes the pooling and this step

  run_window_chains(a.pl, a.p, a.ws, reinterpret_cast<float*>(smem));
}

// Row sums (tempered) of the pooled rows and the W x W window chain of each
// absorbing chain: y_0 (query one-hot or uniform), y_{k+1} = gamma * Pww^T y_k.
// Writes y_k, the weights w_k = gamma * y_k / rowsum used by the prefix sweep,
// and max_c y_k.  One CTA; `smem` >= W*W + 5*W + 32 floats.
__device__ void run_window_chains(const Plan& pl, const ckv_params& prm, char* ws, float* smem) {
  // row sums (tempered), then the W x W window chain of each absorbing chain
  const int W = pl.W, K = pl.K;
  const bool tempered = prm.neumann_temperature != 1.0f && prm.neumann_temperature > 0.f;
  const float invT = tempered ? 1.0f / prm.neumann_temperature : 1.0f;
  const float gam = prm.neumann_gamma;
  const float* rspart = reinterpret_cast<const float*>(ws + pl.off_rspart);
  float* wk = reinterpret_cast<float*>(ws + pl.off_wk);     // [2][K][W]
  float* yk = reinterpret_cast<float*>(ws + pl.off_yk);     // [2][K+1][W]
  float* ymax = reinterpret_cast<float*>(ws + pl.off_ymax); // [2][K+1]
  float* sPw = smem;                                          // [W][W]
  float* sRs = smem + W * W;                                  // [W]
  float* sY = sRs + W;                                        // [2][W]
  const int nchain = pl.nchains;
  for (int ch = 0; ch < nchain; ++ch) {
    const bool own = (ch == 0) || pl.hi_rows;
    const float* rows = reinterpret_cast<const float*>(ws + (own && ch == 1 ? pl.off_rows_hi
                                                                               : pl.off_rows_qi));
    const int src = own ? ch : 0;
    for (int r = threadIdx.x; r < W; r += blockDim.x) {
      float s = 0.f;
      for (int t = 0; t < pl.ncol_tiles; ++t)
        s += __ldcg(rspart + ((size_t)src * pl.ncol_tiles + t) * W + r);
      sRs[r] = fmaxf(s, 1e-8f);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < W * W; i += blockDim.x) {
      const int r = i / W, c = i % W;
      float v = __ldcg(rows + (size_t)r * pl.n_pad + pl.n_p + c);
      if (tempered) v = v > 0.f ? powf(v, invT) : 0.f;
      sPw[i] = v / sRs[r];
    }
    // start vector: the query one-hot (QI) or uniform 1/n_transient (HI)
    const bool query_start = (ch == 0);
    const float u = 1.0f / (float)(pl.n - pl.s);
    for (int c = threadIdx.x; c < W; c += blockDim.x) sY[c] = query_start ? (c == W - 1 ? 1.f : 0.f) : u;
    __syncthreads();
    for (int k = 0; k <= K; ++k) {
      float* cur = sY + (k & 1) * W;
      float* nxt = sY + ((k + 1) & 1) * W;
      for (int c = threadIdx.x; c < W; c += blockDim.x) {
        yk[((size_t)ch * (K + 1) + k) * W + c] = cur[c];
        if (k < K) wk[((size_t)ch * K + k) * W + c] = gam * cur[c] / sRs[c];
      }
      float mx = 0.f;
      for (int c = threadIdx.x; c < W; c += blockDim.x) mx = fmaxf(mx, fabsf(cur[c]));
      mx = block_reduce<true>(mx, smem + W * W + 3 * W);
      if (threadIdx.x == 0) ymax[ch * (K + 1) + k] = mx;
      if (k < K) {
        for (int c = threadIdx.x; c < W; c += blockDim.x) {
          float s = 0.f;
          for (int r = c; r < W; ++r) s = fmaf(sPw[r * W + c], cur[r], s);
          nxt[c] = gam * s;
        }
      }
      __syncthreads();
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// stage entry: pooled rows given by the caller (ckv_neumann_rows)
// ---------------------------------------------------------------------------
// Per column tile: column sums, g-tile totals and row-sum partials of rows already
// placed in the workspace (same outputs as the pooling pass's finalize step).
__global__ void __launch_bounds__(256) k_rows_prep(const Plan pl, const ckv_params prm, char* ws) {
  const int tile = blockIdx.x, ch = blockIdx.y;
  const int j0 = tile * kColTile;
  const bool tempered = prm.neumann_temperature != 1.0f && prm.neumann_temperature > 0.f;
  const float invT = tempered ? 1.0f / prm.neumann_temperature : 1.0f;
  const float* rows = reinterpret_cast<const float*>(ws + (ch == 0 ? pl.off_rows_qi : pl.off_rows_hi));
  float* colsum = reinterpret_cast<float*>(ws + pl.off_colsum);
  float* gtile = reinterpret_cast<float*>(ws + pl.off_gtile);
  float* rspart = reinterpret_cast<float*>(ws + pl.off_rspart);
  __shared__ float red[32];
  // column sums (sequential over rows) and g
  float g = 0.f;
  if (threadIdx.x < kColTile) {
    const int j = j0 + threadIdx.x;
    float c = 0.f;
    for (int r = 0; r < pl.W; ++r) c += rows[(size_t)r * pl.n_pad + j];
    colsum[(size_t)ch * pl.n_pad + j] = c;
    if (j < pl.n_p) {
      g = fmaxf(c, 1e-6f);
      if (tempered) g = powf(g, invT);
    }
  }
  g = block_reduce<false>(g, red);
  if (threadIdx.x == 0) gtile[(size_t)ch * pl.ncol_tiles + tile] = g;
  // row sums over this tile
  for (int r = threadIdx.x; r < pl.W; r += blockDim.x) {
    float s = 0.f;
    for (int c = 0; c < kColTile; ++c) {
      float v = rows[(size_t)r * pl.n_pad + j0 + c];
      if (tempered) v = v > 0.f ? powf(v, invT) : 0.f;
      s += v;
    }
    rspart[((size_t)ch * pl.ncol_tiles + tile) * pl.W + r] = s;
  }
}

__global__ void __launch_bounds__(256) k_rows_chain(const Plan pl, const ckv_params prm, char* ws) {
  extern __shared__ __align__(16) float fsmem[];
  run_window_chains(pl, prm, ws, fsmem);
}

cudaError_t launch_rows_prep(const Plan& pl, const ckv_params& prm, char* ws, cudaStream_t st) {
  k_rows_prep<<<dim3(pl.ncol_tiles, pl.hi_rows ? 2 : 1), 256, 0, st>>>(pl, prm, ws);
  const size_t sm = sizeof(float) * ((size_t)pl.W * pl.W + 5 * pl.W + 64);
  static size_t have = 0;
  if (sm > have) {
    const cudaError_t e = cudaFuncSetAttribute(k_rows_chain, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    if (e != cudaSuccess) return e;
    have = sm;
  }
  k_rows_chain<<<1, 256, sm, st>>>(pl, prm, ws);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------
template <int DT> size_t stats_smem(const Plan& pl) {
  return (size_t)pl.rows_per_batch * row_bytes<DT>() +
         2 * (size_t)pl.ktiles_per_batch * kColTile * row_bytes<DT>() +
         sizeof(void*) * (size_t)(pl.rows_per_batch + pl.ktiles_per_batch * kColTile + 2);
}
template <int DT> size_t pool_smem(const Plan& pl) {
  return (size_t)pl.rows_per_batch * row_bytes<DT>() +
         (size_t)pl.ktiles_per_batch * kColTile * row_bytes<DT>() +
         (size_t)pl.rows_per_batch * kStageStride * sizeof(float) +
         sizeof(void*) * (size_t)(pl.rows_per_batch + pl.ktiles_per_batch * kColTile + 2);
}

size_t window_smem_bytes(const Plan& pl, bool pool) {
  switch (pl.dtype) {
    case CKV_BF16: return pool ? pool_smem<CKV_BF16>(pl) : stats_smem<CKV_BF16>(pl);
    case CKV_FP16: return pool ? pool_smem<CKV_FP16>(pl) : stats_smem<CKV_FP16>(pl);
    default: return pool ? pool_smem<CKV_FP32>(pl) : stats_smem<CKV_FP32>(pl);
  }
}

template <int DT>
static cudaError_t launch_window_t(const WinArgs& a, int stage, cudaStream_t st) {
  const Plan& pl = a.pl;
  // opt in to the dynamic shared memory this launch needs (kernels also hold a little static smem)
  static size_t set_stats = 0, set_pool = 0;
  const size_t need = stage == 0 ? stats_smem<DT>(pl) : pool_smem<DT>(pl);
  size_t& have = stage == 0 ? set_stats : set_pool;
  if (need > have) {
    const cudaError_t e = stage == 0
        ? cudaFuncSetAttribute(k_window_stats<DT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)need)
        : cudaFuncSetAttribute(k_window_pool<DT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)need);
    if (e != cudaSuccess) return e;
    have = need;
  }
  if (stage == 0) {
    k_window_stats<DT><<<dim3(pl.nstat_chunks, pl.nbatch), 256, stats_smem<DT>(pl), st>>>(a);
  } else {
    WinArgs b = a;
    b.fixup_pass = stage == 2 ? 1 : 0;
    k_window_pool<DT><<<pl.ncol_tiles, 256, pool_smem<DT>(pl), st>>>(b);
  }
  return cudaGetLastError();
}

// stage 0: row moments; 1: pooling pass; 2: pooling re-run (returns at once unless flagged)
cudaError_t launch_window_stage(const WinArgs& a, int stage, cudaStream_t st) {
  switch (a.pl.dtype) {
    case CKV_BF16: return launch_window_t<CKV_BF16>(a, stage, st);
    case CKV_FP16: return launch_window_t<CKV_FP16>(a, stage, st);
    default: return launch_window_t<CKV_FP32>(a, stage, st);
  }
}

cudaError_t launch_window(const WinArgs& a, cudaStream_t st) {
  for (int s = 0; s < 3; ++s) {
    const cudaError_t e = launch_window_stage(a, s, st);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace ckv
