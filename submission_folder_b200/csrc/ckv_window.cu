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

#include <cooperative_groups.h>
#include <cuda.h>
#include <cudaTypedefs.h>

#include "ckv_common.cuh"
#include "ckv_plan.h"
#include "ckv_tc.cuh"
#include "ckv_window.h"

namespace ckv {

__device__ void stats_finish(const WinArgs& a, char* smem, int h0, int nh, int gidx, int per_group, int ngroups);
CKV_DEV float sum_parts(const float* base, int nparts, size_t stride, int first, int step);
template <int DT> size_t pool_smem(const Plan& pl);

constexpr float kGeps = 1.8420680743952367e-07f;   // -1e-8 * ln(1e-8): a clamped entry
constexpr float kLog2Eps = -26.575424759098897f;     // log2(1e-8)

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

// Bytes of one row of D=128 elements, and the stride of a staged row in shared memory.
// fp32 rows are padded by 16 bytes (132 words): the SIMT tile reads float4s of 8 query rows
// (or 4 key rows 2 apart) at one offset, which then fall in distinct banks (an unpadded
// 512-byte stride put them all in the same four banks).
template <int DT> __host__ __device__ constexpr int row_data_bytes() { return DT == CKV_FP32 ? 512 : 256; }
template <int DT> __host__ __device__ constexpr int row_bytes() { return DT == CKV_FP32 ? 528 : 256; }

// 16-byte chunk position inside a staged row (XOR swizzle for the 16-bit ldmatrix path).
template <int DT> CKV_DEV int chunk_off(int row, int chunk) {
  if (DT == CKV_FP32) return chunk << 4;
  return ((chunk ^ (row & 7)) << 4);
}

// Stage `rows` rows of 128 elements; row i comes from base + row_src(i) (nullptr -> zeros).
template <int DT>
CKV_DEV void stage_rows(char* smem, const char* const* srcs, int rows) {
  constexpr int kChunks = row_data_bytes<DT>() / 16;
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
      constexpr int RB = row_bytes<CKV_FP32>();
      const float* qa = reinterpret_cast<const float*>(sQ + (row0 + g) * RB);
      const float* qb = reinterpret_cast<const float*>(sQ + (row0 + g + 8) * RB);
      for (int k = 0; k < kHeadDim; k += 4) {
        const float4 a = *reinterpret_cast<const float4*>(qa + k);
        const float4 b = *reinterpret_cast<const float4*>(qb + k);
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float4 kv =
                *reinterpret_cast<const float4*>(sK + (nt * 8 + 2 * t + e) * RB + k * 4);
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
// (bf16: the reciprocal product of the reference's CUDA division by a scalar; fp16 divides.)
// Logit of one accumulator; inv_scale = RN(1 / scale).
template <int DT> CKV_DEV float logit_of(float acc, float scale, float inv_scale) {
  if constexpr (DT == CKV_FP32) return div_rcp(acc, scale, inv_scale);
  if constexpr (DT == CKV_FP16) return round_dt<DT>(div_rcp(round_dt<DT>(acc), scale, inv_scale));
  return round_dt<DT>(round_dt<DT>(acc) * inv_scale);
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
// Called by every thread of the block (>= 64 threads); ent / mass in shared or
// global memory, visible to all.  Ranks are computed one head per thread.
__device__ void select_heads(const ckv_params& p, int H, const float* ent, const float* mass,
                             uint64_t* qi_set, uint64_t* hi_set, int* hi_mode, int* n_hi) {
  __shared__ unsigned long long sq, sh_, ssel;
  __shared__ int s_order[kMaxHeads];
  __shared__ int s_mode, s_nhi;
  const uint64_t all = (H >= 64) ? ~0ull : ((1ull << H) - 1);
  const int h = threadIdx.x;
  if (h == 0) { sq = 0; sh_ = 0; ssel = 0; }
  __syncthreads();
  if (!p.entropy_aware) {
    *qi_set = all; *hi_set = all; *hi_mode = 2; *n_hi = H;
    return;
  }
  const int k = min(p.top_k_heads, H);
  int rank_q = 0, rank_m = 0;
  if (h < H) {
    for (int o = 0; o < H; ++o) {
      const bool bq = (p.head_selection_mode == 1) ? (mass[o] > mass[h] || (mass[o] == mass[h] && o < h))
                                                   : (ent[o] < ent[h] || (ent[o] == ent[h] && o < h));
      rank_q += bq ? 1 : 0;
      rank_m += (mass[o] > mass[h] || (mass[o] == mass[h] && o < h)) ? 1 : 0;   // descending mass
    }
    if (rank_q < k) atomicOr(&sq, 1ull << h);
    s_order[rank_m] = h;
  }
  __syncthreads();
  if (h == 0) {
    uint64_t hs = all;
    int mode = 0;
    if (p.hi_pooling_mode == 1) {
      mode = 1;
    } else if (p.hi_mass_cdf > 0.f) {
      float total = 0.f;
      for (int o = 0; o < H; ++o) total += mass[o];
      if (total > 0.f) {
        float cum = 0.f;
        int below = 0;
        for (int i = 0; i < H; ++i) { cum += mass[s_order[i]]; if (cum / total < p.hi_mass_cdf) ++below; }
        const int need = min(below + 1, H);
        hs = 0;
        for (int i = 0; i < need; ++i) hs |= 1ull << s_order[i];
      }
    } else if (p.hi_top_k_heads > 0) {
      const int kh = min(p.hi_top_k_heads, H);
      hs = 0;
      for (int i = 0; i < kh; ++i) hs |= 1ull << s_order[i];
    } else if (p.hi_mass_threshold > 0.f) {
      hs = 0;
      for (int o = 0; o < H; ++o)
        if (mass[o] >= p.hi_mass_threshold) hs |= 1ull << o;
      if (hs == 0) hs = all;
    }
    sh_ = hs;
    s_mode = mode;
    s_nhi = __popcll(hs);
  }
  __syncthreads();
  *qi_set = sq; *hi_set = sh_; *hi_mode = s_mode; *n_hi = s_nhi;
  __syncthreads();
}

// Whether the head sets chosen from the moments pass's entropies and masses are the
// ones the exact values would give (one thread).  The exact entropy of head h lies in
// [ent[h], ent[h] + bnd[h]] (the clamp at 1e-8 only raises it; bnd bounds the raise),
// up to rounding; the exact mass equals the moments pass's up to rounding.  A decision
// is certain when every margin it depends on exceeds the bound plus a rounding slack
// of 1e-5 relative; otherwise the pooling pass recomputes both exactly (and, if the
// sets change, re-runs).  The slack is orders of magnitude above the fp32 rounding of
// either computation.
CKV_DEV float certainty_slack(float a, float b) { return 1e-5f * fmaxf(fabsf(a), fabsf(b)) + 1e-6f; }

__device__ bool selection_certain(const ckv_params& p, int H, const float* ent, const float* mass,
                                  const float* bnd, uint64_t qs) {
  if (!p.entropy_aware) return true;
  const int k = min(p.top_k_heads, H);
  if (k < H) {
    if (p.head_selection_mode == 1) {   // QI: the k heads of largest mass
      float lo_in = INFINITY, hi_out = -INFINITY;
      for (int h = 0; h < H; ++h) {
        if ((qs >> h) & 1ull) lo_in = fminf(lo_in, mass[h]);
        else hi_out = fmaxf(hi_out, mass[h]);
      }
      if (!(lo_in - hi_out > certainty_slack(lo_in, hi_out))) return false;
    } else {                            // QI: the k heads of smallest entropy
      float hi_in = -INFINITY, lo_out = INFINITY;
      for (int h = 0; h < H; ++h) {
        if ((qs >> h) & 1ull) hi_in = fmaxf(hi_in, ent[h] + bnd[h]);
        else lo_out = fminf(lo_out, ent[h]);
      }
      if (!(lo_out - hi_in > certainty_slack(hi_in, lo_out))) return false;
    }
  }
  if (p.hi_pooling_mode == 1) return true;   // HI: every head
  if (p.hi_mass_cdf > 0.f || p.hi_top_k_heads > 0) {
    // masses in descending order with clear gaps, and clear CDF crossings
    float prev = INFINITY, cum = 0.f, total = 0.f;
    for (int h = 0; h < H; ++h) total += mass[h];
    uint64_t used = 0;
    for (int i = 0; i < H; ++i) {
      int best = -1;
      for (int h = 0; h < H; ++h)
        if (!((used >> h) & 1ull) && (best < 0 || mass[h] > mass[best])) best = h;
      used |= 1ull << best;
      const float m = mass[best];
      if (i > 0 && !(prev - m > certainty_slack(prev, m))) return false;
      prev = m;
      cum += m;
      if (p.hi_mass_cdf > 0.f && total > 0.f && !(fabsf(cum / total - p.hi_mass_cdf) > 1e-5f)) return false;
    }
    return true;
  }
  if (p.hi_mass_threshold > 0.f)
    for (int h = 0; h < H; ++h)
      if (!(fabsf(mass[h] - p.hi_mass_threshold) > certainty_slack(mass[h], p.hi_mass_threshold))) return false;
  return true;
}

// The same head sets (and their certainty) computed by ONE warp for H <= 32: lane h holds
// head h's entropy, mass and clamp bound in registers, ranks come from 32 shuffles, sets from
// ballots and the certainty margins from warp max / min reductions.  It runs once per layer
// at the end of a pass, as cold code on one SM, so it keeps to one short loop and no
// shared-memory round trips (the block-wide form above spent ~10 us there).  Same
// decisions as select_heads / selection_certain; the CDF mode keeps their sequential
// fp32 running sum (lane 0, in mass order).
struct HeadSets {
  uint64_t qs, hs;
  int hm, nhi, certain;
};

// The parameters the head selection reads (passed by value: the noinline function below
// has one copy of its code, which a warm-up warp can run ahead of time).
struct HeadSelParams {
  int entropy_aware, top_k_heads, head_selection_mode, hi_pooling_mode, hi_top_k_heads;
  float hi_mass_cdf, hi_mass_threshold;
};

__device__ __noinline__ HeadSets select_heads_warp_impl(const HeadSelParams p, int H, float ent, float mass, float bnd) {
  const int lane = threadIdx.x & 31;
  const bool valid = lane < H;
  const uint32_t all32 = H >= 32 ? 0xffffffffu : ((1u << H) - 1u);
  HeadSets r;
  r.certain = 1;
  if (!p.entropy_aware) {
    r.qs = all32; r.hs = all32; r.hm = 2; r.nhi = H;
    return r;
  }
  const int k = min(p.top_k_heads, H);
  const bool by_mass = p.head_selection_mode == 1;
  int rank_q = 0, rank_m = 0;
  for (int o = 0; o < H; ++o) {
    const float eo = __shfl_sync(0xffffffffu, ent, o), mo = __shfl_sync(0xffffffffu, mass, o);
    rank_q += (by_mass ? (mo > mass || (mo == mass && o < lane)) : (eo < ent || (eo == ent && o < lane))) ? 1 : 0;
    rank_m += (mo > mass || (mo == mass && o < lane)) ? 1 : 0;   // descending mass
  }
  const uint32_t qs = __ballot_sync(0xffffffffu, valid && rank_q < k);
  uint32_t hs = all32;
  int mode = 0;
  __shared__ float s_sorted[32];
  if (p.hi_pooling_mode == 1) {
    mode = 1;
  } else if (p.hi_mass_cdf > 0.f || p.hi_top_k_heads > 0) {
    if (valid) s_sorted[rank_m] = mass;
    __syncwarp();
    if (p.hi_mass_cdf > 0.f) {
      int need = H;
      // the running sum in mass order, sequential as the block-wide form (lane 0)
      float total = 0.f;
      for (int o = 0; o < H; ++o) total += __shfl_sync(0xffffffffu, mass, o);
      int below = 0;
      if (total > 0.f) {
        if (lane == 0) {
          float cum = 0.f;
          for (int i = 0; i < H; ++i) { cum += s_sorted[i]; if (cum / total < p.hi_mass_cdf) ++below; }
        }
        below = __shfl_sync(0xffffffffu, below, 0);
        need = min(below + 1, H);
        hs = __ballot_sync(0xffffffffu, valid && rank_m < need);
      }
    } else {
      hs = __ballot_sync(0xffffffffu, valid && rank_m < min(p.hi_top_k_heads, H));
    }
  } else if (p.hi_mass_threshold > 0.f) {
    hs = __ballot_sync(0xffffffffu, valid && mass >= p.hi_mass_threshold);
    if (hs == 0) hs = all32;
  }
  r.qs = qs; r.hs = hs; r.hm = mode; r.nhi = __popc(hs);
  // certainty of the decisions (selection_certain)
  bool ok = true;
  const bool in_q = (qs >> lane) & 1u;
  if (k < H) {
    if (by_mass) {
      const float lo_in = warp_min(valid && in_q ? mass : INFINITY);
      const float hi_out = warp_max(valid && !in_q ? mass : -INFINITY);
      ok = lo_in - hi_out > certainty_slack(lo_in, hi_out);
    } else {
      const float hi_in = warp_max(valid && in_q ? ent + bnd : -INFINITY);
      const float lo_out = warp_min(valid && !in_q ? ent : INFINITY);
      ok = lo_out - hi_in > certainty_slack(hi_in, lo_out);
    }
  }
  if (ok && p.hi_pooling_mode != 1) {
    if (p.hi_mass_cdf > 0.f || p.hi_top_k_heads > 0) {
      // masses in descending order with clear gaps, and clear CDF crossings
      float total = 0.f;
      for (int o = 0; o < H; ++o) total += __shfl_sync(0xffffffffu, mass, o);
      int bad = 0;
      if (lane == 0) {
        float prev = INFINITY, cum = 0.f;
        for (int i = 0; i < H && !bad; ++i) {
          const float m = s_sorted[i];
          if (i > 0 && !(prev - m > certainty_slack(prev, m))) bad = 1;
          prev = m;
          cum += m;
          if (p.hi_mass_cdf > 0.f && total > 0.f && !(fabsf(cum / total - p.hi_mass_cdf) > 1e-5f)) bad = 1;
        }
      }
      ok = __shfl_sync(0xffffffffu, bad, 0) == 0;
    } else if (p.hi_mass_threshold > 0.f) {
      ok = __ballot_sync(0xffffffffu, valid && !(fabsf(mass - p.hi_mass_threshold) >
                                                 certainty_slack(mass, p.hi_mass_threshold))) == 0;
    }
  }
  r.certain = ok ? 1 : 0;
  return r;
}

CKV_DEV HeadSelParams head_sel_params(const ckv_params& p) {
  HeadSelParams q;
  q.entropy_aware = p.entropy_aware; q.top_k_heads = p.top_k_heads;
  q.head_selection_mode = p.head_selection_mode; q.hi_pooling_mode = p.hi_pooling_mode;
  q.hi_top_k_heads = p.hi_top_k_heads; q.hi_mass_cdf = p.hi_mass_cdf; q.hi_mass_threshold = p.hi_mass_threshold;
  return q;
}
CKV_DEV HeadSets select_heads_warp(const ckv_params& p, int H, float ent, float mass, float bnd) {
  return select_heads_warp_impl(head_sel_params(p), H, ent, mass, bnd);
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
  const float inv_scale = 1.0f / scale;
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
            if (j <= lim) v = logit_of<DT>(acc[mt][nt][2 * hf + e], scale, inv_scale) * kLog2e;
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

  stats_finish(a, smem, bg.h0, pl.heads_per_batch, blockIdx.y, gridDim.x, gridDim.y);
}

// The last CTA of a head group: merges the chunk partials of the group's rows into their
// log-sum-exp (to lse), the unclamped entropy, the transient mass and the clamp bound (to
// rowE / rowM / rowB); thread tid of nthreads.  dry: the same loads and arithmetic with
// every store switched off (the moments pass's warm-up warp runs it ahead of time, so the
// instructions are in the SM's cache when a last CTA needs them: this code runs once per
// layer on a few SMs and otherwise spends most of its time being fetched).
__device__ __noinline__ void merge_group_rows(const float4* part, const float* minx, float* lse, float* rowE,
                                              float* rowM, float* rowB, int H, int W, int n, int nchunks, int tc_min,
                                              int i0, int nrows, int tid, int nthreads, bool dry) {
  // tpr consecutive lanes share a row; each merges every tpr-th chunk, 8 loads in flight
  int tpr = 1;
  while (tpr < 8 && tpr * 2 * nrows <= nthreads) tpr *= 2;
  const int sub = tid % tpr;
  for (int base = 0; base < nrows * tpr; base += nthreads) {
    const int li = (base + tid) / tpr;
    const bool valid = li < nrows;
    Moments M{-INFINITY, 0.f, 0.f, 0.f};
    float xmin = INFINITY;
    if (valid) {
      for (int c0 = sub; c0 < nchunks; c0 += 8 * tpr) {
        float4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (c0 + u * tpr < nchunks) v[u] = __ldcg(part + (size_t)(c0 + u * tpr) * H * W + i0 + li);
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (c0 + u * tpr < nchunks) M = merge(M, Moments{v[u].x, v[u].y, v[u].z, v[u].w});
        if (tc_min)
          for (int u = 0; u < 8; ++u)
            if (c0 + u * tpr < nchunks) xmin = fminf(xmin, __ldcg(minx + (size_t)(c0 + u * tpr) * H * W + i0 + li));
      }
    }
    for (int o = 1; o < tpr; o <<= 1) {   // lanes of one row are consecutive within a warp
      Moments O;
      O.m = __shfl_xor_sync(0xffffffffu, M.m, o);
      O.z = __shfl_xor_sync(0xffffffffu, M.z, o);
      O.t = __shfl_xor_sync(0xffffffffu, M.t, o);
      O.s = __shfl_xor_sync(0xffffffffu, M.s, o);
      M = merge(M, O);
      xmin = fminf(xmin, __shfl_xor_sync(0xffffffffu, xmin, o));
    }
    if (valid && sub == 0) {
      const float l2z = log2f(M.z);
      const float iz = 1.0f / M.z;
      const float L = M.m + l2z;
      const int r = li % W;
      const float e = l2z * kLn2 - kLn2 * div_rcp(M.t, M.z, iz) + (float)(W - 1 - r) * kGeps;
      const float m = 1.f - div_rcp(M.s, M.z, iz);
      // the clamp at 1e-8 adds at most kGeps per visible entry to the row's entropy; a
      // row whose smallest probability is above the clamp (with margin) adds nothing
      const bool clamp_free = tc_min && fmaf(xmin, kLog2e, -L) >= kLog2Eps + 1e-3f;
      const float bnd = clamp_free ? 0.f : (float)(n - W + r + 1) * kGeps;
      if (!dry) {
        lse[i0 + li] = L;
        rowE[li] = e;
        rowM[li] = m;
        rowB[li] = bnd;
      }
    }
  }
}

// Per-head means of the merged rows (warp `warp` of nw takes heads warp, warp + nw, ...);
// dry as above.
__device__ __noinline__ void group_head_means(const float* rowE, const float* rowM, const float* rowB, float* spec,
                                              int H, int W, int tc_min, int h0, int nh, int warp, int nw, bool dry) {
  const int lane = threadIdx.x & 31;
  for (int hl = warp; hl < nh; hl += nw) {
    float e = 0.f, m = 0.f, b = 0.f;
    for (int r = lane; r < W; r += 32) {
      e += rowE[hl * W + r]; m += rowM[hl * W + r]; b += rowB[hl * W + r];
    }
    e = warp_sum(e);
    m = warp_sum(m);
    b = warp_sum(b);
    if (lane == 0 && !dry) {
      spec[h0 + hl] = e / (float)W;
      spec[H + h0 + hl] = m / (float)W;
      spec[4 * H + h0 + hl] = tc_min ? b / (float)W : INFINITY;
    }
  }
}

// Last-CTA steps of the moments pass (PU:2905-2999).  The last CTA of each head
// group merges the chunk partials of the group's rows into their log-sum-exp, the
// unclamped entropy and the transient mass, and writes the group's per-head means;
// the last group then speculates the head sets from them.
__device__ void stats_finish(const WinArgs& a, char* smem, int h0, int nh, int gidx, int per_group, int ngroups) {
  const Plan& pl = a.pl;
  const float4* part = reinterpret_cast<const float4*>(a.ws + pl.off_stats);
  Header* hdr = reinterpret_cast<Header*>(a.ws);
  __shared__ bool last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(&hdr->cnt_group[gidx], 1u) == (unsigned)per_group - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  float* lse = reinterpret_cast<float*>(a.ws + pl.off_lse);
  float* spec = reinterpret_cast<float*>(a.ws + pl.off_spec);   // [H] entropy, [H] mass; [4H..5H) bounds
  const float* minx = reinterpret_cast<const float*>(a.ws + pl.off_minx);
  const int nrows = nh * pl.W, i0 = h0 * pl.W;
  float* rowE = reinterpret_cast<float*>(smem);                  // [nrows]
  float* rowM = rowE + nrows;
  float* rowB = rowM + nrows;
  merge_group_rows(part, minx, lse, rowE, rowM, rowB, pl.H, pl.W, pl.n, pl.nstat_chunks, a.tc_min, i0, nrows,
                   threadIdx.x, blockDim.x, false);
  __syncthreads();
  group_head_means(rowE, rowM, rowB, spec, pl.H, pl.W, a.tc_min, h0, nh, threadIdx.x >> 5, blockDim.x >> 5, false);
  // the last group selects the heads
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    hdr->cnt_group[gidx] = 0;
    last = atomicAdd(&hdr->cnt_stats, 1u) == (unsigned)ngroups - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (pl.H <= 32) {   // one warp, registers and shuffles
    if (threadIdx.x < 32) {
      const int h = threadIdx.x;
      const bool v = h < pl.H;
      const float e = v ? __ldcg(spec + h) : INFINITY;
      const float m = v ? __ldcg(spec + pl.H + h) : -INFINITY;
      const float b = v ? __ldcg(spec + 4 * pl.H + h) : 0.f;
      const HeadSets r = select_heads_warp(a.p, pl.H, e, m, b);
      if (h == 0) {
        hdr->qi_heads = r.qs;
        hdr->hi_heads = r.hs;
        hdr->hi_mode = r.hm;
        hdr->n_hi = r.nhi;
        hdr->fixup = 0;
        hdr->cnt_stats = 0;
        hdr->need_exact = (a.force_exact || !(pl.tc_pool || pl.lanes_pool) || !r.certain) ? 1 : 0;
      }
    }
    return;
  }
  float* sSpec = rowE;                                           // [2H] + [H] bounds
  for (int h = threadIdx.x; h < 2 * pl.H; h += blockDim.x) sSpec[h] = __ldcg(spec + h);
  for (int h = threadIdx.x; h < pl.H; h += blockDim.x) sSpec[2 * pl.H + h] = __ldcg(spec + 4 * pl.H + h);
  __syncthreads();
  uint64_t qs, hs;
  int hm, nhi;
  select_heads(a.p, pl.H, sSpec, sSpec + pl.H, &qs, &hs, &hm, &nhi);
  if (threadIdx.x == 0) {
    hdr->qi_heads = qs;
    hdr->hi_heads = hs;
    hdr->hi_mode = hm;
    hdr->n_hi = nhi;
    hdr->fixup = 0;
    hdr->cnt_stats = 0;
    hdr->need_exact = (a.force_exact || !(pl.tc_pool || pl.lanes_pool) ||
                       !selection_certain(a.p, pl.H, sSpec, sSpec + pl.H, sSpec + 2 * pl.H, qs)) ? 1 : 0;
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
  // with a keys-on-lanes pass beside it, this pass runs only when the head sets need the
  // exact recomputation (or for the re-run)
  if (pl.lanes_pool && !a.fixup_pass && *reinterpret_cast<volatile int32_t*>(&hdr->need_exact) == 0) return;

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
  const float inv_nhi = 1.0f / (float)(nhi > 0 ? nhi : 1);   // mean = sum * (1 / count)
  const float* lse = reinterpret_cast<const float*>(a.ws + pl.off_lse);
  float* epart = reinterpret_cast<float*>(a.ws + pl.off_epart);
  float* mpart = reinterpret_cast<float*>(a.ws + pl.off_mpart);
  const float scale = sqrtf((float)pl.D);
  const float inv_scale = 1.0f / scale;

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
              const float y = logit_of<DT>(acc[mt][nt][2 * hf + e], scale, inv_scale) * kLog2e;
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
        float v = ch == 0 ? qacc[i] : (hmode == 1 ? hacc[i] : hacc[i] * inv_nhi);
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
      rspart[((size_t)ch * pl.rs_parts + tile) * pl.W + r] = sRed[i][w] + sRed[i][w + 1];
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
    if (threadIdx.x == 0) gtile[(size_t)ch * pl.ncol_tiles * 8 + tile] = red[0] + red[1];
    __syncthreads();
  }

}

// ---------------------------------------------------------------------------
// per-head eviction pass (PU:2208-2382)
// ---------------------------------------------------------------------------
// Exact window probabilities (as in the pooling pass) reduced per head and column:
// the query row p[h, W-1, j], the two-hop term sum_r q2w[h, r] p[h, r, j] with
// q2w[h, r] = p[h, W-1, n-W+r], the column sum over the window rows, and the
// query row's entropy partial sum_j p ln(p + 1e-10) per tile.  The prelude launch
// covers only the tiles holding the window columns and writes q2w from the same
// MMA tiles, so both launches see bit-identical probabilities.
template <int DT>
__global__ void __launch_bounds__(256) k_ph_pass(WinArgs a, int prelude) {
  using WT = WarpTile<DT>;
  constexpr int MT = WT::MT;
  extern __shared__ __align__(128) char smem[];
  const Plan& pl = a.pl;
  const int tile = prelude ? (pl.n_p / kColTile + (int)blockIdx.x) : (int)blockIdx.x;
  const int j0 = tile * kColTile;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  char* sQ = smem;
  char* sK = sQ + pl.rows_per_batch * row_bytes<DT>();
  float* sP = reinterpret_cast<float*>(sK + pl.ktiles_per_batch * kColTile * row_bytes<DT>());
  const char** srcs =
      reinterpret_cast<const char**>(sP + pl.rows_per_batch * kStageStride) + 1;
  __shared__ float sq2w[kWarps * 32];            // the batch's q2w rows (rows_per_batch <= 256)
  __shared__ float part[2][4][kColTile];
  __shared__ float entw[2];
  const float* lse = reinterpret_cast<const float*>(a.ws + pl.off_lse);
  float* q2w = reinterpret_cast<float*>(a.ws + pl.off_ph_q2w);
  float* qrow = reinterpret_cast<float*>(a.ws + pl.off_ph_qrow);
  float* two = reinterpret_cast<float*>(a.ws + pl.off_ph_two);
  float* col = reinterpret_cast<float*>(a.ws + pl.off_ph_col);
  float* entp = reinterpret_cast<float*>(a.ws + pl.off_ph_ent);
  const float scale = sqrtf((float)pl.D);
  const float inv_scale = 1.0f / scale;
  const int pc = threadIdx.x % kColTile, pr0 = threadIdx.x / kColTile;
  const int W = pl.W;
  for (int b = 0; b < pl.nbatch; ++b) {
    const BatchGeom bg = batch_geom(pl, b);
    __syncthreads();
    stage_q<DT>(a, bg, sQ, srcs);
    stage_k<DT>(a, bg, j0, sK, srcs);
    cp_async_commit();
    if (!prelude)
      for (int i = threadIdx.x; i < pl.heads_per_batch * W; i += blockDim.x) sq2w[i] = __ldcg(q2w + bg.h0 * W + i);
    cp_async_wait<0>();
    __syncthreads();
    const int row0 = warp * pl.rows_per_warp;
    const int hl = row0 / W;
    const int kt = (bg.h0 + hl) / pl.G - bg.g0;
    float acc[MT][8][4];
    WT::compute(sQ, sK + kt * kColTile * row_bytes<DT>(), row0, acc);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int rl = row0 + mt * 16 + (lane >> 2) + 8 * hf;
        const int h = bg.h0 + rl / W, r = rl % W;
        const int lim = pl.n - W + r;
        const float L = lse[h * W + r];
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          float pv[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int j = j0 + nt * 8 + 2 * (lane & 3) + e;
            float p = 0.f;
            if (j <= lim) p = ex2(logit_of<DT>(acc[mt][nt][2 * hf + e], scale, inv_scale) * kLog2e - L);
            pv[e] = p;
          }
          *reinterpret_cast<float2*>(sP + rl * kStageStride + nt * 8 + 2 * (lane & 3)) =
              make_float2(pv[0], pv[1]);
        }
      }
    __syncthreads();
    if (prelude) {
      for (int i = threadIdx.x; i < pl.heads_per_batch * kColTile; i += blockDim.x) {
        const int hh = i / kColTile, c = i % kColTile, j = j0 + c;
        if (j >= pl.n_p && j < pl.n) q2w[(bg.h0 + hh) * W + (j - pl.n_p)] = sP[(hh * W + W - 1) * kStageStride + c];
      }
      continue;
    }
    for (int hh = 0; hh < pl.heads_per_batch; ++hh) {
      const int h = bg.h0 + hh;
      float s2 = 0.f, sc = 0.f;
      for (int r = pr0; r < W; r += 4) {
        const float p = sP[(hh * W + r) * kStageStride + pc];
        s2 = fmaf(sq2w[hh * W + r], p, s2);
        sc += p;
      }
      part[0][pr0][pc] = s2;
      part[1][pr0][pc] = sc;
      __syncthreads();
      if (threadIdx.x < kColTile) {
        const int j = j0 + threadIdx.x;
        const float qa = sP[(hh * W + W - 1) * kStageStride + threadIdx.x];
        if (j < pl.n) {
          two[(size_t)h * pl.n + j] = (part[0][0][threadIdx.x] + part[0][1][threadIdx.x]) +
                                      (part[0][2][threadIdx.x] + part[0][3][threadIdx.x]);
          col[(size_t)h * pl.n + j] = (part[1][0][threadIdx.x] + part[1][1][threadIdx.x]) +
                                      (part[1][2][threadIdx.x] + part[1][3][threadIdx.x]);
          qrow[(size_t)h * pl.n + j] = qa;
        }
        const float t = j < pl.n ? qa * logf(qa + 1e-10f) : 0.f;
        const float ws_ = warp_sum(t);
        if (lane == 0) entw[warp] = ws_;
      }
      __syncthreads();
      if (threadIdx.x == 0) entp[(size_t)tile * pl.H + h] = entw[0] + entw[1];
    }
  }
}

template <int DT>
static cudaError_t launch_ph_pass_t(const WinArgs& a, cudaStream_t st) {
  const Plan& pl = a.pl;
  const size_t sm = pool_smem<DT>(pl);
  { const cudaError_t e = ensure_dynamic_smem((const void*)k_ph_pass<DT>, sm); if (e != cudaSuccess) return e; }
  const int t0 = pl.n_p / kColTile, t1 = (pl.n - 1) / kColTile;
  k_ph_pass<DT><<<t1 - t0 + 1, 256, sm, st>>>(a, 1);
  k_ph_pass<DT><<<pl.ncol_tiles, 256, sm, st>>>(a, 0);
  return cudaGetLastError();
}

static cudaError_t launch_ph_pass_mma(const WinArgs& a, cudaStream_t st) {
  switch (a.pl.dtype) {
    case CKV_BF16: return launch_ph_pass_t<CKV_BF16>(a, st);
    case CKV_FP16: return launch_ph_pass_t<CKV_FP16>(a, st);
    default: return launch_ph_pass_t<CKV_FP32>(a, st);
  }
}

// ---------------------------------------------------------------------------
// window chains: the W x W block of the pooled rows (PU:2060-2206)
// ---------------------------------------------------------------------------
// Shared memory of the chain step, in floats: the raw then normalised window blocks
// [2][W][W], row sums and their reciprocals [2][W] each, the fallback iteration's
// vectors / partials / maxima, and (pooling finish only, before the chains) the row
// entropies and masses [2][H*W] and the per-head means [2][H] in the same region.
struct ChainSmem {
  size_t pw, rs, inv, y, part, mx, rowe, head, total;
};
__host__ __device__ inline ChainSmem chain_smem(int W, int H) {
  ChainSmem c;
  size_t off = 0;
  c.pw = off; off += (size_t)2 * W * W;
  c.rs = off; off += (size_t)2 * W;
  c.inv = off; off += (size_t)2 * W;
  // the fallback iteration's scratch and the pooling finish's row statistics are
  // never live together: they share one region
  const size_t shared0 = off;
  c.y = off; off += (size_t)4 * W;
  c.part = off; off += (size_t)2 * 32 * kMaxWindow;
  c.mx = off; off += 64;
  const size_t end_fallback = off;
  off = shared0;
  c.rowe = off; off += (size_t)2 * H * W;
  c.head = off; off += (size_t)2 * H;
  c.total = off > end_fallback ? off : end_fallback;
  return c;
}

CKV_DEV void cp_async4(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(smem_u32(smem)), "l"(gmem));
}

// Start copying the window block of each chain's pooled rows (columns n_p .. n-1 of
// its W rows) into shared memory; completes at cp_async_wait<0>().
__device__ __forceinline__ void stage_window_block(const Plan& pl, const char* ws, float* smem) {
  const ChainSmem cs = chain_smem(pl.W, pl.H);
  const int W = pl.W, nw = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* rows0 = reinterpret_cast<const float*>(ws + pl.off_rows_qi);
  const float* rows1 = reinterpret_cast<const float*>(ws + (pl.hi_rows ? pl.off_rows_hi : pl.off_rows_qi));
  for (int g = warp; g < pl.nchains * W; g += nw) {
    const int ch = g >= W ? 1 : 0, r = g - ch * W;
    const float* src = (ch ? rows1 : rows0) + (size_t)r * pl.n_pad + pl.n_p;
    for (int c = lane; c < W; c += 32) cp_async4(smem + cs.pw + (size_t)g * W + c, src + c);
  }
  cp_async_commit();
}

// One chain on one warp, W = 32 * KC: lane l holds y[l + 32 q]; the rows of Pww are
// read from shared memory at fixed offsets and y[r] is broadcast by a shuffle.  Pww
// is causal (Pww[r, c] = 0 for c > r), so summing every row in ascending order adds
// exact zeros before row c and matches the triangular sum bit for bit.
template <int KC>
__device__ __forceinline__ void chain_warp(const float* Pw, const float* rs, const float* inv, int K, float gam,
                                           float y0_uniform, bool query_start, float* yk, float* wk,
                                           float* ymax) {
  constexpr int W = 32 * KC;
  const int lane = threadIdx.x & 31;
  float y[KC];
#pragma unroll
  for (int q = 0; q < KC; ++q) {
    const int c = lane + 32 * q;
    y[q] = query_start ? (c == W - 1 ? 1.f : 0.f) : y0_uniform;
  }
  for (int k = 0; k <= K; ++k) {
    float mx = 0.f;
#pragma unroll
    for (int q = 0; q < KC; ++q) {
      const int c = lane + 32 * q;
      yk[(size_t)k * W + c] = y[q];
      if (k < K) wk[(size_t)k * W + c] = div_rcp(gam * y[q], rs[c], inv[c]);
      mx = fmaxf(mx, fabsf(y[q]));
    }
    mx = warp_max(mx);
    if (lane == 0) ymax[k] = mx;
    if (k == K) break;
    float s[KC];
#pragma unroll
    for (int q = 0; q < KC; ++q) s[q] = 0.f;
#pragma unroll
    for (int rq = 0; rq < KC; ++rq) {
#pragma unroll
      for (int l = 0; l < 32; ++l) {
        const float yr = __shfl_sync(0xffffffffu, y[rq], l);
        const int r = 32 * rq + l;
#pragma unroll
        for (int q = 0; q < KC; ++q) s[q] = fmaf(Pw[r * W + lane + 32 * q], yr, s[q]);
      }
    }
#pragma unroll
    for (int q = 0; q < KC; ++q) y[q] = gam * s[q];
  }
}

// Row sums (tempered) of the pooled rows and the W x W window chain of each
// absorbing chain: y_0 (query one-hot or uniform), y_{k+1} = gamma * Pww^T y_k.
// Writes y_k, the weights w_k = gamma * y_k / rowsum used by the prefix sweep,
// and max_c y_k.  One CTA; the window block is being copied by stage_window_block.
// W a multiple of 32 (<= 128): one warp per chain (chain_warp).  Otherwise the
// chains run side by side on half of the warps each with a named barrier: warp j
// sums its block of rows for every column and the partials are added in row order.
__device__ __forceinline__ void run_window_chains(const Plan& pl, const ckv_params& prm, char* ws, float* smem,
                                                  bool use_rowsums) {
  const ChainSmem cs = chain_smem(pl.W, pl.H);
  const int W = pl.W, K = pl.K;
  const bool tempered = prm.neumann_temperature != 1.0f && prm.neumann_temperature > 0.f;
  const float invT = tempered ? 1.0f / prm.neumann_temperature : 1.0f;
  const float gam = prm.neumann_gamma;
  const float* rspart = reinterpret_cast<const float*>(ws + pl.off_rspart);
  const float* rowS = reinterpret_cast<const float*>(ws + pl.off_stats) + 2 * pl.H * W;   // from k_pool_reduce
  float* wk = reinterpret_cast<float*>(ws + pl.off_wk);     // [2][K][W]
  float* yk = reinterpret_cast<float*>(ws + pl.off_yk);     // [2][K+1][W]
  float* ymax = reinterpret_cast<float*>(ws + pl.off_ymax); // [2][K+1]
  float* sPw = smem + cs.pw;
  float* sRs = smem + cs.rs;
  float* sInv = smem + cs.inv;
  const int nchain = pl.nchains;
  for (int i = threadIdx.x; i < nchain * W; i += blockDim.x) {
    const int ch = i / W, r = i % W;
    const int src = (ch == 0 || pl.hi_rows) ? ch : 0;
    const float s = use_rowsums ? __ldcg(rowS + ch * W + r)
                                : sum_parts(rspart + (size_t)src * pl.rs_parts * W + r, pl.rs_parts, (size_t)W, 0, 1);
    sRs[i] = fmaxf(s, 1e-8f);
    sInv[i] = 1.0f / sRs[i];
  }
  cp_async_wait<0>();
  __syncthreads();
  for (int i = threadIdx.x; i < nchain * W * W; i += blockDim.x) {
    float x = sPw[i];
    if (tempered) x = x > 0.f ? powf(x, invT) : 0.f;
    const int g = i / W;
    sPw[i] = div_rcp(x, sRs[g], sInv[g]);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const float u0 = 1.0f / (float)(pl.n - pl.s);
  if (W % 32 == 0 && W <= kMaxWindow) {
    if (warp < nchain) {
      const int ch = warp;
      const float* Pw = sPw + (size_t)ch * W * W;
      float* yko = yk + (size_t)ch * (K + 1) * W;
      float* wko = wk + (size_t)ch * K * W;
      float* ymo = ymax + ch * (K + 1);
      switch (W / 32) {
        case 1: chain_warp<1>(Pw, sRs + ch * W, sInv + ch * W, K, gam, u0, ch == 0, yko, wko, ymo); break;
        case 2: chain_warp<2>(Pw, sRs + ch * W, sInv + ch * W, K, gam, u0, ch == 0, yko, wko, ymo); break;
        case 3: chain_warp<3>(Pw, sRs + ch * W, sInv + ch * W, K, gam, u0, ch == 0, yko, wko, ymo); break;
        default: chain_warp<4>(Pw, sRs + ch * W, sInv + ch * W, K, gam, u0, ch == 0, yko, wko, ymo); break;
      }
    }
    __syncthreads();
    return;
  }
  float* sY = smem + cs.y;                                    // [2][2][W]
  float* sPart = smem + cs.part;                              // [2][32][W]
  float* sMx = smem + cs.mx;                                  // [2][32]
  const int wpc = min(32, nw / nchain);                       // warps per chain
  const int tpc = wpc * 32;
  const int ch = warp / wpc;
  if (ch < nchain) {
    const int j = warp - ch * wpc;                            // row block of this warp
    const int ct = threadIdx.x - ch * tpc;
    const int rpw = (W + wpc - 1) / wpc;
    const int r0 = min(W, j * rpw), r1 = min(W, r0 + rpw);
    const float* Pw = sPw + (size_t)ch * W * W;
    const float* rs = sRs + ch * W;
    const float* inv = sInv + ch * W;
    float* Y = sY + ch * 2 * W;
    float* part = sPart + ch * 32 * kMaxWindow;
    float* mxw = sMx + ch * 32;
    auto chain_sync = [&]() { asm volatile("bar.sync %0, %1;" ::"r"(1 + ch), "r"(tpc) : "memory"); };
    for (int c = ct; c < W; c += tpc) Y[c] = (ch == 0) ? (c == W - 1 ? 1.f : 0.f) : u0;
    chain_sync();
    for (int k = 0; k <= K; ++k) {
      const float* cur = Y + (k & 1) * W;
      float* nxt = Y + ((k + 1) & 1) * W;
      if (k < K) {
        float s[kMaxWindow / 32];
#pragma unroll
        for (int q = 0; q < kMaxWindow / 32; ++q) s[q] = 0.f;
        for (int r = r0; r < r1; ++r) {
          const float yr = cur[r];
#pragma unroll
          for (int q = 0; q < kMaxWindow / 32; ++q) {
            const int c = lane + 32 * q;
            if (c < W) s[q] = fmaf(Pw[r * W + c], yr, s[q]);
          }
        }
#pragma unroll
        for (int q = 0; q < kMaxWindow / 32; ++q) {
          const int c = lane + 32 * q;
          if (c < W) part[j * W + c] = s[q];
        }
      }
      float mx = 0.f;
      for (int c = ct; c < W; c += tpc) {
        const float y = cur[c];
        yk[((size_t)ch * (K + 1) + k) * W + c] = y;
        if (k < K) wk[((size_t)ch * K + k) * W + c] = div_rcp(gam * y, rs[c], inv[c]);
        mx = fmaxf(mx, fabsf(y));
      }
      mx = warp_max(mx);
      if (lane == 0) mxw[j] = mx;
      chain_sync();
      if (ct == 0) {
        float m = 0.f;
        for (int i = 0; i < wpc; ++i) m = fmaxf(m, mxw[i]);
        ymax[ch * (K + 1) + k] = m;
      }
      if (k < K)
        for (int c = ct; c < W; c += tpc) {
          float t = 0.f;
          for (int b = 0; b < wpc; ++b) t += part[b * W + c];
          nxt[c] = gam * t;
        }
      chain_sync();
    }
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// last-CTA work of the pooling pass
// ---------------------------------------------------------------------------
__device__ __forceinline__ void window_pool_finish(const WinArgs& a, char* smem_c) {
  const Plan& pl = a.pl;
  float* smem = reinterpret_cast<float*>(smem_c);
  const ChainSmem cs = chain_smem(pl.W, pl.H);
  stage_window_block(pl, a.ws, smem);   // overlaps the head selection below
  Header* hdr = reinterpret_cast<Header*>(a.ws);
  float* exact = reinterpret_cast<float*>(a.ws + pl.off_spec) + 2 * pl.H;   // [H] ent, [H] mass
  const float* rowE = reinterpret_cast<const float*>(a.ws + pl.off_stats);   // [H*W] (k_pool_reduce)
  float* sE = smem + cs.rowe;                        // [H*W] entropy, then [H*W] mass
  float* sM = sE + pl.H * pl.W;
  float* sHead = smem + cs.head;                     // [H] entropy, [H] mass means
  if (!hdr->need_exact) {
    // the head sets of the moments pass are certain: its entropies and masses stand
    const float* spec = reinterpret_cast<const float*>(a.ws + pl.off_spec);
    for (int h = threadIdx.x; h < 2 * pl.H; h += blockDim.x) exact[h] = __ldcg(spec + h);
    if (threadIdx.x == 0) hdr->cnt_pool = 0;
    __syncthreads();
    run_window_chains(a.pl, a.p, a.ws, smem, true);
    return;
  }
  const int HW2 = 2 * pl.H * pl.W;                  // rowM follows rowE
  for (int base = threadIdx.x; base < HW2; base += 8 * blockDim.x) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = base + u * (int)blockDim.x;
      v[u] = i < HW2 ? __ldcg(rowE + i) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = base + u * (int)blockDim.x;
      if (i < HW2) sE[i] = v[u];
    }
  }
  __syncthreads();
  {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int h = warp; h < pl.H; h += nw) {
      float e = 0.f, m = 0.f;
      for (int r = lane; r < pl.W; r += 32) { e += sE[h * pl.W + r]; m += sM[h * pl.W + r]; }
      e = warp_sum(e);
      m = warp_sum(m);
      if (lane == 0) {
        sHead[h] = e / (float)pl.W;
        sHead[pl.H + h] = m / (float)pl.W;
        exact[h] = sHead[h];
        exact[pl.H + h] = sHead[pl.H + h];
      }
    }
  }
  __syncthreads();
  __shared__ int redo;
  uint64_t qs = 0, hs = 0;
  int hm = 0, nh = 0;
  if (pl.H <= 32) {   // one warp, registers and shuffles
    if (threadIdx.x < 32) {
      const int h = threadIdx.x;
      const bool v = h < pl.H;
      const HeadSets r = select_heads_warp(a.p, pl.H, v ? sHead[h] : INFINITY, v ? sHead[pl.H + h] : -INFINITY, 0.f);
      qs = r.qs; hs = r.hs; hm = r.hm; nh = r.nhi;
    }
  } else {
    select_heads(a.p, pl.H, sHead, sHead + pl.H, &qs, &hs, &hm, &nh);
  }
  if (threadIdx.x == 0) {
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
  if (redo) {   // the fixup launch redoes the pooling and this step
    cp_async_wait<0>();
    return;
  }
  run_window_chains(a.pl, a.p, a.ws, smem, true);
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
  if (threadIdx.x == 0) gtile[(size_t)ch * pl.ncol_tiles * 8 + tile] = g;
  // row sums over this tile
  for (int r = threadIdx.x; r < pl.W; r += blockDim.x) {
    float s = 0.f;
    for (int c = 0; c < kColTile; ++c) {
      float v = rows[(size_t)r * pl.n_pad + j0 + c];
      if (tempered) v = v > 0.f ? powf(v, invT) : 0.f;
      s += v;
    }
    rspart[((size_t)ch * pl.rs_parts + tile) * pl.W + r] = s;
  }
}

__global__ void __launch_bounds__(256) k_rows_chain(const Plan pl, const ckv_params prm, char* ws) {
  extern __shared__ __align__(16) float fsmem[];
  stage_window_block(pl, ws, fsmem);
  run_window_chains(pl, prm, ws, fsmem, false);
}

cudaError_t launch_rows_prep(const Plan& pl, const ckv_params& prm, char* ws, cudaStream_t st) {
  k_rows_prep<<<dim3(pl.ncol_tiles, pl.hi_rows ? 2 : 1), 256, 0, st>>>(pl, prm, ws);
  const size_t sm = sizeof(float) * chain_smem(pl.W, pl.H).total;
  { const cudaError_t e = ensure_dynamic_smem((const void*)k_rows_chain, sm); if (e != cudaSuccess) return e; }
  k_rows_chain<<<1, 256, sm, st>>>(pl, prm, ws);
  return cudaGetLastError();
}


// ---------------------------------------------------------------------------
// pass 1 on the 5th-generation tensor cores (bf16 / fp16)
// ---------------------------------------------------------------------------
// One CTA per (column chunk, KV group).  The group's G*W window-query rows stay in
// shared memory (TMA, 128-byte swizzle, two 64-element K panels); K tiles of TN
// keys stream through a `stages`-deep TMA ring.  One thread issues the UMMAs of a
// tile (M = 128 rows per m-tile, N = TN, K = 128 in 8 steps) into one of two TMEM
// accumulator buffers and commits them to an mbarrier, so the MMAs of tile t+1
// run while all 8 warps drain tile t: each thread owns one accumulator row
// (TMEM lane) and folds its logits into that row's running moments without
// shuffles.  Logits are rounded as the reference does for 16-bit inputs:
// dtype(dtype(acc) * fp32(1/sqrt(D))).
CKV_DEV char* align1024(char* p) {
  return reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~(uintptr_t)1023);
}

// Round a pair of fp32 accumulators as the reference rounds a 16-bit logit.
// bf16: RN_bf16(RN_f32(r * rs)) for a bf16 product r and rs = RN_f32(1 / sqrt(128))
// equals RN_bf16(r * kRsHi + RN_bf16(r * kRsLo)), rs split into two bf16 parts: the
// result depends only on r's 7-bit mantissa (the exponent scales every term alike) and
// all 128 mantissas agree (checked exhaustively in exact rational arithmetic), so the
// second rounding runs on packed bf16 pairs.  Head dim 128 only (the plan enforces it).
constexpr uint32_t kRsHi2 = 0x3db53db5u;   // bf16(rs) in both halves
constexpr uint32_t kRsLo2 = 0x371e371eu;   // bf16(rs - bf16(rs)) in both halves
template <int DT> CKV_DEV void round_pair(float a, float b, float rs, float& x, float& y);
template <> CKV_DEV void round_pair<CKV_BF16>(float a, float b, float rs, float& x, float& y) {
  uint32_t p, t;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(p) : "f"(b), "f"(a));
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(t) : "r"(p), "r"(kRsLo2));
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(p) : "r"(p), "r"(kRsHi2), "r"(t));
  x = __uint_as_float(p << 16);
  y = __uint_as_float(p & 0xffff0000u);
}
// The same, returning the two rounded logits as a packed fp32 pair.
template <int DT> CKV_DEV F2 round_f2(float a, float b, float rs);
template <> CKV_DEV F2 round_f2<CKV_BF16>(float a, float b, float rs) {
  uint32_t p, t;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(p) : "f"(b), "f"(a));
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(t) : "r"(p), "r"(kRsLo2));
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(p) : "r"(p), "r"(kRsHi2), "r"(t));
  F2 r;
  asm("{\n\t.reg .b32 lo, hi;\n\tshl.b32 lo, %1, 16;\n\tand.b32 hi, %1, 0xffff0000;\n\tmov.b64 %0, {lo, hi};\n\t}"
      : "=l"(r.v) : "r"(p));
  return r;
}
// The same, also returning the two rounded logits packed as a 16-bit pair (exact), for
// packed max / min.
template <int DT> CKV_DEV uint32_t round_pack(float a, float b, float rs, float& x, float& y);
template <> CKV_DEV uint32_t round_pack<CKV_BF16>(float a, float b, float rs, float& x, float& y) {
  uint32_t p, t;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(p) : "f"(b), "f"(a));
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(t) : "r"(p), "r"(kRsLo2));
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(p) : "r"(p), "r"(kRsHi2), "r"(t));
  x = __uint_as_float(p << 16);
  y = __uint_as_float(p & 0xffff0000u);
  return p;
}
// A packed pair of rounded logits (low half first) as a packed fp32 pair (exact).
template <int DT> CKV_DEV F2 unpack_f2(uint32_t p) {
  if constexpr (DT == CKV_BF16) {
    F2 r;
    asm("{\n\t.reg .b32 lo, hi;\n\tshl.b32 lo, %1, 16;\n\tand.b32 hi, %1, 0xffff0000;\n\tmov.b64 %0, {lo, hi};\n\t}"
        : "=l"(r.v) : "r"(p));
    return r;
  } else {
    return f2(__half2float(__ushort_as_half((unsigned short)(p & 0xffffu))),
              __half2float(__ushort_as_half((unsigned short)(p >> 16))));
  }
}
template <int DT> CKV_DEV uint32_t pmax2(uint32_t a, uint32_t b) {
  uint32_t r;
  if constexpr (DT == CKV_BF16) asm("max.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  else asm("max.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
template <int DT> CKV_DEV uint32_t pmin2(uint32_t a, uint32_t b) {
  uint32_t r;
  if constexpr (DT == CKV_BF16) asm("min.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  else asm("min.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
// The larger / smaller of the two halves of a packed pair, as fp32.
template <int DT> CKV_DEV float phalf_max(uint32_t p) {
  if constexpr (DT == CKV_BF16) return fmaxf(__uint_as_float(p << 16), __uint_as_float(p & 0xffff0000u));
  else return fmaxf(__half2float(__ushort_as_half((unsigned short)(p & 0xffffu))),
                    __half2float(__ushort_as_half((unsigned short)(p >> 16))));
}
template <int DT> CKV_DEV float phalf_min(uint32_t p) {
  if constexpr (DT == CKV_BF16) return fminf(__uint_as_float(p << 16), __uint_as_float(p & 0xffff0000u));
  else return fminf(__half2float(__ushort_as_half((unsigned short)(p & 0xffffu))),
                    __half2float(__ushort_as_half((unsigned short)(p >> 16))));
}
// fp16 keeps 3 more mantissa bits than bf16, so dividing (the reference on CPU) and
// multiplying by the reciprocal (its CUDA scalar division) round apart often enough to
// matter: fp16 divides.  (bf16: no difference in 1M sampled logits.)
template <> CKV_DEV void round_pair<CKV_FP16>(float a, float b, float rs, float& x, float& y) {
  const float sd = 11.313708305358887f;   // fp32(sqrt(128)); rs = RN(1 / sd)
  x = __half2float(__float2half_rn(div_rcp(__half2float(__float2half_rn(a)), sd, rs)));
  y = __half2float(__float2half_rn(div_rcp(__half2float(__float2half_rn(b)), sd, rs)));
}
template <> CKV_DEV uint32_t round_pack<CKV_FP16>(float a, float b, float rs, float& x, float& y) {
  round_pair<CKV_FP16>(a, b, rs, x, y);
  const __half2 h = __floats2half2_rn(x, y);   // exact: x, y are fp16 values
  return *reinterpret_cast<const uint32_t*>(&h);
}
template <> CKV_DEV F2 round_f2<CKV_FP16>(float a, float b, float rs) {
  float x, y;
  round_pair<CKV_FP16>(a, b, rs, x, y);
  return f2(x, y);
}

// v^e for v > 0, else 0 (the tempered pooled rows), out of line: the temperature is
// rarely set, and sixteen inlined copies of powf in a tile's row loop would spread the
// hot epilogue code over many more instruction-cache lines.
__device__ __noinline__ float pow_pos(float v, float e) { return v > 0.f ? powf(v, e) : 0.f; }

constexpr int kStatsEpiWarps = 16;                       // epilogue warps of the moments pass
constexpr int kStatsWarmWarp = kStatsEpiWarps + 1;         // warm-up warp (after the producer warp)
constexpr int kStatsThreads = 32 * (kStatsEpiWarps + 2);  // + one producer warp + the warm-up warp

// EXACT: the exact branch of the W = 32 / 128 pooling pass instead (returns at once when the
// moments pass settled the head sets): the same tiles, with each row's log-sum-exp known,
// give the clamped entropy and the transient mass of PU:1452-1508 as one partial per
// 64-key tile (the layout the reduction kernel sums), no moments.
template <int DT, bool EXACT>
__global__ void __launch_bounds__(kStatsThreads, 1)
    k_tc_stats(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk, WinArgs a) {
  extern __shared__ char smem_raw[];
  const Plan& pl = a.pl;
  Header* hdr = reinterpret_cast<Header*>(a.ws);
  if constexpr (EXACT) {
    if (*reinterpret_cast<volatile int32_t*>(&hdr->need_exact) == 0) return;
  }
  int32_t* status = &hdr->status;
  const int m_tiles = (pl.G * pl.W) / 128;            // 128-row m-tiles of a KV group
  const int chunk = blockIdx.x, g = blockIdx.y / m_tiles, mtc = blockIdx.y % m_tiles;
  const int hpm = 128 / pl.W;                          // heads per m-tile
  const int hfirst = g * pl.G + mtc * hpm;             // first head of this CTA's m-tile
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int TN = a.tc_tn, S = a.tc_stages;
  const int ntn = (pl.n + TN - 1) / TN;
  const int t0 = chunk * a.tc_tpc, t1 = min(t0 + a.tc_tpc, ntn);
  const int ntile = max(0, t1 - t0);
  char* sA = align1024(smem_raw);                      // the m-tile's 128 window-query rows
  char* sB = sA + 2 * 128 * 128;                       // K stages
  // K stage full / free, accumulator buffer full / free (16 epilogue warps arrive)
  __shared__ __align__(8) uint64_t bar_q, bar_k[4], bar_kfree[4], bar_full[2], bar_tfree[2];
  __shared__ uint32_t tmem_base_sh;
  const uint32_t ncols = (2 * TN <= 256) ? 256u : 512u;   // two accumulator buffers of N = TN
  if (warp == 0) tc::tmem_alloc(&tmem_base_sh, ncols);
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar_q, 1);
    for (int i = 0; i < 4; ++i) { tc::mbar_init(&bar_k[i], 1); tc::mbar_init(&bar_kfree[i], 1); }
    for (int i = 0; i < 2; ++i) { tc::mbar_init(&bar_full[i], 1); tc::mbar_init(&bar_tfree[i], kStatsEpiWarps); }
    tc::fence_barrier_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_base_sh;

  // 16 epilogue warps: TMEM lane group lg (32 rows of the m-tile), column split sp of 4
  const int lg = warp & 3;
  constexpr int nsplit = kStatsEpiWarps / 4;
  const int sp = warp >> 2;
  const int cw = TN / nsplit;                          // columns per thread per tile (>= 32)
  const int row = 32 * lg + lane;
  const int r = row % pl.W;
  const int lim = pl.n - pl.W + r;                     // last visible key of this window row
  Moments M{-INFINITY, 0.f, 0.f, 0.f};
  float xmin = INFINITY;                               // smallest visible rounded logit of the row

  if (warp == kStatsEpiWarps) {
    // ---------------- producer: TMA ring of K tiles and the UMMAs (one thread) ----------------
    if (lane == 0 && ntile > 0) {
      const uint32_t idesc = tc::idesc_f16(DT == CKV_BF16, 128, TN);
      auto load_tile = [&](int i) {   // K tile i of this chunk into stage i % S
        const int st = i % S;
        tc::mbar_expect_tx(&bar_k[st], (uint32_t)TN * 256u);
        for (int p = 0; p < 2; ++p)
          tc::tma_load_3d(sB + (st * 2 + p) * TN * 128, &tmk, &bar_k[st], p * 64, (t0 + i) * TN, g);
      };
      tc::mbar_expect_tx(&bar_q, 128u * 256u);
      for (int hl = 0; hl < hpm; ++hl)
        for (int p = 0; p < 2; ++p)
          tc::tma_load_3d(sA + p * 128 * 128 + hl * pl.W * 128, &tmq, &bar_q, p * 64, pl.n - pl.W, hfirst + hl);
      int issued = min(S, ntile), consumed = 0, mmas = 0;
      for (int i = 0; i < issued; ++i) load_tile(i);
      bool ok = tc::mbar_wait_backoff(&bar_q, 0, status);
      for (int i = 0; ok && i < ntile; ++i) {
        const int st = i % S, b = i & 1;
        if (i >= 2 && !tc::mbar_wait_backoff(&bar_tfree[b], ((i - 2) >> 1) & 1, status)) { ok = false; break; }
        if (!tc::mbar_wait_backoff(&bar_k[st], (i / S) & 1, status)) { ok = false; break; }
        consumed = i + 1;
        tc::fence_after_sync();
        const uint32_t dcol = (uint32_t)(b * TN);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {   // M = 128 query rows, N = TN keys, K = 128 in 8 steps
          const int p = ks >> 2, koff = (ks & 3) * 32;
          const uint64_t ad = tc::sw128_kmajor_desc(tc::smem_addr(sA + p * 128 * 128 + koff));
          const uint64_t bd = tc::sw128_kmajor_desc(tc::smem_addr(sB + (st * 2 + p) * TN * 128 + koff));
          tc::umma_f16(tmem + dcol, ad, bd, idesc, ks > 0 ? 1u : 0u);
        }
        tc::umma_commit(&bar_full[b]);
        tc::umma_commit(&bar_kfree[st]);
        mmas = i + 1;
        if (i + S < ntile) {
          if (!tc::mbar_wait_backoff(&bar_kfree[st], (i / S) & 1, status)) { ok = false; break; }
          load_tile(i + S);
          issued = i + S + 1;
        }
      }
      if (!ok) {
        // gave up: let the copies and MMAs already issued land before the CTA frees its
        // shared memory and TMEM (each wait bounded again)
        for (int i = consumed; i < issued; ++i) tc::mbar_wait(&bar_k[i % S], (i / S) & 1, status);
        if (mmas > 0) tc::mbar_wait(&bar_kfree[(mmas - 1) % S], ((mmas - 1) / S) & 1, status);
      }
    }
    __syncwarp();
  } else if (warp == kStatsWarmWarp) {
    // ---------------- warm-up warp: the last CTA's tail code, dry ----------------
    // Runs merge_group_rows, group_head_means and the head selection with every store
    // switched off while the epilogue works, so that if this CTA is the last of its group
    // (or of all groups) those instructions are already in this SM's cache.  `dry` comes
    // from an opaque move so the calls keep their one shared copy of the code.
    if constexpr (!EXACT) {
      int dryv;
      asm volatile("mov.b32 %0, 1;" : "=r"(dryv));
      const bool dry = dryv != 0;
      const int nrows = pl.G * pl.W, i0 = g * pl.G * pl.W;
      float* rw = reinterpret_cast<float*>(smem_raw);   // read only (stores are off)
      merge_group_rows(reinterpret_cast<const float4*>(a.ws + pl.off_stats),
                       reinterpret_cast<const float*>(a.ws + pl.off_minx), reinterpret_cast<float*>(a.ws + pl.off_lse),
                       rw, rw + nrows, rw + 2 * nrows, pl.H, pl.W, pl.n, pl.nstat_chunks, 1, i0, nrows, lane,
                       (int)blockDim.x, dry);
      group_head_means(rw, rw + nrows, rw + 2 * nrows, reinterpret_cast<float*>(a.ws + pl.off_spec), pl.H, pl.W, 1,
                       g * pl.G, pl.G, 0, 1, dry);
      if (dry) {
        const HeadSets hs = select_heads_warp(a.p, pl.H, (float)lane, 0.5f, 0.f);
        asm volatile("" ::"l"(hs.qs), "l"(hs.hs), "r"(hs.certain));
      }
    }
  } else if constexpr (EXACT) {
    // ---------------- epilogue: clamped entropy and transient mass of this thread's row ----
    // warp (lg, sp) holds keys [64 sp, 64 sp + 64) of each 256-key tile: one 64-key tile
    const float rs = 1.0f / sqrtf((float)pl.D);
    const int h = hfirst + row / pl.W;
    const float L = __ldcg(reinterpret_cast<const float*>(a.ws + pl.off_lse) + h * pl.W + r);   // log2 units
    float* epart = reinterpret_cast<float*>(a.ws + pl.off_epart);
    float* mpart = reinterpret_cast<float*>(a.ws + pl.off_mpart);
    const uint32_t lane_base = tmem + ((uint32_t)(32 * lg) << 16);
    for (int i = 0; i < ntile; ++i) {
      const int b = i & 1;
      if (!__all_sync(0xffffffffu, tc::mbar_wait(&bar_full[b], (i >> 1) & 1, status))) break;
      tc::fence_after_sync();
      float ent = 0.f, mass = 0.f;
      for (int c = sp * cw; c < (sp + 1) * cw; c += 32) {
        float v[32];
        __syncwarp();
        tc::tmem_ld32(lane_base + (uint32_t)(b * TN + c), v);
        if (c + 32 >= (sp + 1) * cw) {   // this warp's last load of the tile: release the buffer
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&bar_tfree[b]);
        }
        const int jb = (t0 + i) * TN + c;
#pragma unroll
        for (int k = 0; k < 32; k += 2) {
          float x[2];
          round_pair<DT>(v[k], v[k + 1], rs, x[0], x[1]);
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int j = jb + k + e;
            if (j <= lim) {
              const float d = fmaf(x[e], kLog2e, -L);
              const float p = ex2(d);
              ent += (p >= 1e-8f) ? -p * d * kLn2 : kGeps;   // -c ln c, c = max(p, 1e-8)
              if (j >= pl.s) mass += p;
            } else if (j < pl.n) {
              ent += kGeps;   // masked entry: probability 0, clamped to 1e-8
            }
          }
        }
      }
      const int t64 = (t0 + i) * (TN / 64) + sp;   // cw == 64
      if (t64 < pl.ncol_tiles) {
        epart[((size_t)t64 * pl.H + h) * pl.W + r] = ent;
        mpart[((size_t)t64 * pl.H + h) * pl.W + r] = mass;
      }
    }
  } else {
    // ---------------- epilogue: running moments of this thread's row ----------------
    const float rs = 1.0f / sqrtf((float)pl.D);
    const uint32_t lane_base = tmem + ((uint32_t)(32 * lg) << 16);
    // Tiles whose every column each row of the m-tile sees (no causal mask, no keys past
    // n): all but the sequence's last one or two.  Their chunks run software-pipelined:
    // chunk k + 1 is loaded from TMEM, rounded and max-reduced in the same straight-line
    // block as chunk k's exponentials and sums, so one chunk's MUFU work overlaps the
    // next chunk's ALU work within a warp.  Every sum, rescale and their order are those
    // of the per-chunk loop further down, which takes the remaining (masked) tiles.
    const int nclean = cw == 64 ? max(0, min(ntile, (pl.n - pl.W + 1) / TN - t0)) : 0;
    bool alive = true;
    // a chunk's 32 rounded logits as 16 packed pairs, with their packed max / min
    auto load_round = [&](uint32_t taddr, uint32_t(&pk)[16], uint32_t& px, uint32_t& pn) {
      float v[32];
      __syncwarp();
      tc::tmem_ld32(taddr, v);
      float xd, yd;
#pragma unroll
      for (int u = 0; u < 16; ++u) pk[u] = round_pack<DT>(v[2 * u], v[2 * u + 1], rs, xd, yd);
      uint32_t mx[8], mn[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) { mx[i] = pmax2<DT>(pk[i], pk[i + 8]); mn[i] = pmin2<DT>(pk[i], pk[i + 8]); }
#pragma unroll
      for (int i = 0; i < 4; ++i) { mx[i] = pmax2<DT>(mx[i], mx[i + 4]); mn[i] = pmin2<DT>(mn[i], mn[i + 4]); }
#pragma unroll
      for (int i = 0; i < 2; ++i) { mx[i] = pmax2<DT>(mx[i], mx[i + 2]); mn[i] = pmin2<DT>(mn[i], mn[i + 2]); }
      px = pmax2<DT>(mx[0], mx[1]);
      pn = pmin2<DT>(mn[0], mn[1]);
    };
    // fold a chunk's max into the running moments (rescaling them when it rises)
    auto fold_max = [&](uint32_t px, uint32_t pn) {
      xmin = fminf(xmin, phalf_min<DT>(pn));
      const float cm2 = phalf_max<DT>(px) * kLog2e;
      if (cm2 > M.m) {
        if (M.m != -INFINITY) {
          const float d = cm2 - M.m;
          const float sc = ex2(-d);
          M.t = sc * (M.t - d * M.z);
          M.z *= sc;
          M.s *= sc;
        }
        M.m = cm2;
      }
    };
    // a clean chunk's exponentials against the running max: sums, entropy moment, sinks
    auto chunk_exps = [&](const uint32_t(&pk)[16], int jb) {
      const float nm = -M.m;
      const F2 l2e = f2(kLog2e, kLog2e), nm2 = f2(nm, nm);
      F2 z2[2] = {f2(0.f, 0.f), f2(0.f, 0.f)}, t2[2] = {f2(0.f, 0.f), f2(0.f, 0.f)};
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const F2 d2 = fma2(unpack_f2<DT>(pk[u]), l2e, nm2);
        const F2 e2 = f2(ex2(f2lo(d2)), ex2(f2hi(d2)));
        const int q = u & 1;
        z2[q] = add2(z2[q], e2);
        t2[q] = fma2(e2, d2, t2[q]);
      }
      const F2 zs = add2(z2[0], z2[1]), ts = add2(t2[0], t2[1]);
      M.z += f2lo(zs) + f2hi(zs);
      M.t += f2lo(ts) + f2hi(ts);
      if (jb < pl.s) {
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const F2 x2 = unpack_f2<DT>(pk[u]);
          if (jb + 2 * u < pl.s) M.s += ex2(fmaf(f2lo(x2), kLog2e, nm));
          if (jb + 2 * u + 1 < pl.s) M.s += ex2(fmaf(f2hi(x2), kLog2e, nm));
        }
      }
    };
    if (nclean > 0) {
      alive = __all_sync(0xffffffffu, tc::mbar_wait(&bar_full[0], 0, status));
      if (alive) {
        tc::fence_after_sync();
        uint32_t pc[16], pnx[16], px, pn;   // the chunk whose exponentials are next; the one after it
        load_round(lane_base + (uint32_t)(sp * cw), pc, px, pn);   // chunk (0, 0)
        fold_max(px, pn);
        for (int i = 0; i < nclean; ++i) {
          const int b = i & 1;
          const int jb0 = (t0 + i) * TN + sp * cw;
          // chunk (i, 1) in, chunk (i, 0) out; then the warp's loads of tile i are done
          load_round(lane_base + (uint32_t)(b * TN + sp * cw + 32), pnx, px, pn);
          chunk_exps(pc, jb0);
          fold_max(px, pn);
#pragma unroll
          for (int u = 0; u < 16; ++u) pc[u] = pnx[u];
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&bar_tfree[b]);
          // chunk (i + 1, 0) in, chunk (i, 1) out
          if (i + 1 < nclean) {
            if (!__all_sync(0xffffffffu, tc::mbar_wait(&bar_full[b ^ 1], ((i + 1) >> 1) & 1, status))) {
              alive = false;
              break;
            }
            tc::fence_after_sync();
            load_round(lane_base + (uint32_t)((b ^ 1) * TN + sp * cw), pnx, px, pn);
            chunk_exps(pc, jb0 + 32);
            fold_max(px, pn);
#pragma unroll
            for (int u = 0; u < 16; ++u) pc[u] = pnx[u];
          } else {
            chunk_exps(pc, jb0 + 32);
          }
        }
      }
    }
    // the remaining tiles, one chunk at a time (causal mask and keys past n)
    for (int i = nclean; alive && i < ntile; ++i) {
      const int b = i & 1;
      if (!__all_sync(0xffffffffu, tc::mbar_wait(&bar_full[b], (i >> 1) & 1, status))) break;
      tc::fence_after_sync();
      const int t = t0 + i;
      const uint32_t base = tmem + ((uint32_t)(32 * lg) << 16) + (uint32_t)(b * TN);
      for (int c = sp * cw; c < (sp + 1) * cw; c += 32) {
        float v[32];
        __syncwarp();
        tc::tmem_ld32(base + c, v);
        if (c + 32 >= (sp + 1) * cw) {   // this warp's last load of the tile: release the buffer
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&bar_tfree[b]);
        }
        const int jb = t * TN + c;
        // a chunk past the row's last visible key adds nothing (after the warp-wide load);
        // folding it in would seed the running max with the mask value when it comes first
        if (jb > lim) continue;
        float x[32];
        uint32_t pk[16];
#pragma unroll
        for (int k = 0; k < 32; k += 2) pk[k >> 1] = round_pack<DT>(v[k], v[k + 1], rs, x[k], x[k + 1]);
        // packed max / min of the chunk's rounded logits: trees of depth 4
        uint32_t px, pn;
        {
          uint32_t mx[8], mn[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) { mx[i] = pmax2<DT>(pk[i], pk[i + 8]); mn[i] = pmin2<DT>(pk[i], pk[i + 8]); }
#pragma unroll
          for (int i = 0; i < 4; ++i) { mx[i] = pmax2<DT>(mx[i], mx[i + 4]); mn[i] = pmin2<DT>(mn[i], mn[i + 4]); }
#pragma unroll
          for (int i = 0; i < 2; ++i) { mx[i] = pmax2<DT>(mx[i], mx[i + 2]); mn[i] = pmin2<DT>(mn[i], mn[i + 2]); }
          px = pmax2<DT>(mx[0], mx[1]);
          pn = pmin2<DT>(mn[0], mn[1]);
        }
        float cm, cmin;
        if (jb + 31 > lim) {   // the masked / out-of-range tail of the row (last tiles only)
          cmin = INFINITY;
          cm = -INFINITY;
#pragma unroll
          for (int k = 0; k < 32; ++k) {
            if (jb + k > lim) x[k] = -1e30f;
            else { cmin = fminf(cmin, x[k]); cm = fmaxf(cm, x[k]); }
          }
        } else {
          cm = phalf_max<DT>(px);
          cmin = phalf_min<DT>(pn);
        }
        xmin = fminf(xmin, cmin);
        const float cm2 = cm * kLog2e;
        if (cm2 > M.m) {
          if (M.m != -INFINITY) {
            const float d = cm2 - M.m;
            const float sc = ex2(-d);
            M.t = sc * (M.t - d * M.z);
            M.z *= sc;
            M.s *= sc;
          }
          M.m = cm2;
        }
        const float nm = -M.m;
        // even / odd columns in the two halves of packed pairs (the same sums as two
        // scalar accumulators)
        const F2 l2e = f2(kLog2e, kLog2e), nm2 = f2(nm, nm);
        F2 z2[2] = {f2(0.f, 0.f), f2(0.f, 0.f)}, t2[2] = {f2(0.f, 0.f), f2(0.f, 0.f)};   // 4 chains each
#pragma unroll
        for (int k = 0; k < 32; k += 2) {
          const F2 d2 = fma2(f2(x[k], x[k + 1]), l2e, nm2);
          const F2 e2 = f2(ex2(f2lo(d2)), ex2(f2hi(d2)));
          const int q = (k >> 1) & 1;
          z2[q] = add2(z2[q], e2);
          t2[q] = fma2(e2, d2, t2[q]);
        }
        const F2 zs = add2(z2[0], z2[1]), ts = add2(t2[0], t2[1]);
        M.z += f2lo(zs) + f2hi(zs);
        M.t += f2lo(ts) + f2hi(ts);
        if (jb < pl.s) {
#pragma unroll
          for (int k = 0; k < 32; ++k)
            if (jb + k < pl.s) M.s += ex2(fmaf(x[k], kLog2e, nm));
        }
      }
    }
  }

  if constexpr (EXACT) {
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (warp == 0) tc::tmem_dealloc(tmem, ncols);
    return;
  }
  // merge the column splits of each row, then write this chunk's partial moments
  float4* part = reinterpret_cast<float4*>(a.ws + pl.off_stats);
  tc::fence_before_sync();
  __syncthreads();
  float4* msh = reinterpret_cast<float4*>(sB);        // K stages are free now: [nsplit][128]
  float* mnsh = reinterpret_cast<float*>(msh + nsplit * 128);
  if (warp < kStatsEpiWarps) {
    msh[sp * 128 + row] = make_float4(M.m, M.z, M.t, M.s);
    mnsh[sp * 128 + row] = xmin;
  }
  __syncthreads();
  if (warp < kStatsEpiWarps && sp == 0) {
    for (int q = 1; q < nsplit; ++q) {
      const float4 o = msh[q * 128 + row];
      M = merge(M, Moments{o.x, o.y, o.z, o.w});
      xmin = fminf(xmin, mnsh[q * 128 + row]);
    }
    const int h = hfirst + row / pl.W;
    part[((size_t)chunk * pl.H + h) * pl.W + r] = make_float4(M.m, M.z, M.t, M.s);
    reinterpret_cast<float*>(a.ws + pl.off_minx)[((size_t)chunk * pl.H + h) * pl.W + r] = xmin;
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 0) tc::tmem_dealloc(tmem, ncols);
  stats_finish(a, smem_raw, g * pl.G, pl.G, g, (int)gridDim.x * m_tiles, pl.Hkv);
}

// ---- TMA descriptors (host) -------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// [heads, n, 128] view with element strides (head, token) -> a 3-D tiled map with a
// (64 x box_rows x 1) box, 128-byte swizzle, zero fill beyond n.
static bool make_tmap(CUtensorMap* m, const void* base, int dtype, int n, int heads, int64_t hs,
                      int64_t ts, int box_rows) {
  auto enc = get_encode();
  if (!enc) return false;
  const cuuint64_t dims[3] = {128, (cuuint64_t)n, (cuuint64_t)heads};
  const cuuint64_t strides[2] = {(cuuint64_t)ts * 2, (cuuint64_t)hs * 2};
  const cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(m, dtype == CKV_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                         3, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

size_t tc_stats_smem(const Plan& pl, int TN, int S) {
  (void)pl;
  return 1024 + (size_t)2 * 128 * 128 + (size_t)S * 2 * TN * 128;
}

template <int DT, bool EXACT = false>
static cudaError_t launch_tc_stats(const WinArgs& a0, cudaStream_t st) {
  WinArgs a = a0;
  const Plan& pl = a.pl;
  const int m_tiles = pl.G * pl.W / 128;
  a.tc_tn = 256;        // keys per tile: UMMA N = 256 over one 128-row m-tile
  a.tc_stages = 3;
  a.tc_min = 1;
  const int ntn = (pl.n + a.tc_tn - 1) / a.tc_tn;
  a.tc_tpc = (ntn + pl.nstat_chunks - 1) / pl.nstat_chunks;
  CUtensorMap tq, tk;
  if (!make_tmap(&tq, a.q, DT, pl.n, pl.H, a.qhs, a.qts, pl.W) ||
      !make_tmap(&tk, a.k, DT, pl.n, pl.Hkv, a.khs, a.kts, a.tc_tn))
    return cudaErrorInvalidResourceHandle;   // TMA descriptor encoding refused the layout
  const size_t smem = tc_stats_smem(pl, a.tc_tn, a.tc_stages);
  { const cudaError_t e = ensure_dynamic_smem((const void*)k_tc_stats<DT, EXACT>, smem); if (e != cudaSuccess) return e; }
  k_tc_stats<DT, EXACT><<<dim3(pl.nstat_chunks, pl.Hkv * m_tiles), kStatsThreads, smem, st>>>(tq, tk, a);
  return cudaGetLastError();
}


// ---------------------------------------------------------------------------
// pass 2 on the tensor cores (W = 64, 4 query heads per KV group)
// ---------------------------------------------------------------------------
// Persistent CTAs (one per SM) take 64-key column tiles from a counter in the
// workspace header (so CTAs that start late, e.g. behind another layer's kernels,
// simply take fewer tiles); each tile is processed for all KV groups in turn
// ((tile, group) steps).  A producer warp streams, per step,
// the group's 256 window-query rows and the K tile through a two-stage ring (TMA)
// and issues the UMMAs (two m-tiles of 128 rows, N = 64) into one of two TMEM
// buffers.  The query map walks (dim, head, token) with the head inside the token,
// so m-tile mt row 2t + e holds window row t of head 4g + 2mt + e: TMEM lanes 2t and
// 2t + 1 carry two heads of one window row, and each thread holds two heads (one per
// m-tile).  A lane pair pools the group's four heads with one shuffle per column
// pair, each lane keeping alternate columns.  16 epilogue warps (TMEM lane group x
// 16-column quarter) turn logits into exact probabilities, add each row's clamped
// entropy and transient mass into TMEM running sums (one per (column quarter,
// group, head pair)), and keep the QI max / HI sum of their columns across the
// groups in registers.  After the last group of a tile the pooled rows go through
// shared memory to coalesced writes of the rows, column sums, row-sum partials and
// g totals (the SIMT kernel's layout).  mbarriers order the producer and the
// epilogue (stage free, accumulator full, accumulator free); the epilogue warps
// synchronise among themselves only around the per-tile writes.
template <bool B> struct BoolTag { static constexpr bool value = B; };
template <int V> struct IntTag { static constexpr int value = V; };
// HI pooling of the tensor-core pooling pass, fixed per launch
constexpr int kHiMeanAll = 0;   // mean over every head (membership factors all 1)
constexpr int kHiMean = 1;      // mean over a head subset
constexpr int kHiMax = 2;       // max over a head subset
constexpr int kHiNone = 3;      // no HI rows of its own (the HI chain reuses the QI rows)

constexpr int kP2TN = 64;                 // keys per tile
constexpr int kP2Stages = 2;              // (queries, K tile) stages
constexpr int kP2EpiWarps = 16;           // epilogue warps
// Five warpgroups: four of epilogue warps and one whose first warp is the producer (the
// other three only give their registers back).  Launched at 96 registers a thread (the
// most 640 threads can have), the producer warpgroup keeps 64 and the epilogue warps get
// 104: 4 x 128 x 104 + 128 x 64 = 640 x 96 (at 96 the epilogue spilled; the producer
// spills below 64).
constexpr int kP2Threads = 32 * (kP2EpiWarps + 4);
constexpr uint32_t kPoolEpiRegs = 104, kPoolProdRegs = 64, kPoolLaunchRegs = 96;
static_assert(4 * 128 * kPoolEpiRegs + 128 * kPoolProdRegs <= kP2Threads * kPoolLaunchRegs,
              "register split above the launch budget");
constexpr int kP2Pitch = kP2TN + 1;       // staging row pitch (conflict-free column writes)

struct P2Smem {
  size_t stage_bytes, off_stage, off_sq, off_sh, off_colpart, off_redrow, off_gsum, off_lse, total;
};

static __host__ __device__ P2Smem p2_layout(const Plan& pl) {
  P2Smem L;
  const size_t R = (size_t)pl.G * pl.W;
  L.stage_bytes = R * 256 + (size_t)kP2TN * 256;
  L.off_stage = 0;
  size_t off = kP2Stages * L.stage_bytes;
  L.off_sq = off; off += (size_t)64 * kP2Pitch * 4;
  L.off_sh = off; off += (size_t)64 * kP2Pitch * 4;
  L.off_colpart = off; off += (size_t)8 * kP2TN * 4;
  L.off_redrow = off; off += (size_t)kP2EpiWarps * 8 * 4;
  L.off_gsum = off; off += 16;
  L.off_lse = off; off += (size_t)pl.H * pl.W * 4;
  L.total = 1024 + off;   // + alignment of the stage ring to 1024 bytes
  return L;
}

size_t tc_pool_smem(const Plan& pl) { return p2_layout(pl).total; }

template <int DT>
__device__ __forceinline__ void tc_pool_body(const CUtensorMap& tmq, const CUtensorMap& tmk, const WinArgs& a) {
  extern __shared__ char smem_raw[];
  const Plan& pl = a.pl;
  Header* hdr = reinterpret_cast<Header*>(a.ws);
  if (a.fixup_pass && *reinterpret_cast<volatile int32_t*>(&hdr->fixup) == 0) return;
  // the branch without the exact recomputation is the keys-on-lanes form (tc_pool_t_body)
  if (!a.fixup_pass && *reinterpret_cast<volatile int32_t*>(&hdr->need_exact) == 0) return;
  int32_t* status = &hdr->status;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int W = pl.W, G = pl.G, R = G * W;          // 64, 4, 256
  const int TN = kP2TN, S = kP2Stages;
  const int ntn = (pl.n + TN - 1) / TN;
  const int ngroups = pl.Hkv;
  const P2Smem Ly = p2_layout(pl);
  char* base = align1024(smem_raw);
  char* stg = base + Ly.off_stage;
  float* sQ = reinterpret_cast<float*>(base + Ly.off_sq);          // [64][kP2Pitch] QI pooled
  float* sH = reinterpret_cast<float*>(base + Ly.off_sh);          // [64][kP2Pitch] HI pooled
  float* colpart = reinterpret_cast<float*>(base + Ly.off_colpart);// [8][TN]
  float* redrow = reinterpret_cast<float*>(base + Ly.off_redrow);  // [16][8]
  float* gsum = reinterpret_cast<float*>(base + Ly.off_gsum);      // [2]
  float* slse = reinterpret_cast<float*>(base + Ly.off_lse);       // [H][W]
  __shared__ __align__(8) uint64_t bar_ld[kP2Stages], bar_sfree[kP2Stages], bar_full[2], bar_tfree[2], bar_tile;
  __shared__ int stage_tile[kP2Stages];   // producer only: tile loaded into each stage (-1: none)
  __shared__ int tile_slot[2];            // tile k of this CTA in slot k & 1 (-1: no tile left)
  __shared__ volatile int epi_abort;      // written by epilogue warps only, read after a barrier
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_sh;
  // TMEM columns [0, 256): two accumulator buffers of two m-tiles of N = 64; [256, 512):
  // running entropy / mass sums, 64 columns per column quarter (4 per group)
  const uint32_t ncols = 512;
  if (warp == 0) tc::tmem_alloc(&tmem_base_sh, ncols);
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) { tc::mbar_init(&bar_ld[i], 1); tc::mbar_init(&bar_sfree[i], 1); }
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&bar_full[i], 1);
      tc::mbar_init(&bar_tfree[i], kP2EpiWarps);
    }
    tc::mbar_init(&bar_tile, 1);
    epi_abort = 0;
    tc::fence_barrier_init();
    abort_sh = 0;
  }
  {
    const float* lse = reinterpret_cast<const float*>(a.ws + pl.off_lse);
    for (int i = threadIdx.x; i < pl.H * W; i += blockDim.x) slse[i] = __ldcg(lse + i);
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_base_sh;

  if (warp >= kP2EpiWarps) {
    tc::reg_dealloc<kPoolProdRegs>();
  } else {
    tc::reg_alloc<kPoolEpiRegs>();
  }
  if (warp >= kP2EpiWarps) {
    // ---------------- producer: tiles, TMA loads and UMMA issue (one thread) ----------------
    if (warp == kP2EpiWarps && lane == 0) {
      const uint32_t idesc = tc::idesc_f16(DT == CKV_BF16, 128, TN);
      uint32_t* ctr = &hdr->tile_ctr[a.fixup_pass ? 1 : 0];
      int load_tile = -1;
      int next_tile = (int)atomicAdd(ctr, 1u);   // fetched one tile ahead: the atomic's latency hides
      // loads step s (a new tile at the first group of each tile; -1 when none is left)
      auto load_step = [&](int s) {
        const int st = s % S, g = s % ngroups;
        if (g == 0) {
          load_tile = next_tile;
          if (load_tile < ntn) next_tile = (int)atomicAdd(ctr, 1u);
        }
        if (load_tile >= ntn) { stage_tile[st] = -1; return; }
        stage_tile[st] = load_tile;
        char* sb = stg + st * Ly.stage_bytes;
        tc::mbar_expect_tx(&bar_ld[st], (uint32_t)(R * 256 + TN * 256));
        for (int mt = 0; mt < 2; ++mt)
          for (int p = 0; p < 2; ++p)   // rows (token, head pair): head 4g + 2mt + e, token n - W + t
            tc::tma_load_3d(sb + p * R * 128 + mt * 128 * 128, &tmq, &bar_ld[st], p * 64, g * G + 2 * mt, pl.n - W);
        for (int p = 0; p < 2; ++p)
          tc::tma_load_3d(sb + R * 256 + p * TN * 128, &tmk, &bar_ld[st], p * 64, load_tile * TN, g);
      };
      for (int s = 0; s < S; ++s) load_step(s);
      for (int s = 0;; ++s) {
        const int st = s % S, b = s & 1;
        if (abort_sh) break;
        if (s >= 2 && !tc::mbar_wait(&bar_tfree[b], ((s - 2) >> 1) & 1, status)) { abort_sh = 1; break; }
        const int tile = stage_tile[st];
        if (s % ngroups == 0) {   // a new tile (or none): publish it to the epilogue
          tile_slot[(s / ngroups) & 1] = tile;
          tc::mbar_arrive(&bar_tile);
        }
        if (tile < 0) break;      // no tile left: the epilogue stops at this tile boundary
        if (!tc::mbar_wait(&bar_ld[st], (s / S) & 1, status)) { abort_sh = 1; break; }
        tc::fence_after_sync();
        const char* sb = stg + st * Ly.stage_bytes;
        const uint32_t dcol = (uint32_t)(b * 2 * TN);
        for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const int p = ks >> 2, koff = (ks & 3) * 32;
            const uint64_t ad = tc::sw128_kmajor_desc(tc::smem_addr(sb + p * R * 128 + mt * 128 * 128 + koff));
            const uint64_t bd = tc::sw128_kmajor_desc(tc::smem_addr(sb + R * 256 + p * TN * 128 + koff));
            tc::umma_f16(tmem + dcol + mt * TN, ad, bd, idesc, ks > 0 ? 1u : 0u);
          }
        }
        tc::umma_commit(&bar_full[b]);
        tc::umma_commit(&bar_sfree[st]);
        if (!tc::mbar_wait(&bar_sfree[st], (s / S) & 1, status)) { abort_sh = 1; break; }
        load_step(s + S);
      }
    }
    __syncwarp();
  } else {
    // ---------------- epilogue: 16 warps ----------------
    const int lg = warp & 3, cq = warp >> 2;
    const int L = 32 * lg + lane;                       // TMEM lane
    const int t = L >> 1;                               // window row
    const int e = lane & 1;                             // head within the m-tile pair
    const int lim = pl.n - W + t;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * lg) << 16);
    const uint32_t acc_base = lane_base + 256u + (uint32_t)(64 * cq);   // 4 columns per group, <= 16 groups
    const uint64_t qset = hdr->qi_heads, hset = hdr->hi_heads;
    const bool hmax = hdr->hi_mode == 1;
    const int nhi = hdr->n_hi;
    const float inv_nhi = 1.0f / (float)(nhi > 0 ? nhi : 1);   // mean = sum * (1 / count)
    const bool hi_rows = pl.hi_rows != 0;
    const uint64_t all_heads = pl.H >= 64 ? ~0ull : ((1ull << pl.H) - 1);
    const int hi_kind = !hi_rows ? kHiNone : (hmax ? kHiMax : (hset == all_heads ? kHiMeanAll : kHiMean));
    // this lane's heads 4g + e (bit g) and 4g + 2 + e (bit 16 + g) in the QI / HI sets
    uint32_t qbits = 0, hbits = 0;
    for (int g = 0; g < ngroups && g < 16; ++g) {
      const int ha = g * G + e, hb = ha + 2;
      qbits |= (uint32_t)((qset >> ha) & 1ull) << g | (uint32_t)((qset >> hb) & 1ull) << (16 + g);
      hbits |= (uint32_t)((hset >> ha) & 1ull) << g | (uint32_t)((hset >> hb) & 1ull) << (16 + g);
    }
    const float rs = 1.0f / sqrtf((float)pl.D);
    const bool tempered = a.p.neumann_temperature != 1.0f && a.p.neumann_temperature > 0.f;
    const float invT = tempered ? 1.0f / a.p.neumann_temperature : 1.0f;
    // epilogue barrier (the 16 epilogue warps).  Every warp takes the same barriers:
    // the loop ends only at a tile boundary, on a decision all warps read after a
    // barrier (no tile left, or a wait that gave up in any epilogue warp).
    auto epi_sync = [&]() { asm volatile("bar.sync 1, %0;" ::"r"(32 * kP2EpiWarps) : "memory"); };
    // exact clamped entropy / mass only when the moments pass could not settle the head sets
    const bool exact = *reinterpret_cast<volatile int32_t*>(&hdr->need_exact) != 0;
    if (exact) {
      const float z[4] = {0.f, 0.f, 0.f, 0.f};
      for (int g = 0; g < ngroups; ++g) tc::tmem_st4(acc_base + 4 * g, z);
    }
    // pooled values of this lane's two heads (4g + e, 4g + 2 + e) over the groups so far,
    // per column of the quarter; the lane pair combines its four heads once per tile
    float qown[16], hown[16];
    int tile = -1;
    for (int s = 0; s < ntn * ngroups; ++s) {
      const int g = s % ngroups;
      if (g == 0) {
        const int k = s / ngroups;
        if (!epi_abort) {
          const bool got = __all_sync(0xffffffffu, tc::mbar_wait(&bar_tile, k & 1, status));
          if (!got && lane == 0) epi_abort = 1;
        }
        epi_sync();
        if (epi_abort) { abort_sh = 1; break; }   // every epilogue warp reads the same flag here
        tile = tile_slot[k & 1];
        if (tile < 0) break;
      }
      const int j0 = tile * TN;
      if (g == 0) {
#pragma unroll
        for (int c = 0; c < 16; ++c) { qown[c] = 0.f; hown[c] = 0.f; }
      }
      bool ok = !epi_abort;
      if (ok && !tc::mbar_wait(&bar_full[s & 1], (s >> 1) & 1, status)) ok = false;
      ok = __all_sync(0xffffffffu, ok);
      if (!ok && lane == 0) epi_abort = 1;   // the rest of the tile is skipped; the loop ends at its boundary
      if (ok) {   // TMEM loads are warp-collective
        tc::fence_after_sync();
        // two halves of 8 columns: the second half's TMEM loads are in flight while the
        // first half is processed
        uint32_t ra[16], rb[16];
        const uint32_t col = (uint32_t)((s & 1) * 2 * TN + cq * 16);
        tc::tmem_ld8_nowait(lane_base + col, ra);
        tc::tmem_ld8_nowait(lane_base + col + TN, rb);
        tc::tmem_wait_ld();
        tc::tmem_ld8_nowait(lane_base + col + 8, ra + 8);
        tc::tmem_ld8_nowait(lane_base + col + TN + 8, rb + 8);
        float va[16], vb[16];
        const int ha = g * G + e, hb = ha + 2;
        const float La = slse[ha * W + t], Lb = slse[hb * W + t];
        const float fqa = ((qbits >> g) & 1u) ? 1.f : 0.f, fqb = ((qbits >> (16 + g)) & 1u) ? 1.f : 0.f;
        const float fha = ((hbits >> g) & 1u) ? 1.f : 0.f, fhb = ((hbits >> (16 + g)) & 1u) ? 1.f : 0.f;
        // the loaded half [h0, h0 + 8): into floats, rounded as the reference rounds a logit
        auto take_half = [&](int h0) {
#pragma unroll
          for (int k = h0; k < h0 + 8; ++k) {
            asm volatile("" : "+r"(ra[k]), "+r"(rb[k]));
            va[k] = __uint_as_float(ra[k]);
            vb[k] = __uint_as_float(rb[k]);
          }
#pragma unroll
          for (int k = h0; k < h0 + 8; k += 2) {
            float x0, x1, y0, y1;
            round_pair<DT>(va[k], va[k + 1], rs, x0, x1);
            round_pair<DT>(vb[k], vb[k + 1], rs, y0, y1);
            va[k] = x0; va[k + 1] = x1; vb[k] = y0; vb[k + 1] = y1;
          }
        };
        take_half(0);
        float ent0 = 0.f, ent1 = 0.f, mass0 = 0.f, mass1 = 0.f;
        const int jb = j0 + cq * 16;
        // warp-uniform (the TMEM wait inside `cols` is warp-collective): a warp with any
        // lane at the masked edge takes the general path
        const bool interior = __all_sync(0xffffffffu, jb + 15 <= lim && jb >= pl.s);
        // one logit pair (heads a, b at column c of the quarter): probabilities, the
        // exact entropy / mass terms when asked for, this lane's pooled values
        auto logit2 = [&](auto xtag, auto itag, auto htag, float xa, float xb, int j, int c) {
          constexpr bool EX = decltype(xtag)::value;
          constexpr int HM = decltype(htag)::value;
          const float da = fmaf(xa, kLog2e, -La), db = fmaf(xb, kLog2e, -Lb);
          float pa = ex2(da), pb = ex2(db);
          if constexpr (decltype(itag)::value) {
            if constexpr (EX) {
              ent0 = fmaf(fmaxf(pa, 1e-8f), fmaxf(da, kLog2Eps), ent0);
              ent1 = fmaf(fmaxf(pb, 1e-8f), fmaxf(db, kLog2Eps), ent1);
              mass0 += pa;
              mass1 += pb;
            }
          } else if (j <= lim) {
            if constexpr (EX) {
              ent0 = fmaf(fmaxf(pa, 1e-8f), fmaxf(da, kLog2Eps), ent0);
              ent1 = fmaf(fmaxf(pb, 1e-8f), fmaxf(db, kLog2Eps), ent1);
              if (j >= pl.s) { mass0 += pa; mass1 += pb; }
            }
          } else {
            pa = 0.f; pb = 0.f;
            if constexpr (EX) {
              if (j < pl.n) {   // masked: probability 0, clamped to 1e-8
                ent0 = fmaf(1e-8f, kLog2Eps, ent0);
                ent1 = fmaf(1e-8f, kLog2Eps, ent1);
              }
            }
          }
          qown[c] = fmaxf(qown[c], fmaxf(pa * fqa, pb * fqb));
          if constexpr (HM == kHiMean) hown[c] += fmaf(pa, fha, pb * fhb);
          else if constexpr (HM == kHiMax) hown[c] = fmaxf(hown[c], fmaxf(pa * fha, pb * fhb));
        };
        auto cols = [&](auto xtag, auto itag, auto htag) {
#pragma unroll
          for (int c = 0; c < 8; ++c) logit2(xtag, itag, htag, va[c], vb[c], jb + c, c);
          __syncwarp();
          tc::tmem_wait_ld();   // the second half; then the accumulator buffer is free
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&bar_tfree[s & 1]);
          take_half(8);
#pragma unroll
          for (int c = 8; c < 16; ++c) logit2(xtag, itag, htag, va[c], vb[c], jb + c, c);
        };
        auto run = [&](auto xtag, auto htag) {
          if (interior) cols(xtag, BoolTag<true>{}, htag);
          else cols(xtag, BoolTag<false>{}, htag);
        };
        auto run_x = [&](auto htag) {
          if (exact) run(BoolTag<true>{}, htag);
          else run(BoolTag<false>{}, htag);
        };
        switch (hi_kind) {   // a mean over every head is a mean with all factors 1
          case kHiMeanAll: case kHiMean: run_x(IntTag<kHiMean>{}); break;
          case kHiMax: run_x(IntTag<kHiMax>{}); break;
          default: run_x(IntTag<kHiNone>{}); break;
        }
        if (exact) {   // exact entropy (log2 units) / mass running sums of the two heads
          float acc[4];
          tc::tmem_ld4(acc_base + 4 * g, acc);
          acc[0] += ent0; acc[1] += ent1; acc[2] += mass0; acc[3] += mass1;
          tc::tmem_st4(acc_base + 4 * g, acc);
        }
      }
      if (g == ngroups - 1) {
        // ---- the tile is complete: the lane pair's four heads (lane e keeps the columns
        // 2m + e of the quarter), then pooled rows through shared memory
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          const float qk = e ? qown[2 * m + 1] : qown[2 * m];
          const float qr = __shfl_xor_sync(0xffffffffu, e ? qown[2 * m] : qown[2 * m + 1], 1);
          float hv = 0.f;
          if (hi_kind != kHiNone) {
            const float hk = e ? hown[2 * m + 1] : hown[2 * m];
            const float hr = __shfl_xor_sync(0xffffffffu, e ? hown[2 * m] : hown[2 * m + 1], 1);
            hv = hi_kind == kHiMax ? fmaxf(hk, hr) : hk + hr;
          }
          const int c = cq * 16 + 2 * m + e;
          sQ[t * kP2Pitch + c] = fmaxf(qk, qr);
          sH[t * kP2Pitch + c] = hv;
        }
        epi_sync();
        float* rows_qi = reinterpret_cast<float*>(a.ws + pl.off_rows_qi);
        float* rows_hi = reinterpret_cast<float*>(a.ws + pl.off_rows_hi);
        float* colsum = reinterpret_cast<float*>(a.ws + pl.off_colsum);
        float* gtile = reinterpret_cast<float*>(a.ws + pl.off_gtile);
        float* rspart = reinterpret_cast<float*>(a.ws + pl.off_rspart);
        const int tid = threadIdx.x;                    // 0..511
        const int pc = tid & 63, pr = tid >> 6;         // column, row group (rows pr + 8k)
        const int j = j0 + pc;
        const int nch = hi_rows ? 2 : 1;
        for (int c2 = 0; c2 < nch; ++c2) {
          float* rows = c2 == 0 ? rows_qi : rows_hi;
          const float* sx = c2 == 0 ? sQ : sH;
          float cs = 0.f;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int rr = pr + 8 * k;
            float v = sx[rr * kP2Pitch + pc];
            if (c2 == 1 && !hmax) v = v * inv_nhi;
            if (j >= pl.n) v = 0.f;
            rows[(size_t)rr * pl.n_pad + j] = v;
            cs += v;
            float rv = tempered ? pow_pos(v, invT) : v;
            rv = warp_sum(rv);
            if (lane == 0) redrow[warp * 8 + k] = rv;   // this warp's 32 columns of row rr
          }
          colpart[pr * TN + pc] = cs;
          epi_sync();
          if (tid < 2 * W) {   // row sums of each 32-key half of the tile (one partial per 32 keys)
            const int rr = tid % W, e = tid / W, k = rr >> 3, w0 = 2 * (rr & 7);
            rspart[((size_t)c2 * pl.rs_parts + 2 * tile + e) * W + rr] = redrow[(w0 + e) * 8 + k];
          }
          if (tid < TN) {
            const int jj = j0 + tid;
            float c = 0.f;
#pragma unroll
            for (int q = 0; q < 8; ++q) c += colpart[q * TN + tid];
            colsum[(size_t)c2 * pl.n_pad + jj] = c;
            float gg = 0.f;
            if (jj < pl.n_p) {
              gg = fmaxf(c, 1e-6f);
              if (tempered) gg = powf(gg, invT);
            }
            gg = warp_sum(gg);
            if (lane == 0) gsum[warp] = gg;
          }
          epi_sync();
          if (tid == 0) gtile[(size_t)c2 * pl.ncol_tiles * 8 + tile] = gsum[0] + gsum[1];
        }
        epi_sync();
      }
    }
    if (exact) {
      // one exact entropy / mass partial per (CTA, head, row): the four column quarters
      // of a TMEM lane are summed through shared memory (the staging rows are free now)
      float* epart = reinterpret_cast<float*>(a.ws + pl.off_epart);   // [e_parts][H][W]
      float* mpart = reinterpret_cast<float*>(a.ws + pl.off_mpart);
      float4* red = reinterpret_cast<float4*>(sQ);                    // [4 quarters][128 lanes]
      for (int g = 0; g < ngroups; ++g) {
        float acc[4];
        tc::tmem_ld4(acc_base + 4 * g, acc);
        red[cq * 128 + L] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        epi_sync();
        if (cq == 0) {
          float4 sum4 = red[L];
#pragma unroll
          for (int q2 = 1; q2 < 4; ++q2) {
            const float4 o = red[q2 * 128 + L];
            sum4.x += o.x; sum4.y += o.y; sum4.z += o.z; sum4.w += o.w;
          }
          const int ha = g * G + e, hb = ha + 2;
          const size_t slot = (size_t)blockIdx.x * pl.H;
          epart[(slot + ha) * W + t] = -sum4.x * kLn2;
          epart[(slot + hb) * W + t] = -sum4.y * kLn2;
          mpart[(slot + ha) * W + t] = sum4.z;
          mpart[(slot + hb) * W + t] = sum4.w;
        }
        epi_sync();
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 0) tc::tmem_dealloc(tmem, ncols);
}

// [heads, n, 128] view -> a 3-D tiled map over (dim, head, token) with a (64 x 2 x rows)
// box: consecutive smem rows alternate between two heads of one token.
static bool make_tmap_pairs(CUtensorMap* m, const void* base, int dtype, int n, int heads, int64_t hs,
                            int64_t ts, int rows, int hbox = 2) {
  auto enc = get_encode();
  if (!enc) return false;
  const cuuint64_t dims[3] = {128, (cuuint64_t)heads, (cuuint64_t)n};
  const cuuint64_t strides[2] = {(cuuint64_t)hs * 2, (cuuint64_t)ts * 2};
  const cuuint32_t box[3] = {64, (cuuint32_t)hbox, (cuuint32_t)rows};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(m, dtype == CKV_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                         3, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// The re-run with the exact head sets (returns at once unless the reduction flagged it).
template <int DT>
__global__ void __launch_bounds__(kP2Threads, 1)
    k_tc_pool(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
              const __grid_constant__ WinArgs a) {
  tc_pool_body<DT>(tmq, tmk, a);
}

template <int DT>
static cudaError_t launch_tc_pool(const WinArgs& a0, cudaStream_t st) {
  WinArgs a = a0;
  const Plan& pl = a.pl;
  CUtensorMap tq, tk;
  if (!make_tmap_pairs(&tq, a.q, DT, pl.n, pl.H, a.qhs, a.qts, pl.W) ||
      !make_tmap(&tk, a.k, DT, pl.n, pl.Hkv, a.khs, a.kts, kP2TN))
    return cudaErrorInvalidResourceHandle;   // TMA descriptor encoding refused the layout
  const size_t smem = tc_pool_smem(pl);
  { const cudaError_t e = ensure_dynamic_smem((const void*)k_tc_pool<DT>, smem); if (e != cudaSuccess) return e; }
  k_tc_pool<DT><<<pl.tc_nclusters, kP2Threads, smem, st>>>(tq, tk, a);
  return cudaGetLastError();
}


// ---------------------------------------------------------------------------
// pooling pass with keys on the TMEM lanes (the branch without the exact recomputation)
// ---------------------------------------------------------------------------
// When the moments pass settled the head sets, the pooling pass only turns logits into
// probabilities and pools them.  This form puts a tile of 128 keys on the UMMA's M side
// (A operand) and the KV group's 256 window-query rows on its N side (B operand; a
// (dim, head, token) tensor map with a 4-head box orders them (window row, head)), so
// 8 UMMAs of N = 256 cover a 128 x 256 block: half the operand traffic per logit of the
// head-pair form and half as many pipeline steps.  A thread owns one key (its TMEM lane)
// and a quarter of the columns (16 window rows x the group's 4 heads): pooling over the
// heads is in-thread, and its rows' pooled values accumulate over the KV groups in
// registers until the tile's rows, column sums, row-sum partials and g totals are written
// (the head-pair form's layout, per 64-key half).
//
// Other windows (template WIN): a step covers RS = min(W, 64) window rows of one KV group
// (N = 4 RS).  W = 32: N = 128, a thread's quarter is 8 rows.  W = 128: the window is
// walked in two halves of 64 rows; the steps of a tile run half by half (all KV groups
// of rows 0..63, then of rows 64..127), each half accumulating and writing its own rows,
// so a thread holds 16 rows' accumulators as for W = 64 (the K tile is loaded once per
// half; the second load comes from L2).
constexpr int kPTTN = 128;                 // keys per tile
constexpr int kPTStages = 2;               // (queries, K tile) stages
constexpr int kPTEpiWarps = 16;
constexpr int kPTThreads = 32 * (kPTEpiWarps + 4);   // as the head-pair form: five warpgroups

struct PTSmem {
  size_t stage_bytes, off_lse, total;
  size_t off_q2w = 0;   // per-head pass: q2w re-laid like the log-sum-exp
};

static __host__ __device__ PTSmem pt_layout(const Plan& pl) {
  PTSmem L;
  const size_t R = (size_t)pl.G * (pl.W < 64 ? pl.W : 64);   // query rows per step
  L.stage_bytes = R * 256 + (size_t)kPTTN * 256;
  size_t off = kPTStages * L.stage_bytes;
  L.off_lse = off; off += (size_t)pl.H * pl.W * 4;       // [group][row][head of the group]
  L.total = 1024 + off;
  return L;
}

template <int DT, int WIN>
__device__ __forceinline__ void tc_pool_t_body(const CUtensorMap& tmq, const CUtensorMap& tmk, const WinArgs& a) {
  static_assert(WIN == 32 || WIN == 64 || WIN == 128, "windows of 32, 64 or 128 rows");
  constexpr int RS = WIN < 64 ? WIN : 64;           // window rows per step
  constexpr int HALVES = WIN / RS;                  // 2 for W = 128
  constexpr int RPQ = RS / 4;                       // rows of a thread's column quarter
  constexpr int NCH = RPQ / 4;                      // 16-column TMEM loads per quarter
  constexpr int NCOL = 4 * RS;                      // UMMA N: RS rows x 4 heads
  extern __shared__ char smem_raw[];
  const Plan& pl = a.pl;
  Header* hdr = reinterpret_cast<Header*>(a.ws);
  int32_t* status = &hdr->status;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int W = WIN;
  const int G = pl.G, R = G * RS;                   // 4, 4 RS
  const int TN = kPTTN, S = kPTStages;
  const int ntn = (pl.n + TN - 1) / TN;
  const int ngroups = pl.Hkv;
  const int nvg = HALVES * ngroups;                 // steps per tile (half-major)
  const PTSmem Ly = pt_layout(pl);
  char* base = align1024(smem_raw);
  char* stg = base;
  const uint32_t snl_base = tc::smem_addr(base + Ly.off_lse);   // -lse table, [group][row][head]
  __shared__ __align__(8) uint64_t bar_ld[kPTStages], bar_sfree[kPTStages], bar_full[2], bar_tfree[2], bar_tile;
  __shared__ int stage_tile[kPTStages];   // producer only: tile loaded into each stage (-1: none)
  __shared__ int tile_slot[2];            // tile k of this CTA in slot k & 1 (-1: no tile left)
  __shared__ volatile int epi_abort;      // written by epilogue warps only, read after a barrier
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_sh;
  constexpr uint32_t ncols = 2 * NCOL;    // two accumulator buffers of N = NCOL
  if (warp == 0) tc::tmem_alloc(&tmem_base_sh, ncols);
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) { tc::mbar_init(&bar_ld[i], 1); tc::mbar_init(&bar_sfree[i], 1); }
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&bar_full[i], 1);
      tc::mbar_init(&bar_tfree[i], kPTEpiWarps);
    }
    tc::mbar_init(&bar_tile, 1);
    epi_abort = 0;
    tc::fence_barrier_init();
    abort_sh = 0;
  }
  __shared__ float4 smask[2 * kMaxHeads / 4];   // per KV group: QI, HI membership factors of its 4 heads
  __shared__ int s_hi_kind;                      // kHiMeanAll / kHiMean / kHiMax / kHiNone
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_base_sh;

  if (warp >= kPTEpiWarps) {
    tc::reg_dealloc<kPoolProdRegs>();
  } else {
    tc::reg_alloc<kPoolEpiRegs>();
  }
  if (warp >= kPTEpiWarps) {
    // ---------------- producer: tiles, TMA loads and UMMA issue (one thread) ----------------
    if (warp == kPTEpiWarps && lane == 0) {
      const uint32_t idesc = tc::idesc_f16(DT == CKV_BF16, 128, NCOL);
      uint32_t* ctr = &hdr->tile_ctr[a.fixup_pass ? 1 : 0];
      int load_tile = -1;
      int next_tile = (int)atomicAdd(ctr, 1u);   // fetched one tile ahead: the atomic's latency hides
      int ld_vg = 0;                             // (half, group) of the next step to load (in order)
      auto load_step = [&](int s) {
        const int st = s % S, vg = ld_vg;
        ld_vg = ld_vg + 1 == nvg ? 0 : ld_vg + 1;
        const int hf = HALVES > 1 ? vg / ngroups : 0, g = HALVES > 1 ? vg - hf * ngroups : vg;
        if (vg == 0) {
          load_tile = next_tile;
          if (load_tile < ntn) next_tile = (int)atomicAdd(ctr, 1u);
        }
        if (load_tile >= ntn) { stage_tile[st] = -1; return; }
        stage_tile[st] = load_tile;
        char* sb = stg + st * Ly.stage_bytes;
        tc::mbar_expect_tx(&bar_ld[st], (uint32_t)(R * 256 + TN * 256));
        for (int p = 0; p < 2; ++p)   // rows (window row, head) of group g: heads 4g .. 4g + 3, tokens n - W + RS hf ..
          tc::tma_load_3d(sb + p * R * 128, &tmq, &bar_ld[st], p * 64, g * G, pl.n - W + RS * hf);
        for (int p = 0; p < 2; ++p)   // the K tile: 128 keys of KV head g
          tc::tma_load_3d(sb + R * 256 + p * TN * 128, &tmk, &bar_ld[st], p * 64, load_tile * TN, g);
      };
      for (int s = 0; s < S; ++s) load_step(s);
      static_assert(kPTStages == 2, "one descriptor base per stage below");
      const uint64_t base0 = tc::sw128_kmajor_desc(tc::smem_addr(stg));
      const uint64_t base1 = tc::sw128_kmajor_desc(tc::smem_addr(stg + Ly.stage_bytes));
      for (int s = 0, g = 0, k = 0;; ++s) {   // g: step of the tile (half-major), k: this CTA's tile count
        const int st = s % S, b = s & 1;
        if (abort_sh) break;
        if (s >= 2 && !tc::mbar_wait_backoff(&bar_tfree[b], ((s - 2) >> 1) & 1, status)) { abort_sh = 1; break; }
        const int tile = stage_tile[st];
        if (g == 0) {   // a new tile (or none): publish it to the epilogue
          tile_slot[k & 1] = tile;
          tc::mbar_arrive(&bar_tile);
        }
        if (++g == nvg) { g = 0; ++k; }
        if (tile < 0) break;      // no tile left: the epilogue stops at this tile boundary
        if (!tc::mbar_wait_backoff(&bar_ld[st], (s / S) & 1, status)) { abort_sh = 1; break; }
        tc::fence_after_sync();
        const uint64_t sbase = st == 0 ? base0 : base1;   // descriptors: base + (offset >> 4)
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const int p = ks >> 2, koff = (ks & 3) * 32;
          const uint64_t ad = sbase + (uint64_t)((R * 256 + p * TN * 128 + koff) >> 4);   // keys (M)
          const uint64_t bd = sbase + (uint64_t)((p * R * 128 + koff) >> 4);              // query rows (N)
          tc::umma_f16(tmem + (uint32_t)(b * NCOL), ad, bd, idesc, ks > 0 ? 1u : 0u);
        }
        tc::umma_commit(&bar_full[b]);
        tc::umma_commit(&bar_sfree[st]);
        if (!tc::mbar_wait_backoff(&bar_sfree[st], (s / S) & 1, status)) { abort_sh = 1; break; }
        load_step(s + S);
      }
    }
    __syncwarp();
  } else {
    // ---------------- epilogue: 16 warps ----------------
    // while the producer's first loads and UMMAs run: the negated log-sum-exp re-laid as
    // [group][window row][head of the group] (one float4 per row) and the head membership
    // factors, then the epilogue warps meet at a named barrier (the producer does not wait)
    if (threadIdx.x == 0)
      s_hi_kind = pl.hi_rows == 0 ? kHiNone
                : (hdr->hi_mode == 1 ? kHiMax
                   : (hdr->hi_heads == (pl.H >= 64 ? ~0ull : (1ull << pl.H) - 1ull) ? kHiMeanAll : kHiMean));
    if (threadIdx.x < 2 * ngroups) {
      const int g = threadIdx.x >> 1;
      const uint32_t m = (uint32_t)(((threadIdx.x & 1) ? hdr->hi_heads : hdr->qi_heads) >> (g * G)) & 0xFu;
      smask[threadIdx.x] = make_float4((m & 1u) ? 1.f : 0.f, (m & 2u) ? 1.f : 0.f, (m & 4u) ? 1.f : 0.f, (m & 8u) ? 1.f : 0.f);
    }
    {
      const float* lse = reinterpret_cast<const float*>(a.ws + pl.off_lse);   // [H][W]
      float* sl = reinterpret_cast<float*>(base + Ly.off_lse);
      for (int i = threadIdx.x; i < pl.H * W; i += 32 * kPTEpiWarps) {
        const int h = i / W, r = i % W;
        sl[((h / G) * W + r) * G + (h % G)] = -__ldcg(lse + i);
      }
    }
    asm volatile("bar.sync 2, %0;" ::"r"(32 * kPTEpiWarps) : "memory");
    const int lg = warp & 3, q = warp >> 2;             // TMEM lane group (32 keys), column quarter
    const int key = 32 * lg + lane;                     // this thread's key within the tile
    const uint32_t lane_base = tmem + ((uint32_t)(32 * lg) << 16);
    // (values used once per tile are re-read there, not held in registers across the steps)
    const float rs = 1.0f / sqrtf((float)pl.D);
    float qacc[RPQ], hacc[RPQ];                         // rows RS hf + RPQ q + i of this thread's key
    int tile = -1;
    // s: step, vg: its (half, KV group), k: tiles this warp has started (no integer division
    // per step); g: the KV group, hf: the half
    int vg = 0, hf = 0;
    // the next step: the group, then the half, then the tile
    auto advance = [&](int& g) {
      if constexpr (HALVES == 1) {
        g = g + 1 == ngroups ? 0 : g + 1;
      } else {
        vg = vg + 1 == nvg ? 0 : vg + 1;
        if (++g == ngroups) { g = 0; hf = hf + 1 == HALVES ? 0 : hf + 1; }
      }
    };
    for (int s = 0, g = 0, k = 0; s < ntn * nvg; ++s, advance(g)) {
      if (HALVES == 1 ? g == 0 : vg == 0) {   // a new tile
        // no barrier among the epilogue warps: the producer's wait for all of them to free
        // a TMEM buffer keeps them within a step of one another, so the tile slot and the
        // tile barrier's phase of the current tile are still the ones each warp reads
        bool got = __shfl_sync(0xffffffffu, epi_abort == 0, 0);   // warp-uniform
        if (got) got = __all_sync(0xffffffffu, tc::mbar_wait(&bar_tile, k & 1, status));
        if (!got) {
          if (lane == 0) { epi_abort = 1; abort_sh = 1; }
          break;
        }
        tile = tile_slot[k & 1];
        ++k;
        if (tile < 0) break;
        if constexpr (HALVES == 1) {
#pragma unroll
          for (int i = 0; i < RPQ; ++i) { qacc[i] = 0.f; hacc[i] = 0.f; }
        }
      }
      if constexpr (HALVES > 1) {
        if (g == 0) {   // the first group of a half: fresh accumulators
#pragma unroll
          for (int i = 0; i < RPQ; ++i) { qacc[i] = 0.f; hacc[i] = 0.f; }
        }
      }
      const int j = tile * TN + key;
      bool ok = !epi_abort;
      if (ok && !tc::mbar_wait(&bar_full[s & 1], (s >> 1) & 1, status)) ok = false;
      ok = __all_sync(0xffffffffu, ok);
      if (!ok && lane == 0) epi_abort = 1;   // the rest of the tile is skipped; the loop ends at its boundary
      if (ok) {   // TMEM loads are warp-collective
        tc::fence_after_sync();
        // head membership factors (1 in the set, 0 outside) as pairs (heads 0 1, 2 3)
        const float4 q4 = smask[2 * g], h4 = smask[2 * g + 1];
        const F2 qm01 = f2(q4.x, q4.y), qm23 = f2(q4.z, q4.w);
        const F2 hm01 = f2(h4.x, h4.y), hm23 = f2(h4.z, h4.w);
        const F2 l2e = f2(kLog2e, kLog2e);
        const uint32_t col0 = (uint32_t)((s & 1) * NCOL + 4 * RPQ * q);
        // the causal mask only touches the tile that reaches the window (warp-uniform)
        const bool edge = tile * TN + TN - 1 > pl.n - W;
        // One copy of the step loop for every group: a group with no QI head has factors of 0
        // and its max stays at 0, as if skipped (a second, QI-free copy of the loop measured
        // slower: the hot code no longer fit the instruction cache as well).
        auto chunks = [&](auto htag, auto etag) {
          constexpr int HM = decltype(htag)::value;
          constexpr bool EDGE = decltype(etag)::value;
#pragma unroll
          for (int c = 0; c < NCH; ++c) {   // 16 columns: window rows RS hf + RPQ q + 4 c + i, heads 0..3
            uint32_t r16[16];
            __syncwarp();
            tc::tmem_ld16_nowait(lane_base + col0 + 16 * c, r16);
            tc::tmem_wait_ld();
            if (c == NCH - 1) {   // the last load of the step: the accumulator buffer is free
              tc::fence_before_sync();
              __syncwarp();
              if (lane == 0) tc::mbar_arrive(&bar_tfree[s & 1]);
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int r = RS * hf + RPQ * q + 4 * c + i;
              const float4 nL = tc::lds128(snl_base + (uint32_t)((g * W + r) * 16));   // -log2-sum-exp of (row, head 0..3)
              const F2 x01 = round_f2<DT>(__uint_as_float(r16[4 * i]), __uint_as_float(r16[4 * i + 1]), rs);
              const F2 x23 = round_f2<DT>(__uint_as_float(r16[4 * i + 2]), __uint_as_float(r16[4 * i + 3]), rs);
              F2 p01 = ex2_2(fma2(x01, l2e, f2(nL.x, nL.y)));
              F2 p23 = ex2_2(fma2(x23, l2e, f2(nL.z, nL.w)));
              if constexpr (EDGE) {
                if (j > pl.n - W + r) { p01 = f2(0.f, 0.f); p23 = p01; }   // causal mask (and keys past n)
              }
              const int u = 4 * c + i;
              {
                const F2 a = mul2(p01, qm01), b = mul2(p23, qm23);
                qacc[u] = max3f(max3f(qacc[u], f2lo(a), f2hi(a)), f2lo(b), f2hi(b));
              }
              if constexpr (HM == kHiMeanAll) {   // every head in the set: factors of 1 dropped
                const F2 t = add2(p01, p23);                 // (the same sums: p * 1 is exact)
                hacc[u] += f2lo(t) + f2hi(t);
              } else if constexpr (HM == kHiMean) {
                const F2 t = fma2(p23, hm23, mul2(p01, hm01));
                hacc[u] += f2lo(t) + f2hi(t);
              } else if constexpr (HM == kHiMax) {
                const F2 a = mul2(p01, hm01), b = mul2(p23, hm23);
                hacc[u] = max3f(max3f(hacc[u], f2lo(a), f2hi(a)), f2lo(b), f2hi(b));
              }
            }
          }
        };
        auto run = [&](auto htag) {
          if (edge) chunks(htag, BoolTag<true>{});
          else chunks(htag, BoolTag<false>{});
        };
        switch (s_hi_kind) {
          case kHiMeanAll: run(IntTag<kHiMeanAll>{}); break;
          case kHiMean: run(IntTag<kHiMean>{}); break;
          case kHiMax: run(IntTag<kHiMax>{}); break;
          default: run(IntTag<kHiNone>{}); break;
        }
      }
      if (g == ngroups - 1) {
        // ---- the tile (or its half) is complete: rows, then partial sums that the
        // reduction kernel completes (no barrier: each warp writes its own partials)
        float* rows_qi = reinterpret_cast<float*>(a.ws + pl.off_rows_qi);
        float* rows_hi = reinterpret_cast<float*>(a.ws + pl.off_rows_hi);
        float* rspart = reinterpret_cast<float*>(a.ws + pl.off_rspart);     // [2][rs_parts][W]
        float* colpart = reinterpret_cast<float*>(a.ws + pl.off_colpart);   // [2][pool_blocks][n_pad]
        const int t32 = tile * 4 + lg;                  // 32-key row-sum partial of this lane group
        const bool hi_rows = pl.hi_rows != 0, hmax = s_hi_kind == kHiMax;
        const int nch = hi_rows ? 2 : 1;
        const int nhi = hdr->n_hi;
        const float inv_nhi = 1.0f / (float)(nhi > 0 ? nhi : 1);   // mean = sum * (1 / count)
        const bool tempered = a.p.neumann_temperature != 1.0f && a.p.neumann_temperature > 0.f;
        const float invT = tempered ? 1.0f / a.p.neumann_temperature : 1.0f;
        // one accumulator set at a time (one copy of this code: a loop, not unrolled); the QI
        // registers take each set's row-sum terms (both sets start again at zero next tile)
#pragma unroll 1
        for (int c2 = 0; c2 < nch; ++c2) {
          float* rp = (c2 == 0 ? rows_qi : rows_hi) + (size_t)(RS * hf + RPQ * q) * pl.n_pad + j;
          float cs = 0.f;
#pragma unroll
          for (int i = 0; i < RPQ; ++i) {
            float v = c2 == 0 ? qacc[i] : hacc[i];
            if (c2 == 1 && !hmax) v = v * inv_nhi;
            if (j >= pl.n) v = 0.f;
            if (j < pl.n_pad) rp[(size_t)i * pl.n_pad] = v;
            cs += v;
            qacc[i] = tempered ? pow_pos(v, invT) : v;
          }
          // row sums over this lane group's 32 keys: with 16 rows, row 16 q + ((lane >> 1) & 15)
          // in lane pairs; with 8, row 8 q + ((lane >> 2) & 7) in lane quads
          if constexpr (RPQ == 16) {
            const float t = warp_sum16(qacc);
            if ((lane & 1) == 0 && t32 < pl.rs_parts)
              rspart[((size_t)c2 * pl.rs_parts + t32) * W + RS * hf + 16 * q + ((lane >> 1) & 15)] = t;
          } else {
            const float t = warp_sum8(qacc);
            if ((lane & 3) == 0 && t32 < pl.rs_parts)
              rspart[((size_t)c2 * pl.rs_parts + t32) * W + 8 * q + ((lane >> 2) & 7)] = t;
          }
          // column sum of this key over the row block's RPQ rows
          if (j < pl.n_pad) colpart[((size_t)c2 * (4 * HALVES) + 4 * hf + q) * pl.n_pad + j] = cs;
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 0) tc::tmem_dealloc(tmem, ncols);
}

// The pooling pass is one launch that takes its branch on the device: the head-pair form
// when the moments pass left the head sets unsettled (need_exact), the keys-on-lanes form
// otherwise.  A second kernel for the branch not taken would cost every layer a launch of
// 148 CTAs that return at once (about 3% of the batched step).  The keys-on-lanes form,
// the usual one, comes first: with the head-pair form's code laid out ahead of it, its loop
// missed the instruction cache about 2.5 times as often (64 instead of 55 us).
static_assert(kP2Threads == kPTThreads, "both pooling forms run in one launch");
template <int DT>
__global__ void __launch_bounds__(kPTThreads, 1)
    k_tc_pool_any(const __grid_constant__ CUtensorMap tmq2, const __grid_constant__ CUtensorMap tmk2,
                  const __grid_constant__ CUtensorMap tmq4, const __grid_constant__ CUtensorMap tmk4,
                  const __grid_constant__ WinArgs a) {
  const Header* hdr = reinterpret_cast<const Header*>(a.ws);
  if (*reinterpret_cast<const volatile int32_t*>(&hdr->need_exact) == 0) tc_pool_t_body<DT, 64>(tmq4, tmk4, a);
  else tc_pool_body<DT>(tmq2, tmk2, a);
}

template <int DT>
static cudaError_t launch_tc_pool_any(const WinArgs& a0, cudaStream_t st) {
  WinArgs a = a0;
  const Plan& pl = a.pl;
  CUtensorMap tq2, tk2, tq4, tk4;
  if (!make_tmap_pairs(&tq2, a.q, DT, pl.n, pl.H, a.qhs, a.qts, pl.W) ||
      !make_tmap(&tk2, a.k, DT, pl.n, pl.Hkv, a.khs, a.kts, kP2TN) ||
      !make_tmap_pairs(&tq4, a.q, DT, pl.n, pl.H, a.qhs, a.qts, pl.W, pl.G) ||
      !make_tmap(&tk4, a.k, DT, pl.n, pl.Hkv, a.khs, a.kts, kPTTN))
    return cudaErrorInvalidResourceHandle;   // TMA descriptor encoding refused the layout
  const size_t s2 = tc_pool_smem(pl), s4 = pt_layout(pl).total;
  const size_t smem = s2 > s4 ? s2 : s4;
  { const cudaError_t e = ensure_dynamic_smem((const void*)k_tc_pool_any<DT>, smem); if (e != cudaSuccess) return e; }
  // grid: one CTA per exact-branch partial (tc_nclusters >= the keys-on-lanes tile count
  // up to 148; surplus CTAs of that branch find no tile and return)
  k_tc_pool_any<DT><<<pl.tc_nclusters, kPTThreads, smem, st>>>(tq2, tk2, tq4, tk4, a);
  return cudaGetLastError();
}

// W = 32 / 128: the keys-on-lanes form as its own launch.  The first pass always pools:
// with the moments pass's head sets, which the exact branch (k_tc_stats<DT, true>, launched
// before it) may overturn; the re-run returns at once unless they were overturned.
template <int DT, int WIN>
__global__ void __launch_bounds__(kPTThreads, 1)
    k_tc_pool_lanes(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                    const __grid_constant__ WinArgs a) {
  const Header* hdr = reinterpret_cast<const Header*>(a.ws);
  if (a.fixup_pass && *reinterpret_cast<const volatile int32_t*>(&hdr->fixup) == 0) return;
  tc_pool_t_body<DT, WIN>(tmq, tmk, a);
}

template <int DT>
static cudaError_t launch_tc_pool_lanes(const WinArgs& a, cudaStream_t st) {
  const Plan& pl = a.pl;
  const int rs = pl.W < 64 ? pl.W : 64;
  CUtensorMap tq, tk;
  if (!make_tmap_pairs(&tq, a.q, DT, pl.n, pl.H, a.qhs, a.qts, rs, pl.G) ||
      !make_tmap(&tk, a.k, DT, pl.n, pl.Hkv, a.khs, a.kts, kPTTN))
    return cudaErrorInvalidResourceHandle;   // TMA descriptor encoding refused the layout
  const size_t smem = pt_layout(pl).total;
  const int ntn = (pl.n + kPTTN - 1) / kPTTN;
  const int grid = ntn < 148 ? ntn : 148;   // persistent CTAs take 128-key tiles from a counter
  if (pl.W == 32) {
    const cudaError_t e = ensure_dynamic_smem((const void*)k_tc_pool_lanes<DT, 32>, smem);
    if (e != cudaSuccess) return e;
    k_tc_pool_lanes<DT, 32><<<grid, kPTThreads, smem, st>>>(tq, tk, a);
  } else {
    const cudaError_t e = ensure_dynamic_smem((const void*)k_tc_pool_lanes<DT, 128>, smem);
    if (e != cudaSuccess) return e;
    k_tc_pool_lanes<DT, 128><<<grid, kPTThreads, smem, st>>>(tq, tk, a);
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// per-head pass on tcgen05 (PU:2208-2382): the keys-on-lanes form of the pooling pass
// ---------------------------------------------------------------------------
// Per step one KV group's 4 heads x RS window rows against a 128-key tile (UMMA M = 128
// keys on TMEM lanes, N = 4 RS).  A thread owns one key and a quarter of the step's rows;
// per head it keeps the two-hop sum (q2w-weighted) and the column sum over those rows and
// writes them, per row block, to partial slots that k_ph_combine adds up in a fixed order.
// The thread holding the last window row (last quarter of the last half) writes the query
// row and the query row's entropy partial per 32 keys.  The prelude launch (PRE) runs only
// the tiles holding the window columns and writes q2w from the same UMMA tiles, so both
// launches see bit-identical probabilities.
static __host__ __device__ PTSmem ph_layout(const Plan& pl) {
  PTSmem L = pt_layout(pl);
  L.off_q2w = L.total - 1024;
  L.total += (size_t)pl.H * pl.W * 4;
  return L;
}

template <int DT, int WIN, bool PRE>
__device__ __forceinline__ void tc_ph_body(const CUtensorMap& tmq, const CUtensorMap& tmk, const WinArgs& a) {
  static_assert(WIN == 32 || WIN == 64 || WIN == 128, "windows of 32, 64 or 128 rows");
  constexpr int RS = WIN < 64 ? WIN : 64;           // window rows per step
  constexpr int HALVES = WIN / RS;
  constexpr int RPQ = RS / 4;                       // rows of a thread's column quarter
  constexpr int NCH = RPQ / 4;                      // 16-column TMEM loads per quarter
  constexpr int NCOL = 4 * RS;                      // UMMA N: RS rows x 4 heads
  constexpr int W = WIN;
  extern __shared__ char smem_raw[];
  const Plan& pl = a.pl;
  Header* hdr = reinterpret_cast<Header*>(a.ws);
  int32_t* status = &hdr->status;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = pl.G, R = G * RS;
  const int TN = kPTTN, S = kPTStages;
  const int t_first = PRE ? (pl.n - W) / TN : 0;
  const int t_end = PRE ? (pl.n - 1) / TN + 1 : (pl.n + TN - 1) / TN;
  const int ntiles = t_end - t_first;
  const int ngroups = pl.Hkv;
  const int nvg = HALVES * ngroups;
  const PTSmem Ly = ph_layout(pl);
  char* base = align1024(smem_raw);
  char* stg = base;
  const float4* snlse4 = reinterpret_cast<const float4*>(base + Ly.off_lse);
  const float4* sq2w4 = reinterpret_cast<const float4*>(base + Ly.off_q2w);
  __shared__ __align__(8) uint64_t bar_ld[kPTStages], bar_sfree[kPTStages], bar_full[2], bar_tfree[2], bar_tile;
  __shared__ int stage_tile[kPTStages];
  __shared__ int tile_slot[2];
  __shared__ volatile int epi_abort;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_sh;
  constexpr uint32_t ncols = 2 * NCOL;
  if (warp == 0) tc::tmem_alloc(&tmem_base_sh, ncols);
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) { tc::mbar_init(&bar_ld[i], 1); tc::mbar_init(&bar_sfree[i], 1); }
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&bar_full[i], 1);
      tc::mbar_init(&bar_tfree[i], kPTEpiWarps);
    }
    tc::mbar_init(&bar_tile, 1);
    epi_abort = 0;
    tc::fence_barrier_init();
    abort_sh = 0;
  }
  {   // negated log-sum-exp and (main pass) q2w as [group][window row][head of the group]
    const float* lse = reinterpret_cast<const float*>(a.ws + pl.off_lse);   // [H][W]
    const float* q2w = reinterpret_cast<const float*>(a.ws + pl.off_ph_q2w);
    float* sl = reinterpret_cast<float*>(base + Ly.off_lse);
    float* sw = reinterpret_cast<float*>(base + Ly.off_q2w);
    for (int i = threadIdx.x; i < pl.H * W; i += blockDim.x) {
      const int h = i / W, r = i % W, o = ((h / G) * W + r) * G + (h % G);
      sl[o] = -__ldcg(lse + i);
      sw[o] = PRE ? 0.f : __ldcg(q2w + i);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_base_sh;

  if (warp >= kPTEpiWarps) {
    tc::reg_dealloc<kPoolProdRegs>();
  } else {
    tc::reg_alloc<kPoolEpiRegs>();
  }
  if (warp >= kPTEpiWarps) {
    // ---------------- producer: tiles, TMA loads and UMMA issue (one thread) ----------------
    if (warp == kPTEpiWarps && lane == 0) {
      const uint32_t idesc = tc::idesc_f16(DT == CKV_BF16, 128, NCOL);
      uint32_t* ctr = &hdr->tile_ctr[PRE ? 1 : 0];
      int load_tile = -1;
      int next_tile = t_first + (int)atomicAdd(ctr, 1u);
      int ld_vg = 0;
      auto load_step = [&](int s) {
        const int st = s % S, vg = ld_vg;
        ld_vg = ld_vg + 1 == nvg ? 0 : ld_vg + 1;
        const int hf = HALVES > 1 ? vg / ngroups : 0, g = HALVES > 1 ? vg - hf * ngroups : vg;
        if (vg == 0) {
          load_tile = next_tile;
          if (load_tile < t_end) next_tile = t_first + (int)atomicAdd(ctr, 1u);
        }
        if (load_tile >= t_end) { stage_tile[st] = -1; return; }
        stage_tile[st] = load_tile;
        char* sb = stg + st * Ly.stage_bytes;
        tc::mbar_expect_tx(&bar_ld[st], (uint32_t)(R * 256 + TN * 256));
        for (int p = 0; p < 2; ++p)
          tc::tma_load_3d(sb + p * R * 128, &tmq, &bar_ld[st], p * 64, g * G, pl.n - W + RS * hf);
        for (int p = 0; p < 2; ++p)
          tc::tma_load_3d(sb + R * 256 + p * TN * 128, &tmk, &bar_ld[st], p * 64, load_tile * TN, g);
      };
      for (int s = 0; s < S; ++s) load_step(s);
      static_assert(kPTStages == 2, "one descriptor base per stage below");
      const uint64_t base0 = tc::sw128_kmajor_desc(tc::smem_addr(stg));
      const uint64_t base1 = tc::sw128_kmajor_desc(tc::smem_addr(stg + Ly.stage_bytes));
      for (int s = 0, g = 0, k = 0;; ++s) {
        const int st = s % S, b = s & 1;
        if (abort_sh) break;
        if (s >= 2 && !tc::mbar_wait(&bar_tfree[b], ((s - 2) >> 1) & 1, status)) { abort_sh = 1; break; }
        const int tile = stage_tile[st];
        if (g == 0) {
          tile_slot[k & 1] = tile;
          tc::mbar_arrive(&bar_tile);
        }
        if (++g == nvg) { g = 0; ++k; }
        if (tile < 0) break;
        if (!tc::mbar_wait(&bar_ld[st], (s / S) & 1, status)) { abort_sh = 1; break; }
        tc::fence_after_sync();
        const uint64_t sbase = st == 0 ? base0 : base1;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const int p = ks >> 2, koff = (ks & 3) * 32;
          const uint64_t ad = sbase + (uint64_t)((R * 256 + p * TN * 128 + koff) >> 4);   // keys (M)
          const uint64_t bd = sbase + (uint64_t)((p * R * 128 + koff) >> 4);              // query rows (N)
          tc::umma_f16(tmem + (uint32_t)(b * NCOL), ad, bd, idesc, ks > 0 ? 1u : 0u);
        }
        tc::umma_commit(&bar_full[b]);
        tc::umma_commit(&bar_sfree[st]);
        if (!tc::mbar_wait(&bar_sfree[st], (s / S) & 1, status)) { abort_sh = 1; break; }
        load_step(s + S);
      }
    }
    __syncwarp();
  } else {
    // ---------------- epilogue: 16 warps ----------------
    const int lg = warp & 3, q = warp >> 2;             // TMEM lane group (32 keys), column quarter
    const int key = 32 * lg + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * lg) << 16);
    const float rs = 1.0f / sqrtf((float)pl.D);
    const bool last_row = q == 3;                       // this quarter ends with window row W - 1 ...
    float* part = reinterpret_cast<float*>(a.ws + pl.off_ph_part);   // [2][slots][H][n]
    float* qrow = reinterpret_cast<float*>(a.ws + pl.off_ph_qrow);
    float* q2w = reinterpret_cast<float*>(a.ws + pl.off_ph_q2w);
    float* entp = reinterpret_cast<float*>(a.ws + pl.off_ph_ent);   // [ph_ent_parts][H]
    const size_t slot_stride = (size_t)pl.H * pl.n;
    const int nslots = 4 * HALVES;
    int tile = -1, vg = 0, hf = 0;
    auto advance = [&](int& g) {
      if constexpr (HALVES == 1) {
        g = g + 1 == ngroups ? 0 : g + 1;
      } else {
        vg = vg + 1 == nvg ? 0 : vg + 1;
        if (++g == ngroups) { g = 0; hf = hf + 1 == HALVES ? 0 : hf + 1; }
      }
    };
    for (int s = 0, g = 0, k = 0; s < ntiles * nvg; ++s, advance(g)) {
      if (HALVES == 1 ? g == 0 : vg == 0) {   // a new tile
        bool got = __shfl_sync(0xffffffffu, epi_abort == 0, 0);
        if (got) got = __all_sync(0xffffffffu, tc::mbar_wait(&bar_tile, k & 1, status));
        if (!got) {
          if (lane == 0) { epi_abort = 1; abort_sh = 1; }
          break;
        }
        tile = tile_slot[k & 1];
        ++k;
        if (tile < 0) break;
      }
      const int j = tile * TN + key;
      bool ok = !epi_abort;
      if (ok && !tc::mbar_wait(&bar_full[s & 1], (s >> 1) & 1, status)) ok = false;
      ok = __all_sync(0xffffffffu, ok);
      if (!ok && lane == 0) epi_abort = 1;
      if (!ok) continue;
      tc::fence_after_sync();
      const F2 l2e = f2(kLog2e, kLog2e);
      const uint32_t col0 = (uint32_t)((s & 1) * NCOL + 4 * RPQ * q);
      const bool edge = tile * TN + TN - 1 > pl.n - W;
      F2 tw01 = f2(0.f, 0.f), tw23 = tw01, cl01 = tw01, cl23 = tw01, qa01 = tw01, qa23 = tw01;
      auto chunks = [&](auto etag) {
        constexpr bool EDGE = decltype(etag)::value;
#pragma unroll
        for (int c = 0; c < NCH; ++c) {   // 16 columns: window rows RS hf + RPQ q + 4 c + i, heads 0..3
          uint32_t r16[16];
          __syncwarp();
          tc::tmem_ld16_nowait(lane_base + col0 + 16 * c, r16);
          tc::tmem_wait_ld();
          if (c == NCH - 1) {
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&bar_tfree[s & 1]);
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int r = RS * hf + RPQ * q + 4 * c + i;
            const float4 nL = snlse4[g * W + r];
            const F2 x01 = round_f2<DT>(__uint_as_float(r16[4 * i]), __uint_as_float(r16[4 * i + 1]), rs);
            const F2 x23 = round_f2<DT>(__uint_as_float(r16[4 * i + 2]), __uint_as_float(r16[4 * i + 3]), rs);
            F2 p01 = ex2_2(fma2(x01, l2e, f2(nL.x, nL.y)));
            F2 p23 = ex2_2(fma2(x23, l2e, f2(nL.z, nL.w)));
            if constexpr (EDGE) {
              if (j > pl.n - W + r) { p01 = f2(0.f, 0.f); p23 = p01; }   // causal mask (and keys past n)
            }
            if constexpr (!PRE) {
              const float4 w4 = sq2w4[g * W + r];
              tw01 = fma2(p01, f2(w4.x, w4.y), tw01);
              tw23 = fma2(p23, f2(w4.z, w4.w), tw23);
              cl01 = add2(cl01, p01);
              cl23 = add2(cl23, p23);
            }
            if (c == NCH - 1 && i == 3) { qa01 = p01; qa23 = p23; }
          }
        }
      };
      if (edge) chunks(BoolTag<true>{});
      else chunks(BoolTag<false>{});
      const int h0 = g * G;
      const float qa[4] = {f2lo(qa01), f2hi(qa01), f2lo(qa23), f2hi(qa23)};
      if constexpr (PRE) {
        if (last_row && hf == HALVES - 1 && j >= pl.n - W && j < pl.n)
#pragma unroll
          for (int hd = 0; hd < 4; ++hd) q2w[(size_t)(h0 + hd) * W + (j - (pl.n - W))] = qa[hd];
      } else {
        if (j < pl.n) {
          const int slot = 4 * hf + q;
          float* pt = part + (size_t)slot * pl.H * pl.n + (size_t)h0 * pl.n + j;
          float* pc = pt + (size_t)nslots * slot_stride;
          const float tw[4] = {f2lo(tw01), f2hi(tw01), f2lo(tw23), f2hi(tw23)};
          const float cl[4] = {f2lo(cl01), f2hi(cl01), f2lo(cl23), f2hi(cl23)};
#pragma unroll
          for (int hd = 0; hd < 4; ++hd) {
            pt[(size_t)hd * pl.n] = tw[hd];
            pc[(size_t)hd * pl.n] = cl[hd];
          }
        }
        if (last_row && hf == HALVES - 1) {   // warp-uniform
          const int t32 = tile * 4 + lg;
#pragma unroll
          for (int hd = 0; hd < 4; ++hd) {
            if (j < pl.n) qrow[(size_t)(h0 + hd) * pl.n + j] = qa[hd];
            const float t = warp_sum(j < pl.n ? qa[hd] * logf(qa[hd] + 1e-10f) : 0.f);
            if (lane == 0) entp[(size_t)t32 * pl.H + h0 + hd] = t;
          }
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 0) tc::tmem_dealloc(tmem, ncols);
}

template <int DT, int WIN, bool PRE>
__global__ void __launch_bounds__(kPTThreads, 1)
    k_tc_ph(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
            const __grid_constant__ WinArgs a) {
  tc_ph_body<DT, WIN, PRE>(tmq, tmk, a);
}

// two / col [H][n] = the sum of the per-head pass's partial slots, in slot order
__global__ void __launch_bounds__(256) k_ph_combine(WinArgs a) {
  const Plan& pl = a.pl;
  const float* part = reinterpret_cast<const float*>(a.ws + pl.off_ph_part);
  float* two = reinterpret_cast<float*>(a.ws + pl.off_ph_two);
  float* col = reinterpret_cast<float*>(a.ws + pl.off_ph_col);
  const size_t total = (size_t)pl.H * pl.n, nsl = (size_t)pl.ph_slots;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    float t = 0.f, c = 0.f;
    for (size_t k = 0; k < nsl; ++k) {
      t += __ldcg(part + k * total + i);
      c += __ldcg(part + (nsl + k) * total + i);
    }
    two[i] = t;
    col[i] = c;
  }
}

template <int DT, int WIN>
static cudaError_t launch_tc_ph_w(const WinArgs& a, const CUtensorMap& tq, const CUtensorMap& tk, cudaStream_t st) {
  const Plan& pl = a.pl;
  const size_t smem = ph_layout(pl).total;
  cudaError_t e = ensure_dynamic_smem((const void*)k_tc_ph<DT, WIN, true>, smem);
  if (e == cudaSuccess) e = ensure_dynamic_smem((const void*)k_tc_ph<DT, WIN, false>, smem);
  if (e != cudaSuccess) return e;
  const int pre = (pl.n - 1) / kPTTN - (pl.n - WIN) / kPTTN + 1;
  const int ntn = (pl.n + kPTTN - 1) / kPTTN;
  k_tc_ph<DT, WIN, true><<<pre, kPTThreads, smem, st>>>(tq, tk, a);
  k_tc_ph<DT, WIN, false><<<ntn < 148 ? ntn : 148, kPTThreads, smem, st>>>(tq, tk, a);
  return cudaGetLastError();
}

template <int DT>
static cudaError_t launch_tc_ph(const WinArgs& a, cudaStream_t st) {
  const Plan& pl = a.pl;
  const int rs = pl.W < 64 ? pl.W : 64;
  CUtensorMap tq, tk;
  if (!make_tmap_pairs(&tq, a.q, DT, pl.n, pl.H, a.qhs, a.qts, rs, pl.G) ||
      !make_tmap(&tk, a.k, DT, pl.n, pl.Hkv, a.khs, a.kts, kPTTN))
    return cudaErrorInvalidResourceHandle;   // TMA descriptor encoding refused the layout
  cudaError_t e;
  if (pl.W == 32) e = launch_tc_ph_w<DT, 32>(a, tq, tk, st);
  else if (pl.W == 64) e = launch_tc_ph_w<DT, 64>(a, tq, tk, st);
  else e = launch_tc_ph_w<DT, 128>(a, tq, tk, st);
  if (e != cudaSuccess) return e;
  const size_t total = (size_t)pl.H * pl.n;
  const unsigned blocks = (unsigned)((total + 255) / 256 < 148 * 8 ? (total + 255) / 256 : 148 * 8);
  k_ph_combine<<<blocks, 256, 0, st>>>(a);
  return cudaGetLastError();
}

// per-head pass: tcgen05 keys-on-lanes form where the plan allows it, else mma.sync / SIMT
cudaError_t launch_ph_pass(const WinArgs& a, cudaStream_t st) {
  if (a.pl.ph_tc) return a.pl.dtype == CKV_BF16 ? launch_tc_ph<CKV_BF16>(a, st) : launch_tc_ph<CKV_FP16>(a, st);
  return launch_ph_pass_mma(a, st);
}

// ---------------------------------------------------------------------------
// exact entropy / mass: reduce the pooling pass's partials, then (last CTA) verify
// the head sets and run the window chain
// ---------------------------------------------------------------------------
// Reduces, per row, a strided set of partials with 8 loads in flight per thread.
CKV_DEV float sum_parts(const float* base, int nparts, size_t stride, int first, int step) {
  float acc = 0.f;
  for (int t = first; t < nparts; t += 8 * step) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = (t + u * step < nparts) ? __ldcg(base + (size_t)(t + u * step) * stride) : 0.f;
#pragma unroll
    for (int u = 0; u < 8; ++u) acc += v[u];
  }
  return acc;
}

// Thread (row lane, stream): 32 rows per CTA, 16 partial streams (one per warp).
// Rows [0, H*W) are the exact entropy of each (head, window row), [H*W, 2*H*W) its
// transient mass, [2*H*W, 2*H*W + 2W) the row sums of the pooled QI / HI rows; the
// three outputs are contiguous in the stats area.
constexpr int kReduceStreams = 16;

__global__ void __launch_bounds__(32 * kReduceStreams) k_pool_reduce(WinArgs a) {
  const Plan& pl = a.pl;
  Header* hdr = reinterpret_cast<Header*>(a.ws);
  if (a.fixup_pass && *reinterpret_cast<volatile int32_t*>(&hdr->fixup) == 0) return;
  extern __shared__ __align__(16) char rsmem[];
  const float* epart = reinterpret_cast<const float*>(a.ws + pl.off_epart);
  const float* mpart = reinterpret_cast<const float*>(a.ws + pl.off_mpart);
  const float* rspart = reinterpret_cast<const float*>(a.ws + pl.off_rspart);
  float* out = reinterpret_cast<float*>(a.ws + pl.off_stats);   // [H*W] entropy, [H*W] mass, [2][W] row sums
  const int HW = pl.H * pl.W;
  const int nrows = 2 * HW + 2 * pl.W;
  const int lane = threadIdx.x & 31, q = threadIdx.x >> 5;
  __shared__ float sp[kReduceStreams][32];
  const bool exact = hdr->need_exact != 0;   // else the moments pass's values stand
  // blocks of 32 rows, strided over the grid (the re-run launches a few CTAs: it returns at
  // once unless the head sets changed, and then speed matters less than launch cost)
  const int nblk = (nrows + 31) / 32;
  for (int blk = blockIdx.x; blk < nblk; blk += gridDim.x) {
    const int row = blk * 32 + lane;
    float e = 0.f;
    if (row < HW) {
      if (exact) e = sum_parts(epart + row, pl.e_parts, (size_t)HW, q, kReduceStreams);
    } else if (row < 2 * HW) {
      if (exact) e = sum_parts(mpart + (row - HW), pl.e_parts, (size_t)HW, q, kReduceStreams);
    } else if (row < nrows) {
      const int ch = (row - 2 * HW) / pl.W, rr = (row - 2 * HW) % pl.W;
      const int src = (ch == 1 && pl.hi_rows) ? 1 : 0;
      e = sum_parts(rspart + (size_t)src * pl.rs_parts * pl.W + rr, pl.rs_parts, (size_t)pl.W, q, kReduceStreams);
    }
    sp[q][lane] = e;
    __syncthreads();
    if (threadIdx.x < 32 && row < nrows) {
      float t = 0.f;
      for (int k = 0; k < kReduceStreams; ++k) t += sp[k][threadIdx.x];
      out[row] = t;
    }
    __syncthreads();   // sp is reused by the next block
  }
  if (pl.lanes_pool || (pl.tc_pool && !exact)) {
    // column sums and g totals behind the keys-on-lanes pooling pass: pool_blocks row-block
    // partials per key (4, or 8 for W = 128), one 64-key slice per warp, added in a fixed order
    const float* colpart = reinterpret_cast<const float*>(a.ws + pl.off_colpart);   // [2][pool_blocks][n_pad]
    float* colsum = reinterpret_cast<float*>(a.ws + pl.off_colsum);
    float* gtile = reinterpret_cast<float*>(a.ws + pl.off_gtile);
    const bool tempered = a.p.neumann_temperature != 1.0f && a.p.neumann_temperature > 0.f;
    const float invT = tempered ? 1.0f / a.p.neumann_temperature : 1.0f;
    const int nslice = (pl.hi_rows ? 2 : 1) * pl.ncol_tiles;
    const int nwarps = (int)(gridDim.x * (blockDim.x >> 5));
    for (int sl = (int)blockIdx.x * (int)(blockDim.x >> 5) + q; sl < nslice; sl += nwarps) {
      const int c2 = sl / pl.ncol_tiles, t = sl % pl.ncol_tiles;
      float gh[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int jj = t * 64 + 32 * h + lane;   // < n_pad
        const float* cp = colpart + (size_t)c2 * pl.pool_blocks * pl.n_pad + jj;
        float c = (__ldcg(cp) + __ldcg(cp + pl.n_pad)) + (__ldcg(cp + 2 * (size_t)pl.n_pad) + __ldcg(cp + 3 * (size_t)pl.n_pad));
        if (pl.pool_blocks == 8) {
          const float* cq = cp + 4 * (size_t)pl.n_pad;
          c += (__ldcg(cq) + __ldcg(cq + pl.n_pad)) + (__ldcg(cq + 2 * (size_t)pl.n_pad) + __ldcg(cq + 3 * (size_t)pl.n_pad));
        }
        colsum[(size_t)c2 * pl.n_pad + jj] = c;
        float gg = 0.f;
        if (jj < pl.n_p) {
          gg = fmaxf(c, 1e-6f);
          if (tempered) gg = powf(gg, invT);
        }
        gh[h] = warp_sum(gg);
      }
      if (lane == 0) gtile[(size_t)c2 * pl.ncol_tiles * 8 + t] = gh[0] + gh[1];
    }
  }
  __shared__ bool last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(&hdr->cnt_pool, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  window_pool_finish(a, rsmem);
}

size_t pool_reduce_smem(const Plan& pl) {
  return sizeof(float) * chain_smem(pl.W, pl.H).total;
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
  // opt in to the dynamic shared memory of the SIMT kernels (tensor-core launchers do their own)
  {
    const cudaError_t e = stage == 0 ? ensure_dynamic_smem((const void*)k_window_stats<DT>, stats_smem<DT>(pl))
                                     : ensure_dynamic_smem((const void*)k_window_pool<DT>, pool_smem<DT>(pl));
    if (e != cudaSuccess) return e;
  }
  if (stage == 0) {
    if constexpr (DT != CKV_FP32) {
      if (pl.tc) return launch_tc_stats<DT>(a, st);
    }
    k_window_stats<DT><<<dim3(pl.nstat_chunks, pl.nbatch), 256, stats_smem<DT>(pl), st>>>(a);
  } else {
    WinArgs b = a;
    b.fixup_pass = stage == 2 ? 1 : 0;
    bool launched = false;
    if constexpr (DT != CKV_FP32) {
      if (pl.tc_pool) {   // each returns at once unless its branch (exact recomputation or not) runs
        const cudaError_t e = stage == 1 ? launch_tc_pool_any<DT>(b, st) : launch_tc_pool<DT>(b, st);
        if (e != cudaSuccess) return e;
        launched = true;
      } else if (pl.lanes_pool) {
        // the exact branch's clamped entropy / mass on the tensor cores (returns at once when
        // the moments pass settled the head sets), then keys-on-lanes pooling; the re-run
        // pools again only when the exact sets differ
        if (stage == 1) {
          const cudaError_t e = launch_tc_stats<DT, true>(b, st);
          if (e != cudaSuccess) return e;
        }
        const cudaError_t e = launch_tc_pool_lanes<DT>(b, st);
        if (e != cudaSuccess) return e;
        launched = true;
      }
    }
    if (!launched) k_window_pool<DT><<<pl.ncol_tiles, 256, pool_smem<DT>(pl), st>>>(b);
    if (stage == 1) stage_mark(st);   // pooling kernels | reduction (timing only)
    const size_t rsm = pool_reduce_smem(pl);
    { const cudaError_t e = ensure_dynamic_smem((const void*)k_pool_reduce, rsm); if (e != cudaSuccess) return e; }
    const int nblk = (2 * pl.H * pl.W + 2 * pl.W + 31) / 32;
    k_pool_reduce<<<stage == 2 ? (nblk < 8 ? nblk : 8) : nblk, 32 * kReduceStreams, rsm, st>>>(b);
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

// ---------------------------------------------------------------------------
// head-sharded scoring: head sets from all ranks' statistics, pooling with given sets
// ---------------------------------------------------------------------------
// One warp: the head sets of the whole layer from its per-head entropy / mass (every
// rank computes the same sets from the same all-gathered values).
__global__ void __launch_bounds__(32) k_choose_heads(ckv_params p, int H, const float* ent, const float* mass,
                                                     uint64_t* sets, int32_t* mode) {
  const int h = threadIdx.x;
  const bool v = h < H;
  const HeadSets r = select_heads_warp(p, H, v ? ent[h] : INFINITY, v ? mass[h] : -INFINITY, 0.f);
  if (h == 0) { sets[0] = r.qs; sets[1] = r.hs; mode[0] = r.hm; mode[1] = r.nhi; }
}

cudaError_t launch_choose_heads(const ckv_params& p, int H, const float* ent, const float* mass, uint64_t* sets,
                                int32_t* mode, cudaStream_t st) {
  k_choose_heads<<<1, 32, 0, st>>>(p, H, ent, mass, sets, mode);
  return cudaGetLastError();
}

// After the moments pass: this rank's share of the given sets (heads head_off ..
// head_off + H_local - 1 of the layer) replaces the workspace's own, the pooling pass
// takes the settled branch, and HI pools as a SUM (n_hi = 1): the ranks' partial rows
// are combined by a max (QI) and a sum (HI) before the mean.
__global__ void k_set_heads(char* ws, int head_off, int h_local, const uint64_t* sets, const int32_t* mode) {
  Header* hdr = reinterpret_cast<Header*>(ws);
  const uint64_t mask = h_local >= 64 ? ~0ull : ((1ull << h_local) - 1ull);
  hdr->qi_heads = (sets[0] >> head_off) & mask;
  hdr->hi_heads = (sets[1] >> head_off) & mask;
  hdr->hi_mode = mode[0];
  hdr->n_hi = 1;
  hdr->need_exact = 0;
  hdr->fixup = 0;
}

cudaError_t launch_set_heads(char* ws, int head_off, int h_local, const uint64_t* sets, const int32_t* mode,
                             cudaStream_t st) {
  k_set_heads<<<1, 1, 0, st>>>(ws, head_off, h_local, sets, mode);
  return cudaGetLastError();
}

cudaError_t launch_window(const WinArgs& a, cudaStream_t st) {
  for (int s = 0; s < 3; ++s) {
    const cudaError_t e = launch_window_stage(a, s, st);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace ckv
