// Shared device helpers for the CircuitKV sm_100a kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/ckv.h"

#define CKV_DEV __device__ __forceinline__

namespace ckv {

constexpr int kMaxHeads = 64;      // head sets are 64-bit masks
constexpr int kMaxIters = 16;      // Neumann terms carried by the sweep (neumann_iterations <= 16)
constexpr int kMaxWindow = 128;    // window rows handled by the window kernels
constexpr int kHeadDim = 128;

// Device status bits recorded in the workspace header (never a trap).
enum : int32_t {
  kStatusTimeout = 1,      // a bounded wait gave up
  kStatusCount = 2,        // a selection produced an unexpected count
  kStatusNonFinite = 4     // non-finite scores were seen
};

// ---------------------------------------------------------------------------
// dtype traits
// ---------------------------------------------------------------------------
template <int DT> struct Elem;
template <> struct Elem<CKV_BF16> { using T = __nv_bfloat16; };
template <> struct Elem<CKV_FP16> { using T = __half; };
template <> struct Elem<CKV_FP32> { using T = float; };

CKV_DEV float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
CKV_DEV float to_f32(__half x) { return __half2float(x); }
CKV_DEV float to_f32(float x) { return x; }

// Round an fp32 value to the storage dtype and back (round to nearest even),
// as the reference's 16-bit matmul output and scalar division do.
template <int DT> CKV_DEV float round_dt(float x);
template <> CKV_DEV float round_dt<CKV_BF16>(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
template <> CKV_DEV float round_dt<CKV_FP16>(float x) { return __half2float(__float2half_rn(x)); }
template <> CKV_DEV float round_dt<CKV_FP32>(float x) { return x; }

// 2^x on the MUFU unit (PTX ex2.approx.ftz.f32; relative error ~2^-22).
CKV_DEV float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32 pairs (sm_100 add / mul / fma .f32x2): each lane of the pair is the
// IEEE-rounded scalar operation, so a pair op equals two scalar ops bit for bit.
struct F2 {
  uint64_t v;
};
CKV_DEV F2 f2(float lo, float hi) {
  F2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r.v) : "f"(lo), "f"(hi));
  return r;
}
CKV_DEV float f2lo(F2 a) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(a.v));
  return lo;
}
CKV_DEV float f2hi(F2 a) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(a.v));
  return hi;
}
CKV_DEV F2 fma2(F2 a, F2 b, F2 c) {
  F2 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r.v) : "l"(a.v), "l"(b.v), "l"(c.v));
  return r;
}
CKV_DEV F2 add2(F2 a, F2 b) {
  F2 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
  return r;
}
CKV_DEV F2 mul2(F2 a, F2 b) {
  F2 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
  return r;
}

// max(a, b, c) in one instruction (sm_100 three-input max.f32).
CKV_DEV float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
CKV_DEV F2 ex2_2(F2 a) { return f2(ex2(f2lo(a)), ex2(f2hi(a))); }

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// ---------------------------------------------------------------------------
// order-preserving float <-> uint32 keys (ascending key == ascending float)
// ---------------------------------------------------------------------------
CKV_DEV uint32_t float_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// ---------------------------------------------------------------------------
// warp / block reductions
// ---------------------------------------------------------------------------
// a / b correctly rounded, from y = RN(1/b) computed once per divisor: Markstein's
// correction (P. Markstein, "Computation of elementary functions on the IBM RISC
// System/6000 processor", IBM J. Res. Develop. 34(1), 1990).  q0 = RN(a*y) lies within
// one ulp of a/b, the residual a - b*q0 is exact in one FMA, and RN(q0 + residual*y)
// is RN(a/b) when no intermediate underflows or overflows.  Replaces a full IEEE
// division in loops that divide many values by the same divisor.
CKV_DEV float div_rcp(float a, float b, float y) {
  const float q0 = __fmul_rn(a, y);
  return __fmaf_rn(__fmaf_rn(-q0, b, a), y, q0);
}

CKV_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
// Sixteen warp sums at once (transpose reduction): returns, in lane l, the sum over
// the 32 lanes of v[idx], idx = ((l >> 4) & 1) * 8 + ((l >> 3) & 1) * 4 + ((l >> 2) & 1) * 2
// + ((l >> 1) & 1).  Each round halves the values a lane holds: it keeps the half
// selected by its lane bit and adds the partner's copy of that half: 16 shuffles and
// adds in place of 16 x 5.  v is clobbered.
CKV_DEV float warp_sum16(float (&v)[16]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 16, m = 8; o >= 2; o >>= 1, m >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int k = 0; k < m; ++k) {
      const float keep = up ? v[m + k] : v[k];
      const float send = up ? v[k] : v[m + k];
      v[k] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
}
// The same transpose reduction for 8 values: lanes 4r .. 4r + 3 end with row r's total,
// for row r = (lane >> 2) & 7.
CKV_DEV float warp_sum8(float (&v)[8]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 16, m = 4; o >= 4; o >>= 1, m >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int k = 0; k < m; ++k) {
      const float keep = up ? v[m + k] : v[k];
      const float send = up ? v[k] : v[m + k];
      v[k] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  const float t = v[0] + __shfl_xor_sync(0xffffffffu, v[0], 2);
  return t + __shfl_xor_sync(0xffffffffu, t, 1);
}
CKV_DEV float warp_min(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
CKV_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
CKV_DEV int warp_sum_int(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide reduction through `scratch` (>= 32 floats).  All threads get the result.
template <bool kMax>
__device__ __forceinline__ float block_reduce(float v, float* scratch) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  v = kMax ? warp_max(v) : warp_sum(v);
  __syncthreads();
  if (lane == 0) scratch[wid] = v;
  __syncthreads();
  float r = (lane < nw) ? scratch[lane] : (kMax ? -INFINITY : 0.f);
  if (wid == 0) r = kMax ? warp_max(r) : warp_sum(r);
  if (threadIdx.x == 0) scratch[0] = r;
  __syncthreads();
  r = scratch[0];
  __syncthreads();
  return r;
}

// Exclusive block scan of ints (returns exclusive prefix; *total = block sum).
__device__ __forceinline__ int block_exclusive_scan(int v, int* scratch, int* total) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  __syncthreads();
  if (lane == 31) scratch[wid] = x;
  __syncthreads();
  if (wid == 0) {
    int s = (lane < nw) ? scratch[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    if (lane < nw) scratch[lane] = s;
  }
  __syncthreads();
  int base = (wid > 0) ? scratch[wid - 1] : 0;
  int t = scratch[nw - 1];
  __syncthreads();
  if (total) *total = t;
  return base + x - v;
}

// Record a device-side failure in the workspace status word.
CKV_DEV void set_status(int32_t* status, int32_t bit) {
  if (status) atomicOr(status, bit);
}

}  // namespace ckv

#include <mutex>
#include <unordered_map>

namespace ckv {

// Opt a kernel in to `bytes` of dynamic shared memory.  The attribute is per
// kernel and only ever raised (a smaller request never lowers it under a larger
// launch issued elsewhere).
inline cudaError_t ensure_dynamic_smem(const void* func, size_t bytes) {
  static std::mutex mu;
  static std::unordered_map<const void*, size_t> have;
  std::lock_guard<std::mutex> lock(mu);
  size_t& h = have[func];
  if (bytes <= h) return cudaSuccess;
  const cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e == cudaSuccess) h = bytes;
  return e;
}

}  // namespace ckv
