// K / V compaction of the CircuitKV prefill path (reference pyramidkv_utils.py
// PU:3496-3517 shared eviction, PU:3448-3462 per-head eviction): the kept prefix
// rows followed by the local window, written once into [H, out_len, D].
// Shared eviction reads each distinct KV head row once and writes it to the
// `groups` query heads that share it (the reference's repeat_kv layout).
#include "ckv_common.cuh"
#include "ckv_gather.h"

namespace ckv {

constexpr int kGatherRows = 16;   // token rows per block; 16 threads per 256-byte bf16 row

// One thread per 16-byte vector of one kept row of one KV head; the vector is
// written to every query head of the group (per-head mode: one query head).
template <typename T>
__global__ void __launch_bounds__(256) k_gather(const GatherArgs a) {
  constexpr int kVec = 16 / sizeof(T);
  const int nvec = a.D / kVec;                     // vectors per row (16 for bf16, 32 for fp32)
  const int rows_per_block = 256 / nvec;
  const int t = blockIdx.x * rows_per_block + threadIdx.x / nvec;   // output token
  const int v = threadIdx.x % nvec;
  const int which = blockIdx.z;                    // 0 = K, 1 = V
  if (t >= a.out_len) return;
  const T* src = static_cast<const T*>(which ? a.v : a.k);
  const int64_t hs = which ? a.vhs : a.khs, ts = which ? a.vts : a.kts;
  T* dst = static_cast<T*>(which ? a.out_v : a.out_k);
  const int nk = a.out_len - a.W;                  // kept prefix rows
  if (a.per_head) {
    const int h = blockIdx.y;                      // query head
    int tok = (t < nk) ? __ldg(a.idx + (size_t)h * nk + t) : (a.n - a.W + (t - nk));
    if (tok < 0 || tok >= a.n) tok = 0;            // never expected: keeps the read in bounds
    const uint4 x = __ldg(reinterpret_cast<const uint4*>(src + (h / a.G) * hs + (int64_t)tok * ts) + v);
    reinterpret_cast<uint4*>(dst + ((size_t)h * a.out_len + t) * a.D)[v] = x;
  } else {
    const int g = blockIdx.y;                      // KV head
    int tok = a.identity ? t : ((t < nk) ? __ldg(a.idx + t) : (a.n - a.W + (t - nk)));
    if (tok < 0 || tok >= a.n) tok = 0;            // never expected: keeps the read in bounds
    const uint4 x = __ldg(reinterpret_cast<const uint4*>(src + g * hs + (int64_t)tok * ts) + v);
    if (a.distinct) {   // each KV head once
      reinterpret_cast<uint4*>(dst + ((size_t)g * a.out_len + t) * a.D)[v] = x;
    } else {
      for (int r = 0; r < a.G; ++r)
        reinterpret_cast<uint4*>(dst + ((size_t)(g * a.G + r) * a.out_len + t) * a.D)[v] = x;
    }
  }
}

cudaError_t launch_gather(const GatherArgs& a, int dtype, cudaStream_t st) {
  const int nvec = a.D / (dtype == CKV_FP32 ? 4 : 8);
  const int rows_per_block = 256 / nvec;
  const dim3 grid((a.out_len + rows_per_block - 1) / rows_per_block, a.per_head ? a.H : a.Hkv, 2);
  switch (dtype) {
    case CKV_BF16: k_gather<__nv_bfloat16><<<grid, 256, 0, st>>>(a); break;
    case CKV_FP16: k_gather<__half><<<grid, 256, 0, st>>>(a); break;
    default: k_gather<float><<<grid, 256, 0, st>>>(a); break;
  }
  return cudaGetLastError();
}

}  // namespace ckv
