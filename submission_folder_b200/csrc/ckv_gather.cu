// K / V compaction of the CircuitKV prefill path (reference pyramidkv_utils.py
// PU:3496-3517 shared eviction, PU:3448-3462 per-head eviction): the kept prefix
// rows followed by the local window, written once into [H, out_len, D].
// Shared eviction reads each distinct KV head row once and writes it to the
// `groups` query heads that share it (the reference's repeat_kv layout).
#include "ckv_common.cuh"
#include "ckv_gather.h"

namespace ckv {

constexpr int kGatherRows = 8;   // one warp per (token row, KV head)

template <typename T>
__global__ void __launch_bounds__(256) k_gather(const GatherArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * kGatherRows + warp;   // output token
  const int which = blockIdx.z;                    // 0 = K, 1 = V
  if (t >= a.out_len) return;
  const T* src = static_cast<const T*>(which ? a.v : a.k);
  const int64_t hs = which ? a.vhs : a.khs, ts = which ? a.vts : a.kts;
  T* dst = static_cast<T*>(which ? a.out_v : a.out_k);
  constexpr int kVec = 16 / sizeof(T);
  const int nvec = a.D / kVec;
  const int nk = a.out_len - a.W;                  // kept prefix rows
  if (a.per_head) {
    const int h = blockIdx.y;                      // query head
    const int g = h / a.G;
    int tok = (t < nk) ? a.idx[(size_t)h * nk + t] : (a.n - a.W + (t - nk));
    if (tok < 0 || tok >= a.n) tok = 0;   // never expected: keeps the read in bounds
    const uint4* s = reinterpret_cast<const uint4*>(src + g * hs + (int64_t)tok * ts);
    uint4* d = reinterpret_cast<uint4*>(dst + ((size_t)h * a.out_len + t) * a.D);
    for (int v = lane; v < nvec; v += 32) d[v] = __ldg(s + v);
  } else {
    const int g = blockIdx.y;                      // KV head
    int tok = a.identity ? t : ((t < nk) ? a.idx[t] : (a.n - a.W + (t - nk)));
    if (tok < 0 || tok >= a.n) tok = 0;   // never expected: keeps the read in bounds
    const uint4* s = reinterpret_cast<const uint4*>(src + g * hs + (int64_t)tok * ts);
    for (int v = lane; v < nvec; v += 32) {
      const uint4 x = __ldg(s + v);
      for (int r = 0; r < a.G; ++r) {
        uint4* d = reinterpret_cast<uint4*>(dst + ((size_t)(g * a.G + r) * a.out_len + t) * a.D);
        d[v] = x;
      }
    }
  }
}

cudaError_t launch_gather(const GatherArgs& a, int dtype, cudaStream_t st) {
  const dim3 grid((a.out_len + kGatherRows - 1) / kGatherRows, a.per_head ? a.H : a.Hkv, 2);
  switch (dtype) {
    case CKV_BF16: k_gather<__nv_bfloat16><<<grid, 256, 0, st>>>(a); break;
    case CKV_FP16: k_gather<__half><<<grid, 256, 0, st>>>(a); break;
    default: k_gather<float><<<grid, 256, 0, st>>>(a); break;
  }
  return cudaGetLastError();
}

}  // namespace ckv
