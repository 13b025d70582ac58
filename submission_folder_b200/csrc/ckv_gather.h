// Launch interface of the K / V gather.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace ckv {

struct GatherArgs {
  const void* k;
  int64_t khs, kts;
  const void* v;
  int64_t vhs, vts;
  void* out_k;
  void* out_v;
  const int32_t* idx;   // [out_len - W] (shared) or [H][out_len - W] (per head)
  int n, W, H, Hkv, G, D, out_len;
  int per_head;
  int identity;         // 1: keep every token (n < budget)
  int distinct;         // 1: write each KV head once ([Hkv, out_len, D]) instead of per query head
};

cudaError_t launch_gather(const GatherArgs& a, int dtype, cudaStream_t st);

}  // namespace ckv
