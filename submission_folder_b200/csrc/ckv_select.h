// Launch interface of the selection kernels.
#pragma once

#include <cuda_runtime.h>

#include "ckv_plan.h"

namespace ckv {

struct SelArgs {
  Plan pl;
  ckv_params p;
  char* ws;
  int32_t* out_idx;
  float* out_scores;     // optional [2][n]: the two vectors the ranks are taken of
  int given;             // 1: score vectors come from ga / gb / gc instead of the sweep
  const float* ga;
  const float* gb;
  const float* gc;
  int finish_only;       // 1: stop after the finished chain scores (written to out_scores)
  int parts;             // CTAs per score vector (set by launch_select)
  int narrow;            // 1: the portable 8-CTA cluster (layers run concurrently, so fewer SMs
                         //    per selection outweigh its longer latency)
};

// Per-head eviction: finishing, global HI ranks and the per-head selection.
struct PhArgs {
  Plan pl;
  ckv_params p;
  char* ws;
  int32_t* out_idx;    // [H][s + kk]
  float eq, eh;        // qi_gamma^(K/2), hi_gamma^(K/2)
};
cudaError_t launch_ph_select(const PhArgs& a, cudaStream_t st);

size_t select_smem_bytes_n(int n);
cudaError_t launch_select(const SelArgs& a, cudaStream_t st);
// Selection stage with its scratch in a static device array (no workspace argument);
// noalloc_scratch gives that array's device address on the current device.
cudaError_t noalloc_scratch(void** out);
int select_scores_noalloc(const ckv_params* p, int32_t n, const float* a, const float* b,
                          const float* c, int32_t* out_idx, float* out_scores, cudaStream_t st,
                          const char** why);
// H2O column sums of full_attn (mode max / weighted) and bridge importance (dis + bridge).
cudaError_t launch_aux(const Plan& pl, const ckv_params& p, char* ws, cudaStream_t st);

}  // namespace ckv
