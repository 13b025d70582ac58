// Launch interface of the window-attention kernels.
#pragma once

#include <cuda_runtime.h>

#include "ckv_plan.h"

namespace ckv {

struct WinArgs {
  const void* q;
  int64_t qhs, qts;
  const void* k;
  int64_t khs, kts;
  char* ws;          // layer workspace base
  int fixup_pass;    // pooling kernel: 1 = the re-run launched after a wrong speculation
  int tc_tn;         // tensor-core path: key columns per MMA tile
  int tc_tpc;        // tensor-core path: tiles per column chunk of the moments pass
  int tc_stages;     // tensor-core path: K-tile stages in shared memory
  int tc_min;        // moments pass: the tensor-core kernel wrote row minima (clamp bounds)
  int force_exact;   // pooling pass: always recompute the clamped entropy / mass
  ckv_params p;
  Plan pl;
};

size_t window_smem_bytes(const Plan& pl, bool pool);
cudaError_t launch_window(const WinArgs& a, cudaStream_t st);
cudaError_t launch_window_stage(const WinArgs& a, int stage, cudaStream_t st);
// Records the next per-stage timing event, if any are set (ckv_set_stage_events); the
// pooling stage marks the boundary between its pooling kernels and their reduction.
void stage_mark(cudaStream_t st);
// Per-head eviction pass: query rows, two-hop terms, column sums, query-row entropy.
cudaError_t launch_ph_pass(const WinArgs& a, cudaStream_t st);
// Head-sharded scoring: head sets of the whole layer from all heads' entropy / mass
// (sets[0] QI, sets[1] HI; mode[0] HI mode, mode[1] HI head count), and the given sets
// written into a workspace header after its moments pass (HI pooled as a sum).
cudaError_t launch_choose_heads(const ckv_params& p, int H, const float* ent, const float* mass, uint64_t* sets,
                                int32_t* mode, cudaStream_t st);
cudaError_t launch_set_heads(char* ws, int head_off, int h_local, const uint64_t* sets, const int32_t* mode,
                             cudaStream_t st);
// Column sums / row sums / window chain of pooled rows already in the workspace.
cudaError_t launch_rows_prep(const Plan& pl, const ckv_params& prm, char* ws, cudaStream_t st);

}  // namespace ckv
