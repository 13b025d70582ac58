// Influence walker of the legacy use_neumann=False path (CircuitKV influence_walker.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "ckv_plan.h"

namespace ckv {

struct WalkArgs {
  int n, current_idx, num_walkers, max_steps, sink;
  float inv_temp, inv_explore_temp, explore_ratio;
  int rng_mode;            // 0 Philox4x64-10 (counter based), 1 PCG-XSH-RR (state per walker)
  uint64_t seed;
  uint64_t* rng_state;     // PCG: [num_walkers][2] (state, inc); Philox: [0] = call counter
  int init_state;          // PCG: initialise the states from seed first
  float* visits;           // [n] raw visit counts (cleared by the launcher)
  float* scores;           // [n] normalised scores
  // dense matrix [n, n] (row i: how much position i attends to each j) ...
  const float* attn;
  // ... or the structured matrix of the pooled window rows (PU:3003-3034)
  const float* rows;       // [W][ld] pooled window rows
  int W, ld;
  const double* pre;       // [2][n_p + 1] prefix sums of h^(1/T) for the two temperatures
  const float* cinv;       // [n_p] 1 / (C[i-1] + 1e-8), 0 for row 0
  float* h2o;              // [n] column sums of full_attn (structured form)
};

// Dense walker: the reference's sampling, step for step (PCG: one thread per walker, the
// reference's sequential sums; Philox: one warp per walker, coalesced row reads).
cudaError_t launch_walk_dense(const WalkArgs& a, cudaStream_t st);
// Structured walker over pooled window rows: prefix rows sampled by binary search on
// prefix sums, window rows scanned; needs rows, hclamp, cinv and pre (see launch_walk_prep).
cudaError_t launch_walk_rows(const WalkArgs& a, cudaStream_t st);
// h, 1 / (C + 1e-8), the temperature prefix sums and the full_attn column sums (a.h2o)
// of pooled rows.
cudaError_t launch_walk_prep(const WalkArgs& a, float* hbuf, float* cinv, double* pre, cudaStream_t st);
// Raw generator output (tests, reproducing a walk): mode 0 Philox4x64-10 outputs for
// (key = seed, counter = {i / 4 block, stream}), mode 1 pcg32 outputs of stream `stream`.
cudaError_t launch_rng_fill(int mode, uint64_t seed, uint64_t stream, int count, uint64_t* out,
                            cudaStream_t st);

}  // namespace ckv
