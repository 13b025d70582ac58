// Launch interface of the decode-time CircuitGraph kernels (graph update, circuit walker,
// spectral power iteration, combined scores).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace ckv {

// Row `row` of the sparse graph: the top_k keys by dot product with q (scores [n] is scratch).
cudaError_t launch_graph_update(const void* q, const void* keys, int dtype, int n, int D, int row, int top_k,
                                float* scores, int32_t* adj, float* weights, cudaStream_t st);
// Absorbing walkers from `source` over the graph; visits (int32, not cleared) and PCG states.
cudaError_t launch_circuit_walk(const int32_t* adj, const float* w, int32_t* visits, uint64_t* states, int source,
                                int n, int top_k, int num_walkers, cudaStream_t st);
// PCG states [num_walkers][2] seeded (seed, walker).
cudaError_t launch_pcg_init(uint64_t* states, uint64_t seed, int num_walkers, cudaStream_t st);
// Power iteration from the uniform vector: v [n] (vtmp [n] scratch).
cudaError_t launch_spectral(const int32_t* adj, const float* w, int n, int top_k, int iters, float* v, float* vtmp,
                            cudaStream_t st);
// walker = visits as floats; spectral and walker divided by their maxima (in place);
// combined = their element-wise maximum.
cudaError_t launch_combine(const int32_t* visits, float* spectral, float* walker, float* combined, int n,
                           cudaStream_t st);

// Landmark walkers: H2O scores, stratified landmarks, walkers from every landmark and the
// query, normalised scores (mode 0 positional, 1 reachability, 2 absorbing form).  visits
// [n] cleared first; positions [32], count [1]; ws: landmark_workspace_floats(n) floats.
size_t landmark_workspace_floats(int n);
cudaError_t launch_landmark_walk(const float* attn, int n, int current_idx, int mode, int num_landmarks,
                                 int walkers_per_source, float query_boost, int min_spacing, float alpha,
                                 int absorb_at_landmarks, uint64_t* states, int32_t* visits, float* scores,
                                 int32_t* positions, int32_t* count, float* ws, cudaStream_t st);

}  // namespace ckv
