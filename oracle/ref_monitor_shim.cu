// Test infrastructure only: C entry points onto the reference's own decode-time graph
// kernels (CircuitKV/csrc/kernels/graph_update.cu, circuit_walker.cu, spectral_power.cu,
// landmark_walker.cu, landmark_absorbing_walker.cu, compiled from their sources in place by
// oracle/Makefile with the reference's flags), so that GPU tests can compare the sm_100a
// kernels with them on the same inputs and PCG states.  The sequences follow
// CircuitGraph::update_and_step_circuit_combined (circuit_manager.cpp:592-740) and the two
// landmark methods (circuit_manager.cpp:768-1164).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace circuit_kv {
void launch_graph_update_kernel(const __half* query, const __half* keys, int32_t* adj_list, float* adj_weights,
                                int current_idx, int seq_len, int head_dim, int top_k, cudaStream_t stream);
void launch_graph_update_kernel_fp32(const float* query, const float* keys, int32_t* adj_list, float* adj_weights,
                                     int current_idx, int seq_len, int head_dim, int top_k, cudaStream_t stream);
void launch_absorbing_walker_kernel(const int32_t* adj_list, const float* adj_weights, int32_t* visit_counts,
                                    uint64_t* rng_states, int source_node, int seq_len, int top_k, int num_walkers,
                                    cudaStream_t stream);
void launch_init_rng_kernel(uint64_t* rng_states, uint64_t seed, int num_walkers, cudaStream_t stream);
void launch_power_iteration(const int32_t* adj_list, const float* adj_weights, float* v, float* v_temp,
                            float* partial_sums, float* norm_out, int seq_len, int top_k, int num_iterations,
                            cudaStream_t stream);
void launch_convert_visits_kernel(const int32_t* visit_counts, float* scores, int seq_len, cudaStream_t stream);
void launch_normalize_to_unit_max(float* v, float* partial_max, float* max_out, int seq_len, int num_reduce_blocks,
                                  cudaStream_t stream);
void launch_max_combine_kernel(const float* spectral_scores, const float* walker_scores, float* combined_scores,
                               int seq_len, cudaStream_t stream);
void launch_reset_counts_kernel(int32_t* visit_counts, int max_seq_len, cudaStream_t stream);
void launch_compute_h2o_scores_kernel(const float* attention_matrix, float* h2o_scores, int seq_len,
                                      cudaStream_t stream);
void launch_select_landmarks_kernel(const float* attention_row_sums, int32_t* landmark_positions,
                                    int* num_landmarks_out, int seq_len, int max_landmarks, int min_spacing,
                                    int sink_buffer, int window_size, cudaStream_t stream);
void launch_cache_landmark_attention_kernel(const float* full_attention, float* landmark_attention,
                                            const int32_t* landmark_positions, int num_landmarks, int seq_len,
                                            cudaStream_t stream);
void launch_landmark_walker_kernel(const float* landmark_attention, const float* query_attention,
                                   const float* h2o_scores, int32_t* visit_counts, uint64_t* rng_states,
                                   const int32_t* landmark_positions, int num_landmarks, int walkers_per_source,
                                   float query_boost, int seq_len, cudaStream_t stream);
void launch_positional_normalize_kernel(const int32_t* visit_counts, float* normalized_scores, float* partial_max,
                                        int seq_len, int sink_size, float alpha, cudaStream_t stream);
void launch_reachability_normalize_kernel(const int32_t* visit_counts, float* normalized_scores,
                                          const int32_t* landmark_positions, int num_landmarks,
                                          int walkers_per_source, float query_boost, int seq_len, int sink_size,
                                          cudaStream_t stream);
void launch_landmark_absorbing_walker_kernel(const float* landmark_attention, const float* query_attention,
                                             const float* h2o_scores, int32_t* visit_counts, uint64_t* rng_states,
                                             const int32_t* landmark_positions, int num_landmarks,
                                             int walkers_per_source, float query_boost, int seq_len,
                                             bool absorb_at_landmarks, cudaStream_t stream);
void launch_landmark_reachability_normalize_kernel(const int32_t* visit_counts, float* normalized_scores,
                                                   const int32_t* landmark_positions, int num_landmarks,
                                                   int walkers_per_source, float query_boost, int seq_len,
                                                   int sink_size, cudaStream_t stream);
}  // namespace circuit_kv

// dtype 1: fp16, 2: fp32 (the reference's two graph kernels)
extern "C" int ref_graph_update(const void* q, const void* keys, int dtype, int n, int head_dim, int row, int top_k,
                                int32_t* adj, float* w, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == 1)
    circuit_kv::launch_graph_update_kernel(static_cast<const __half*>(q), static_cast<const __half*>(keys), adj, w, row,
                                           n, head_dim, top_k, st);
  else
    circuit_kv::launch_graph_update_kernel_fp32(static_cast<const float*>(q), static_cast<const float*>(keys), adj, w,
                                                row, n, head_dim, top_k, st);
  return (int)cudaGetLastError();
}

extern "C" int ref_init_rng(uint64_t* states, uint64_t seed, int num_walkers, void* stream) {
  circuit_kv::launch_init_rng_kernel(states, seed, num_walkers, static_cast<cudaStream_t>(stream));
  return (int)cudaGetLastError();
}

extern "C" int ref_circuit_walk(const int32_t* adj, const float* w, int32_t* visits, uint64_t* states, int source,
                                int n, int top_k, int num_walkers, void* stream) {
  circuit_kv::launch_absorbing_walker_kernel(adj, w, visits, states, source, n, top_k, num_walkers,
                                             static_cast<cudaStream_t>(stream));
  return (int)cudaGetLastError();
}

// scratch: partial sums [256] + one scalar
extern "C" int ref_spectral_combined(const int32_t* adj, const float* w, const int32_t* visits, int n, int top_k,
                                     int iters, float* v, float* vtmp, float* walker, float* combined, float* scratch,
                                     void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  circuit_kv::launch_power_iteration(adj, w, v, vtmp, scratch, scratch + 256, n, top_k, iters, st);
  circuit_kv::launch_convert_visits_kernel(visits, walker, n, st);
  int nb = (n + 255) / 256;
  if (nb > 256) nb = 256;
  circuit_kv::launch_normalize_to_unit_max(v, scratch, scratch + 256, n, nb, st);
  circuit_kv::launch_normalize_to_unit_max(walker, scratch, scratch + 256, n, nb, st);
  circuit_kv::launch_max_combine_kernel(v, walker, combined, n, st);
  return (int)cudaGetLastError();
}

// The landmark methods' sequence (circuit_manager.cpp:768-1164) on caller buffers: mode 0
// positional, 1 reachability (update_and_step_landmark_walker), 2 the absorbing walker.
// positions [32] and count [1] as the reference's landmark_positions_ / num_landmarks_selected_
// (count zeroed first, as at the reference's allocation); h2o [n] out.  Synchronises.
extern "C" int ref_landmark_walk(const float* attn, int n, int current_idx, int mode, int num_landmarks,
                                 int walkers_per_source, float query_boost, int min_spacing, float alpha,
                                 int absorb_at_landmarks, uint64_t* states, int32_t* visits, float* scores,
                                 int32_t* positions, int32_t* count, float* h2o, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float *lm_attn = nullptr, *q_attn = nullptr, *pmax = nullptr;
  cudaMalloc(&lm_attn, (size_t)32 * n * sizeof(float));
  cudaMalloc(&q_attn, (size_t)n * sizeof(float));
  cudaMalloc(&pmax, (size_t)((n + 255) / 256 + 1) * sizeof(float));
  circuit_kv::launch_compute_h2o_scores_kernel(attn, h2o, n, st);
  circuit_kv::launch_select_landmarks_kernel(h2o, positions, count, n, num_landmarks, min_spacing, 20, 64, st);
  cudaStreamSynchronize(st);
  int actual = 0;
  cudaMemcpy(&actual, count, sizeof(int), cudaMemcpyDeviceToHost);
  if (actual > 0) circuit_kv::launch_cache_landmark_attention_kernel(attn, lm_attn, positions, actual, n, st);
  cudaMemcpyAsync(q_attn, attn + (size_t)current_idx * n, (size_t)n * sizeof(float), cudaMemcpyDeviceToDevice, st);
  circuit_kv::launch_reset_counts_kernel(visits, n, st);
  if (mode == 2) {
    circuit_kv::launch_landmark_absorbing_walker_kernel(lm_attn, q_attn, h2o, visits, states, positions, actual,
                                                        walkers_per_source, query_boost, n, absorb_at_landmarks != 0,
                                                        st);
    circuit_kv::launch_landmark_reachability_normalize_kernel(visits, scores, positions, actual, walkers_per_source,
                                                              query_boost, n, 4, st);
  } else {
    circuit_kv::launch_landmark_walker_kernel(lm_attn, q_attn, h2o, visits, states, positions, actual,
                                              walkers_per_source, query_boost, n, st);
    if (mode == 1)
      circuit_kv::launch_reachability_normalize_kernel(visits, scores, positions, actual, walkers_per_source,
                                                       query_boost, n, 4, st);
    else
      circuit_kv::launch_positional_normalize_kernel(visits, scores, pmax, n, 4, alpha, st);
  }
  cudaError_t e = cudaStreamSynchronize(st);
  if (e == cudaSuccess) e = cudaGetLastError();
  cudaFree(lm_attn);
  cudaFree(q_attn);
  cudaFree(pmax);
  return (int)e;
}
