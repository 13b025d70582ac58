// Test infrastructure only: C entry points onto the reference's own decode-time graph
// kernels (CircuitKV/csrc/kernels/graph_update.cu, circuit_walker.cu, spectral_power.cu,
// compiled from their sources in place by oracle/Makefile with the reference's flags), so
// that GPU tests can compare the sm_100a kernels with them on the same inputs and PCG
// states.  The sequences follow CircuitGraph::update_and_step_circuit_combined
// (circuit_manager.cpp:592-740).
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
