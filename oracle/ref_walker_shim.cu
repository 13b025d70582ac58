// Test infrastructure only: a C entry point onto the reference's own influence walker
// (CircuitKV/csrc/kernels/influence_walker.cu, compiled from its source in place by
// oracle/Makefile) so that GPU tests can compare the sm_100a walker with it on the same
// attention matrix and PCG states.  The sequence follows
// CircuitGraph::update_and_step_influence_walker (circuit_manager.cpp:1241-1287): clear
// the visits, walk, positional adjustment and max normalisation over
// min(256, ceil(n / 256)) partial maxima.
#include <cuda_runtime.h>
#include <stdint.h>

namespace circuit_kv {
void launch_influence_walker_kernel(const float* attention, float* visits, uint64_t* rng_states, int seq_len,
                                    int current_idx, int num_walkers, int max_steps, int sink_size,
                                    cudaStream_t stream, float temperature, float explore_temp,
                                    float explore_ratio);
void launch_clear_influence_visits_kernel(float* visits, int seq_len, cudaStream_t stream);
void launch_find_max_and_normalize_kernel(float* visits, float* normalized, float* partial_max, int seq_len,
                                          int num_blocks, cudaStream_t stream, int sink_size);
}  // namespace circuit_kv

// states: [num_walkers][2] (state, inc); partial_max: 256 floats; visits, normalized: [n].
extern "C" int ref_influence_walk(const float* attn, int n, int current_idx, int num_walkers, int max_steps,
                                  int sink_size, float temperature, float explore_temp, float explore_ratio,
                                  uint64_t* states, float* visits, float* normalized, float* partial_max,
                                  void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  circuit_kv::launch_clear_influence_visits_kernel(visits, n, st);
  circuit_kv::launch_influence_walker_kernel(attn, visits, states, n, current_idx, num_walkers, max_steps,
                                             sink_size, st, temperature, explore_temp, explore_ratio);
  int blocks = (n + 255) / 256;
  if (blocks > 256) blocks = 256;
  circuit_kv::launch_find_max_and_normalize_kernel(visits, normalized, partial_max, n, blocks, st, sink_size);
  return (int)cudaGetLastError();
}
