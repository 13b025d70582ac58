/*
 * ckv.h -- C ABI of the B200-native CircuitKV prefill scoring + eviction path.
 *
 * The library replaces, for one prefill layer, the reference's
 * CircuitKVCluster.update_kv(key_states, query_states, value_states,
 * attention_mask, num_key_value_groups)
 * (KVCache-Factory/pyramidkv/pyramidkv_utils.py:2775-3519): window attention,
 * entropy-aware head pooling, the absorbing-Markov (Neumann) importance solve,
 * smoothing, rank-MAX selection, and the K/V gather.  It also replaces the
 * influence-walker pair of circuit_kv._C.CircuitGraph
 * (CircuitKV/csrc/pybind.cpp:263-300, circuit_manager.cpp:1190-1311).
 *
 * Conventions
 *   - All tensor arguments are raw device pointers; strides are in ELEMENTS.
 *   - Every entry point returns an int status (CKV_OK == 0, negative on error),
 *     never throws, and never synchronises the host.  Work is enqueued on the
 *     caller's stream.  ckv_last_error_string() describes the last failure of
 *     the calling thread.
 *   - The caller owns all memory: inputs, outputs and a workspace sized by
 *     ckv_workspace_size().  A workspace may be reused by calls that are
 *     ordered on one stream; calls that overlap on the GPU need separate
 *     workspaces.
 *   - Device-side failures (a bounded wait that ran out, an inconsistent
 *     count) are recorded in the workspace's status word and read back with
 *     ckv_read_status(); no kernel traps.
 */
#ifndef CKV_H_
#define CKV_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* ckv_stream_t;   /* == cudaStream_t */

enum ckv_status {
  CKV_OK = 0,
  CKV_ERR_ARG = -1,          /* bad shape, stride, pointer or parameter */
  CKV_ERR_DTYPE = -2,        /* unsupported dtype */
  CKV_ERR_UNSUPPORTED = -3,  /* a parameter combination this build does not implement */
  CKV_ERR_WORKSPACE = -4,    /* workspace too small or misaligned */
  CKV_ERR_CUDA = -5,         /* a CUDA runtime call failed */
  CKV_ERR_DEVICE = -6        /* a kernel recorded a failure in the status word */
};

enum ckv_dtype { CKV_BF16 = 0, CKV_FP16 = 1, CKV_FP32 = 2 };

/* combination_mode of PU:1308 */
enum ckv_combination {
  CKV_COMB_DIS = 0,        /* MAX(rank QI, rank HI) (default) */
  CKV_COMB_MAX = 1,        /* MAX(rank H2O, rank influence); "geometric" and "sum" take this branch */
  CKV_COMB_WEIGHTED = 2,   /* h2o_weight * rank H2O + (1 - h2o_weight) * rank influence */
  CKV_COMB_UNION = 3,      /* union of QI / HI top-k split by qi_ratio */
  CKV_COMB_UNION_DA = 4    /* union on DA-weighted QI / HI */
};

/*
 * Mirrors the kwargs of CircuitKVCluster.__init__ (PU:1244-1331) that the
 * prefill path reads.  Booleans are 0/1.  ckv_default_params() fills the
 * values KVCache-Factory's run_longbench.py passes by default
 * (run_longbench.py:295-296, 505-548).
 */
typedef struct ckv_params {
  int32_t window_size;          /* W */
  int32_t max_capacity_prompt;  /* B: total kept tokens incl. sinks and window */
  int32_t sink_size;
  int32_t neumann_iterations;
  float neumann_temperature;
  float neumann_gamma;
  float qi_gamma;               /* per-head mode; already resolved (no None) */
  float hi_gamma;
  int32_t combination_mode;     /* enum ckv_combination */
  float h2o_weight;
  float qi_ratio;
  int32_t ablate_qi;
  int32_t ablate_hi;
  int32_t per_head_eviction;
  int32_t true_hub_hi;
  int32_t entropy_adaptive;
  int32_t smoothing_kernel;
  int32_t smooth_hi_only;
  int32_t use_gaussian;
  int32_t qi_kernel_size;
  int32_t hi_kernel_size;
  float gaussian_sigma;
  int32_t entropy_aware;
  int32_t top_k_heads;
  int32_t head_selection_mode;  /* 0 = entropy, 1 = mass */
  int32_t hi_pooling_mode;      /* 0 = mean, 1 = max */
  float hi_mass_threshold;
  int32_t hi_top_k_heads;
  float hi_mass_cdf;
  int32_t use_bridge_importance;
  int32_t bi_kernel_size;
} ckv_params;

/*
 * One layer's inputs, batch 1 (the reference's bsz == 1 semantics).
 * q: [num_heads, n, head_dim] view; only its last W rows are read.
 * k, v: the DISTINCT KV heads, [num_kv_heads, n, head_dim] view.  For the
 * reference's repeat_kv'd [1, H, n, D] tensors pass kv_head_stride =
 * groups * (their head stride): query head h reads KV head h / groups.
 */
typedef struct ckv_layer {
  const void* q;
  int64_t q_head_stride, q_tok_stride;
  const void* k;
  int64_t k_head_stride, k_tok_stride;
  const void* v;
  int64_t v_head_stride, v_tok_stride;
  int32_t n;             /* sequence length (q_len of PU:2806) */
  int32_t num_heads;     /* H (query heads) */
  int32_t num_kv_heads;  /* H / num_key_value_groups */
  int32_t head_dim;      /* D (128) */
  int32_t dtype;         /* enum ckv_dtype, shared by q, k, v and the K/V outputs */
} ckv_layer;

/* Outputs of one layer.  out_k / out_v: contiguous [H, out_len, D] in the input
 * dtype.  out_idx: the kept prefix positions in ascending order (sinks
 * included, local window excluded) -- [out_len - W] for shared eviction,
 * [H, out_len - W] for per-head eviction.  out_scores (optional, may be NULL): the
 * vectors the selection ranks, fp32.  Shared eviction: [2, n], the two smoothed vectors
 * (QI / HI for dis / union, influence / H2O for max / weighted).  Per-head eviction:
 * [H, 2, n - W] per head the finished, smoothed QI and HI vectors (HI: the raw window-row
 * column sums, H2O, when both are ablated), then [H] the query rows' entropies.
 * distinct_kv_heads: 0 (zero-initialised callers) writes the reference's layout, every
 * query head its KV head's rows (repeat_kv, llama_model.py:2918-2928); 1 writes each
 * DISTINCT KV head once, out_k / out_v [num_kv_heads, out_len, D] -- a quarter of the
 * writes and of the decode cache for 4 query heads per KV head, for a GQA-aware decode
 * attention (no reference counterpart; shared eviction only). */
typedef struct ckv_outputs {
  void* out_k;
  void* out_v;
  int32_t* out_idx;
  float* out_scores;
  int32_t distinct_kv_heads;
} ckv_outputs;

/* Fill *p with the CLI defaults of the reference (see above). */
void ckv_default_params(ckv_params* p);

/* Number of tokens each head keeps for a layer of length n (== n when
 * n < max_capacity_prompt: the reference returns its inputs unchanged). */
int ckv_output_len(const ckv_params* p, int32_t n, int32_t* out_len);

/* Workspace bytes one ckv_score_evict call on a layer of (n, H, D) needs. */
int ckv_workspace_size(const ckv_params* p, int32_t n, int32_t num_heads, int32_t num_kv_heads,
                       int32_t head_dim, size_t* bytes);

/* Replaces CircuitKVCluster.update_kv (PU:2775-3519) for one layer with
 * n >= max_capacity_prompt.  Enqueues the whole path on `stream`. */
int ckv_score_evict(const ckv_params* p, const ckv_layer* layer, void* workspace,
                    size_t workspace_bytes, const ckv_outputs* out, ckv_stream_t stream);

/* Many independent layers / sequences (each with batch-1 semantics, ragged n
 * allowed) in one call: the same results as `count` ckv_score_evict calls whose
 * workspaces are consecutive slices of `workspace` (each slice sized by
 * ckv_workspace_size for that layer, rounded up to 256 bytes).  `params` holds one
 * struct shared by every layer (params_count 1) or one per layer (params_count ==
 * count, e.g. per-layer budgets).  The layers run concurrently on internal streams
 * forked from and joined back to `stream`; every output is complete when `stream`
 * reaches the point of the call.  Arguments are validated before anything is
 * enqueued. */
int ckv_score_evict_batched(const ckv_params* params, int32_t params_count, const ckv_layer* layers,
                            int32_t count, void* workspace, size_t workspace_bytes,
                            const ckv_outputs* outs, ckv_stream_t stream);

/* Reads (synchronising on `stream`) and clears the device status word of a
 * workspace: 0 when every kernel since the last read finished normally.
 * workspace NULL reads the status word of ckv_select_scores_noalloc's static
 * scratch on the current device (the status of the last such call there). */
int ckv_read_status(void* workspace, ckv_stream_t stream, int32_t* device_status);

/* ---- stage entry points (used by the parity tests; same kernels as above) --- */

/* Selection from given fp32 score vectors (PU:3131-3196 + PU:2591-2644 /
 * PU:2489-2589): smoothing (dis mode), ranks, combination, keep mask and
 * compaction.  For dis: a = QI, b = HI, c = BI or NULL.  For max / weighted:
 * a = influence, b = H2O.  For union modes: a = QI, b = HI (already
 * DA-weighted for union_da).  Writes out_idx (ascending kept prefix positions,
 * length returned in *kept on the host after a synchronise) and optionally
 * out_scores [n]. */
int ckv_select_scores(const ckv_params* p, int32_t n, const float* a, const float* b,
                      const float* c, void* workspace, size_t workspace_bytes, int32_t* out_idx,
                      float* out_scores, ckv_stream_t stream);

/* ckv_select_scores without a workspace argument.  No counterpart in the
 * reference: it is for callers that cannot allocate device memory for us -- a
 * serving engine that reserved almost all HBM for its KV-cache pool at start-up
 * (a per-call cudaMalloc would fail or fragment the pool, and cudaMalloc
 * synchronises the device), or a C / FFI caller with no device allocator.  The
 * scratch is a static __device__ array inside the library sized for n <= 32768
 * (about 0.9 MiB held on every GPU that loads the library until exit); larger n
 * is rejected with CKV_ERR_ARG.  Each call looks up the array's device address on
 * the current device; the first call on a device may load the library's module,
 * so make it before any stream capture.  All calls share the array (each call
 * clears its header first): calls that overlap on the GPU race, so order them on
 * one stream.  Device-side failures are read with ckv_read_status(NULL, ...).
 * Modes: dis (with or without the bridge vector c), max, union and union_da give
 * the same results as ckv_select_scores; combination_mode weighted and per-head
 * eviction return CKV_ERR_UNSUPPORTED.  Calls no cudaMalloc / cudaFree. */
int ckv_select_scores_noalloc(const ckv_params* p, int32_t n, const float* a, const float* b,
                              const float* c, int32_t* out_idx, float* out_scores,
                              ckv_stream_t stream);

/* The absorption solve alone (PU:2060-2206, or PU:1939-2058 when rows_hi is
 * NULL and single_chain != 0): pooled window rows [W, n] fp32 in, finished
 * [n] scores out (sinks = 1% of the total, divided by the max). */
int ckv_neumann_rows(const ckv_params* p, int32_t n, const float* rows_qi, const float* rows_hi,
                     int32_t single_chain, void* workspace, size_t workspace_bytes,
                     float* out_qi, float* out_hi, int32_t* out_steps, ckv_stream_t stream);

/* Window attention statistics and pooling alone (PU:2874-2999): per-head
 * entropy and transient mass [H] (fp32), the chosen head sets as bit masks
 * (bit h set), and the pooled rows [W, n] fp32 (rows_hi untouched when HI
 * reuses the QI matrix). */
int ckv_window_pool(const ckv_params* p, const ckv_layer* layer, void* workspace,
                    size_t workspace_bytes, float* out_entropy, float* out_mass,
                    uint64_t* out_qi_heads, uint64_t* out_hi_heads, float* rows_qi, float* rows_hi,
                    ckv_stream_t stream);

/* ---- head-sharded (tensor-parallel) scoring -------------------------------------
 * No counterpart in the reference, which scores all heads of a layer in one process
 * (the entropy ranking and the QI / HI pooling run across heads, PU:2905-2999).  With the
 * KV heads split over ranks, each rank:
 *   1. computes its heads' exact entropy / transient mass (ckv_window_pool);
 *   2. all-gathers them and derives the layer's head sets with ckv_choose_heads (the same
 *      sets on every rank);
 *   3. pools its heads with those sets (ckv_pool_rows_given): QI rows = max over its QI
 *      heads, HI rows = SUM over its HI heads;
 *   4. all-reduces the rows (max for QI, sum for HI) and scales HI by 1 / (HI head count);
 *   5. scores and selects from the combined rows (ckv_neumann_rows, ckv_select_scores;
 *      combination modes dis / union) and gathers its heads' K / V (ckv_gather).
 * The host side is submission_folder_b200.tp.  Layers with at most 32 query heads. */

/* Head sets of a layer from its per-head exact entropy / mass (device arrays [num_heads]):
 * out_sets[0] = QI heads, out_sets[1] = HI heads (bit h), out_mode[0] = HI mode (0 mean,
 * 1 max, 2 the HI chain reuses the QI rows), out_mode[1] = number of HI heads (device
 * memory; PU:2905-2999 with the tie rules of the single-process path). */
int ckv_choose_heads(const ckv_params* p, int32_t num_heads, const float* entropy, const float* mass,
                     uint64_t* out_sets, int32_t* out_mode, ckv_stream_t stream);

/* This rank's pooled window rows [W, n] fp32 for given head sets (device arrays from
 * ckv_choose_heads): layer holds the rank's heads, which are heads head_offset ..
 * head_offset + num_heads - 1 of the layer.  rows_qi = max over the rank's QI heads (0
 * where it has none), rows_hi = sum over its HI heads (untouched when the HI chain reuses
 * the QI rows).  Workspace as ckv_workspace_size for the local layer. */
int ckv_pool_rows_given(const ckv_params* p, const ckv_layer* layer, int32_t head_offset, const uint64_t* sets,
                        const int32_t* mode, void* workspace, size_t workspace_bytes, float* rows_qi,
                        float* rows_hi, ckv_stream_t stream);

/* ---- influence walker (legacy use_neumann=False path) ------------------------
 * Replaces CircuitGraph.update_and_step_influence_walker + get_influence_scores /
 * get_influence_raw_visits (CircuitKV/csrc/pybind.cpp:263-300; circuit_manager.cpp:
 * 1190-1311; influence_walker.cu:66-456).  Walkers step along full_attn rows; visits
 * are counted per landing position, divided by sqrt(n - p + 1), normalised by their
 * maximum (over the first min(n, 65536) positions, as the reference) and the sinks set
 * to 1.  rng_mode CKV_RNG_PCG: PCG-XSH-RR, walker w seeded (seed, w) as the reference's
 * init_rng_kernel (circuit_walker.cu:157-171; CircuitGraph passes its constructor
 * seed + 3000); CKV_RNG_PHILOX: Philox4x64-10,
 * key (seed, 0), counter (draw / 4, walker, call, 0).  rng_state: device uint64
 * [2 * num_walkers] (PCG states; for Philox [0] counts the calls) kept by the caller
 * across calls as the reference keeps its states, or NULL to seed on every call;
 * init_state = 1 seeds it first.  Argument checks follow the reference
 * (circuit_manager.cpp:1200-1226). */
enum ckv_rng_mode { CKV_RNG_PHILOX = 0, CKV_RNG_PCG = 1 };

/* Dense form: attn [n, n] fp32 row-major on the device (the reference's input). */
int ckv_influence_walk_dense(const float* attn, int32_t n, int32_t current_idx, int32_t num_walkers,
                             int32_t max_steps, int32_t sink_size, float temperature, float explore_temp,
                             float explore_ratio, int32_t rng_mode, uint64_t seed, uint64_t* rng_state,
                             int32_t init_state, float* visits, float* scores, ckv_stream_t stream);

/* Structured form for the hook (PU:3244-3263): full_attn defined by pooled window rows
 * rows [W, ld] fp32 (PU:3003-3034), never materialised, so n is not limited by n^2
 * memory.  Also writes h2o [n] = full_attn column sums (PU:3253).  workspace:
 * ckv_walk_workspace_size bytes, 256-byte aligned. */
int ckv_walk_workspace_size(int32_t n, int32_t window, size_t* bytes);
int ckv_influence_walk(const float* rows, int32_t W, int32_t ld, int32_t n, int32_t current_idx,
                       int32_t num_walkers, int32_t max_steps, int32_t sink_size, float temperature,
                       float explore_temp, float explore_ratio, int32_t rng_mode, uint64_t seed,
                       uint64_t* rng_state, int32_t init_state, void* workspace, size_t workspace_bytes,
                       float* visits, float* scores, float* h2o, ckv_stream_t stream);

/* ---- decode-time graph scoring (circuit walker, spectral, combined) -------------
 * Replace the CircuitGraph methods behind CircuitKVMonitor (CircuitKV/csrc/pybind.cpp:
 * 65-130, circuit_manager.cpp:433-766; kernels graph_update.cu, circuit_walker.cu,
 * spectral_power.cu).  The caller owns the sparse graph (adj_list int32 and adj_weights
 * fp32, [max_seq_len, top_k], empty rows -1 / 0), the per-walker PCG states
 * ([num_walkers][2] uint64) and the visit counts (int32). */

/* Row current_idx of the graph: the top_k keys (of keys [n, head_dim], dtype fp16, bf16 or
 * fp32, like query [head_dim]) by dot product with the query, in descending order (ties:
 * lower key index first), the dot products as weights; -1 / 0 past n keys
 * (graph_update.cu:174-325).  scratch: [n] floats.  top_k in (0, 64]. */
int ckv_graph_update(const void* query, const void* keys, int32_t dtype, int32_t n, int32_t head_dim,
                     int32_t current_idx, int32_t top_k, float* scratch, int32_t* adj_list, float* adj_weights,
                     ckv_stream_t stream);

/* Absorbing walkers (circuit_walker.cu:69-147): num_walkers walkers start at source, add 1 to
 * visits at every position they reach, step to a neighbour with probability proportional to
 * its weight, and stop at the sink tokens [0, 4), a dead end or 1500 steps.  clear_visits = 1
 * zeroes visits [n] first.  rng_state is advanced in place. */
int ckv_circuit_walk(const int32_t* adj_list, const float* adj_weights, int32_t n, int32_t top_k, int32_t source,
                     int32_t num_walkers, uint64_t* rng_state, int32_t* visits, int32_t clear_visits,
                     ckv_stream_t stream);

/* PCG states of num_walkers walkers seeded (seed, walker) (circuit_walker.cu:157-171). */
int ckv_pcg_seed(uint64_t seed, int32_t num_walkers, uint64_t* rng_state, ckv_stream_t stream);

/* Spectral scores (spectral_power.cu:379-404): iters power iterations v <- A v / ||A v||_2 from
 * v = 1 / sqrt(n) over the graph's first n rows.  v, scratch: [n]. */
int ckv_spectral_scores(const int32_t* adj_list, const float* adj_weights, int32_t n, int32_t top_k, int32_t iters,
                        float* v, float* scratch, ckv_stream_t stream);

/* Combined scores (circuit_manager.cpp:700-730): walker_scores = visits as floats; spectral and
 * walker_scores each divided by their maximum (in place, when it is above 1e-8); combined =
 * their element-wise maximum.  All [n]. */
int ckv_combine_scores(const int32_t* visits, float* spectral, float* walker_scores, float* combined, int32_t n,
                       ckv_stream_t stream);

/* Landmark walkers (CircuitGraph.update_and_step_landmark_walker and
 * update_and_step_landmark_absorbing_walker, CircuitKV/csrc/circuit_manager.cpp:768-1164;
 * kernels landmark_walker.cu, landmark_absorbing_walker.cu) over a dense fp32 attention
 * matrix attn [n, n] (row-major):
 *   1. H2O scores: column sums of attn over the rows at or below the diagonal;
 *   2. landmarks: [24, n - 64) cut into num_landmarks equal segments (fewer when a segment
 *      would be shorter than min_spacing > 0), the highest H2O score of each; written to
 *      positions [32] and their number to count [1] (0 when n < 89);
 *   3. walkers_per_source walkers from each landmark and from the query (the last token,
 *      whose attention row is attn[current_idx]); visits [n] (int32) is cleared first, then
 *      gets 1 per landmark-walker visit and (int)query_boost per query-walker visit; walkers
 *      stop at [0, 4) or after 1500 steps (CKV_LANDMARK_ABSORBING with absorb_at_landmarks:
 *      also with probability 0.1 at another source's landmark);
 *   4. scores [n]: CKV_LANDMARK_POSITIONAL visits / (1 / (p - 3)^position_alpha + 1e-8),
 *      CKV_LANDMARK_REACHABILITY visits / (walkers able to reach p), CKV_LANDMARK_ABSORBING
 *      the same with 0.9 pass-through per landmark; 0 on [0, 4).
 * rng_state: [(num_landmarks + 1) * walkers_per_source][2] PCG states (ckv_pcg_seed), walker
 * w = source * walkers_per_source + k, advanced in place.  num_landmarks in [1, 32].
 * workspace: ckv_landmark_workspace_size(n) bytes, 16-byte aligned.  No host
 * synchronisation: the landmark count stays on the device. */
enum { CKV_LANDMARK_POSITIONAL = 0, CKV_LANDMARK_REACHABILITY = 1, CKV_LANDMARK_ABSORBING = 2 };
int ckv_landmark_workspace_size(int32_t n, size_t* bytes);
int ckv_landmark_walk(const float* attn, int32_t n, int32_t current_idx, int32_t mode, int32_t num_landmarks,
                      int32_t walkers_per_source, float query_boost, int32_t min_spacing, float position_alpha,
                      int32_t absorb_at_landmarks, uint64_t* rng_state, int32_t* visits, float* scores,
                      int32_t* positions, int32_t* count, void* workspace, size_t workspace_bytes,
                      ckv_stream_t stream);

/* Raw generator output (no reference counterpart; tests and callers that reproduce a
 * walk): CKV_RNG_PHILOX: out[i] = Philox4x64-10(key (seed, 0), counter (i / 4, stream_id,
 * 0, 0))[i % 4]; CKV_RNG_PCG: out[i] = the i-th pcg32 output of the state seeded
 * (seed, stream_id), i.e. pcg32_srandom_r(seed, stream_id). */
int ckv_rng_fill(int32_t mode, uint64_t seed, uint64_t stream_id, int32_t count, uint64_t* out,
                 ckv_stream_t stream);

/* Whether the current device can read `ptr` in place (no reference counterpart): device
 * memory of the current device, managed memory, or page-locked host memory mapped at the
 * same address.  The hook uses it to let the final gather read V rows straight from a
 * caller's pinned host tensor instead of copying all of V to the device first.  Sets
 * *accessible to 0 for pageable host memory and unknown pointers. */
int ckv_device_accessible(const void* ptr, int32_t* accessible);

/* `rows` rows of row_bytes each, from src (rows src_pitch bytes apart) to dst (dst_pitch bytes
 * apart), either direction, as one asynchronous DMA on the stream (no reference counterpart:
 * the hook moves the window queries of all heads, 32 strided row blocks of a host tensor, in
 * one copy instead of one per head). */
int ckv_copy_rows(void* dst, size_t dst_pitch, const void* src, size_t src_pitch, size_t row_bytes, int32_t rows,
                  ckv_stream_t stream);

/* K / V compaction alone (PU:3496-3517 shared, PU:3448-3462 per head): the `kept`
 * positions idx ([kept] or [H, kept] with per_head) then the last `window` rows, into
 * [H, kept + window, D] outputs.  For callers that chose the positions themselves (the
 * influence-walker path). */
int ckv_gather(const ckv_layer* layer, int32_t window, const int32_t* idx, int32_t kept, int32_t per_head,
               void* out_k, void* out_v, ckv_stream_t stream);

/* Per-stage timing (no counterpart in the reference; for benchmarks): while
 * set, each ckv_score_evict call on this thread records events[0] before its
 * first kernel and events[i] after its i-th stage (window moments, pooling,
 * pooling re-run, sweep maps, sweep terms, aux, selection, gather: 9 events).
 * Records are graph-capturable (external event records).  The array must stay
 * valid while set; count 0 clears it. */
int ckv_set_stage_events(void* const* events, int32_t count);

/* Human-readable description of the calling thread's last error. */
const char* ckv_last_error_string(void);

/* Library version string ("circuitkv-b200 <semver>"). */
const char* ckv_version(void);

#ifdef __cplusplus
}
#endif

#endif /* CKV_H_ */
