// C ABI of the CircuitKV prefill scoring + eviction path (include/ckv.h):
// parameter checks, the per-layer plan and workspace carve-up, and the launch
// sequence that replaces CircuitKVCluster.update_kv
// (KVCache-Factory/pyramidkv/pyramidkv_utils.py:2775-3519).
#include <cuda_runtime.h>
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <mutex>
#include <string>
#include <vector>

#include "ckv_common.cuh"
#include "ckv_gather.h"
#include "ckv_monitor.h"
#include "ckv_neumann.h"
#include "ckv_plan.h"
#include "ckv_select.h"
#include "ckv_walker.h"
#include "ckv_window.h"

namespace ckv {

static thread_local std::string g_last_error = "no error";

// Optional per-stage timing: events recorded (as graph-capturable external
// records) before the first and after every kernel of a layer call.
static thread_local cudaEvent_t* g_stage_events = nullptr;
static thread_local int g_stage_count = 0;
static thread_local int g_stage_next = 0;

void stage_mark(cudaStream_t st) {
  if (g_stage_events && g_stage_next < g_stage_count)
    cudaEventRecordWithFlags(g_stage_events[g_stage_next++], st, cudaEventRecordExternal);
}

static int fail(int code, const char* msg) {
  g_last_error = msg;
  return code;
}

static int cuda_fail(cudaError_t e, const char* where) {
  g_last_error = std::string(where) + ": " + cudaGetErrorString(e);
  return CKV_ERR_CUDA;
}

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

int make_plan(const ckv_params& p, int n, int H, int Hkv, int D, int dtype, Plan* out,
              const char** why) {
  Plan pl;
  memset(&pl, 0, sizeof(pl));
  if (dtype != CKV_BF16 && dtype != CKV_FP16 && dtype != CKV_FP32) { *why = "dtype must be bf16, fp16 or fp32"; return CKV_ERR_DTYPE; }
  if (n <= 0 || H <= 0 || Hkv <= 0 || H % Hkv != 0) { *why = "need n > 0 and num_heads divisible by num_kv_heads"; return CKV_ERR_ARG; }
  if (H > kMaxHeads) { *why = "at most 64 query heads"; return CKV_ERR_UNSUPPORTED; }
  if (D != kHeadDim) { *why = "head_dim must be 128"; return CKV_ERR_UNSUPPORTED; }
  if (p.window_size <= 0 || p.sink_size < 0) { *why = "window_size must be > 0 and sink_size >= 0"; return CKV_ERR_ARG; }
  if (p.neumann_iterations < 1 || p.neumann_iterations > kMaxIters) { *why = "neumann_iterations must be in [1, 16]"; return CKV_ERR_UNSUPPORTED; }
  pl.n = n; pl.H = H; pl.Hkv = Hkv; pl.G = H / Hkv; pl.D = D; pl.dtype = dtype;
  pl.W = p.window_size; pl.s = p.sink_size; pl.K = p.neumann_iterations;
  pl.mode = p.combination_mode;
  pl.per_head = p.per_head_eviction;
  if (pl.mode < 0 || pl.mode > CKV_COMB_UNION_DA) { *why = "unknown combination_mode"; return CKV_ERR_ARG; }
  if (n < p.max_capacity_prompt) {
    // the reference returns its inputs unchanged (PU:2864)
    pl.out_len = n;
    pl.total = align256(sizeof(Header));
    *out = pl;
    return CKV_OK;
  }
  if (pl.W > kMaxWindow) { *why = "window_size must be <= 128"; return CKV_ERR_UNSUPPORTED; }
  if (pl.per_head && n - pl.W > 65536) {
    *why = "per_head_eviction supports n - window_size <= 65536"; return CKV_ERR_UNSUPPORTED;
  }
  pl.rows_per_warp = (dtype == CKV_FP32) ? 16 : 32;
  pl.rows_per_batch = kWarps * pl.rows_per_warp;
  if (pl.W % pl.rows_per_warp != 0 || pl.rows_per_batch % pl.W != 0) {
    *why = "window_size must be 32, 64 or 128 (16-bit) / 16, 32, 64 or 128 (fp32)";
    return CKV_ERR_UNSUPPORTED;
  }
  if (pl.W > pl.rows_per_batch) { *why = "window_size too large for this dtype"; return CKV_ERR_UNSUPPORTED; }
  pl.heads_per_batch = pl.rows_per_batch / pl.W;
  if (pl.heads_per_batch > H) pl.heads_per_batch = H;
  if (H % pl.heads_per_batch != 0) { *why = "num_heads must be a multiple of the heads per window batch"; return CKV_ERR_UNSUPPORTED; }
  // a batch smaller than rows_per_batch would leave warps idle: require full batches
  if (pl.heads_per_batch * pl.W != pl.rows_per_batch) { *why = "num_heads * window_size too small"; return CKV_ERR_UNSUPPORTED; }
  pl.nbatch = H / pl.heads_per_batch;
  int ktiles = 0;
  for (int b = 0; b < pl.nbatch; ++b) {
    const int h0 = b * pl.heads_per_batch;
    const int ng = (h0 + pl.heads_per_batch - 1) / pl.G - h0 / pl.G + 1;
    ktiles = ng > ktiles ? ng : ktiles;
  }
  pl.ktiles_per_batch = ktiles;
  pl.n_p = n - pl.W;
  if (pl.n_p < pl.s) { *why = "sequence shorter than sink_size + window_size"; return CKV_ERR_UNSUPPORTED; }
  // keep-set sizes (PU:2616-2644)
  const int target = p.max_capacity_prompt > pl.s + pl.W ? p.max_capacity_prompt : pl.s + pl.W;
  const int forced = pl.s + pl.W;                 // n - W >= s
  const int cand = n - forced;
  int remaining = target - forced;
  if (remaining < 0) remaining = 0;
  pl.kk = remaining < cand ? remaining : cand;
  pl.out_len = pl.s + pl.kk + pl.W;
  if (pl.kk + pl.s + pl.W > 8192) { *why = "budget above 8192 tokens is not supported"; return CKV_ERR_UNSUPPORTED; }
  if (pl.mode == CKV_COMB_UNION || pl.mode == CKV_COMB_UNION_DA) {
    if (2 * pl.kk > 8192) { *why = "union budget above 4096 tokens is not supported"; return CKV_ERR_UNSUPPORTED; }
  }
  pl.nchains = (pl.mode == CKV_COMB_MAX || pl.mode == CKV_COMB_WEIGHTED) ? 1 : 2;
  pl.tc = (dtype != CKV_FP32 && (pl.G * pl.W) % 128 == 0 && pl.G * pl.W <= 512 && pl.W <= 128) ? 1 : 0;
  // tensor-core pooling pass: 4 query heads per KV group, window 64 (the Llama / Mistral shapes)
  // tensor-core pooling: 4 query heads per KV group, W = 64, and at least two KV groups
  // (its per-tile handshake relies on a tile spanning two or more steps)
  pl.tc_pool = (pl.tc && pl.G == 4 && pl.W == 64 && pl.Hkv >= 2) ? 1 : 0;
  // W = 32 / 128: the keys-on-lanes form alone (its exact branch is the SIMT pass)
  pl.lanes_pool = (pl.tc && pl.G == 4 && (pl.W == 32 || pl.W == 128) && pl.Hkv >= 2) ? 1 : 0;
  pl.pool_blocks = pl.W > 64 ? pl.W / 16 : 4;
  pl.hi_rows = (pl.nchains == 2 && p.entropy_aware) ? 1 : 0;
  pl.ncol_tiles = (n + kColTile - 1) / kColTile;
  pl.n_pad = pl.ncol_tiles * kColTile;
  // moments pass: one wave of CTAs (tensor-core path: one CTA per SM per KV group)
  // tensor-core moments: one CTA per (column chunk, KV group, 128-row m-tile), one wave
  // (SIMT: two CTAs per SM for 16-bit rows; one for fp32, whose staged rows fill most of
  // the shared memory, so one wave of 148 CTAs with longer column chunks)
  int chunks = pl.tc ? 148 / (Hkv * ((pl.G * pl.W) / 128))
                     : ((dtype == CKV_FP32 ? 148 : 296) + pl.nbatch - 1) / pl.nbatch;
  if (chunks > pl.ncol_tiles) chunks = pl.ncol_tiles;
  if (chunks < 1) chunks = 1;
  pl.tiles_per_chunk = (pl.ncol_tiles + chunks - 1) / chunks;
  pl.nstat_chunks = (pl.ncol_tiles + pl.tiles_per_chunk - 1) / pl.tiles_per_chunk;
  pl.nscan = (pl.n_p + kScanChunk - 1) / kScanChunk;
  if (pl.nscan < 1) pl.nscan = 1;
  pl.tc_nclusters = pl.ncol_tiles < 148 ? pl.ncol_tiles : 148;   // CTAs of the tensor-core pooling pass
  pl.e_parts = pl.tc_pool ? pl.tc_nclusters : pl.ncol_tiles;   // TC: one partial per CTA
  pl.rs_parts = (pl.tc_pool || pl.lanes_pool) ? 2 * pl.ncol_tiles : pl.ncol_tiles;
  pl.g_slice = kColTile;
  if (window_smem_bytes(pl, true) > 227 * 1024 || window_smem_bytes(pl, false) > 227 * 1024) {
    *why = "window tile does not fit in shared memory"; return CKV_ERR_UNSUPPORTED;
  }
  // workspace carve-up
  size_t off = align256(sizeof(Header));
  auto take = [&](size_t bytes) { const size_t o = off; off = align256(off + bytes); return o; };
  const size_t HW = (size_t)H * pl.W;
  pl.off_stats = take(((size_t)pl.nstat_chunks * HW * 16 > (2 * HW + 2 * (size_t)pl.W) * 4)
                         ? (size_t)pl.nstat_chunks * HW * 16 : (2 * HW + 2 * (size_t)pl.W) * 4);
  pl.off_lse = take(HW * 4);
  pl.off_spec = take((size_t)5 * H * 4);   // [H] ent, [H] mass (speculated), [H] ent, [H] mass (final), [H] bound
  pl.off_minx = take((size_t)pl.nstat_chunks * HW * 4);
  pl.off_epart = take((size_t)pl.e_parts * HW * 4);
  pl.off_mpart = take((size_t)pl.e_parts * HW * 4);
  pl.off_rows_qi = take((size_t)pl.W * pl.n_pad * 4);
  pl.off_rows_hi = take((size_t)pl.W * pl.n_pad * 4);
  pl.off_colsum = take((size_t)2 * pl.n_pad * 4);
  pl.off_gtile = take((size_t)2 * pl.ncol_tiles * 8 * 4);
  pl.off_rspart = take((size_t)2 * pl.ncol_tiles * 8 * pl.W * 4);
  pl.off_colpart = take((pl.tc_pool || pl.lanes_pool) ? (size_t)2 * pl.pool_blocks * pl.n_pad * 4 : 0);
  pl.off_wk = take((size_t)2 * pl.K * pl.W * 4);
  pl.off_yk = take((size_t)2 * (pl.K + 1) * pl.W * 4);
  pl.off_ymax = take((size_t)2 * (pl.K + 1) * 4);
  pl.off_bk = take((size_t)2 * pl.K * pl.n_p * 4 + 4);
  pl.off_cg = take((size_t)2 * pl.n_p * 8 + 8);
  pl.off_agg = take((size_t)2 * pl.nscan * 2 * kMaxIters * 4);
  pl.off_sin = take((size_t)2 * pl.nscan * kMaxIters * 4);   // incoming carry of each chunk
  pl.off_cum = take((size_t)2 * (pl.K + 1) * pl.n_p * 4 + 4);
  pl.off_cmax = take((size_t)2 * pl.nscan * (kMaxIters + 1) * 4);
  pl.sel_bytes = (size_t)6 * n * 4 + (size_t)n * 4 + (size_t)n;
  if (pl.mode == CKV_COMB_WEIGHTED)   // full-rank radix buffers [2][2][n] u64 and ranks [2][n]
    pl.sel_bytes = (((size_t)29 * n + 15) & ~(size_t)15) + (size_t)40 * n;
  pl.off_sel = take(pl.sel_bytes);
  pl.off_ph = off;
  if (pl.per_head) {
    const size_t nw = (size_t)(n - pl.W), Hs = (size_t)H, nn = (size_t)n;
    pl.ph_nw = n - pl.W;
    pl.off_ph_q2w = take(Hs * pl.W * 4);
    pl.off_ph_qrow = take(Hs * nn * 4);
    pl.off_ph_two = take(Hs * nn * 4);
    pl.off_ph_col = take(Hs * nn * 4);
    // tcgen05 per-head pass: the pooling pass's keys-on-lanes shapes, and its shared memory
    // (two stages, log-sum-exp and q2w re-laid) within the 227 KB a CTA may have
    const int rs = pl.W < 64 ? pl.W : 64;
    const size_t ph_smem = 2 * ((size_t)pl.G * rs * 256 + 128 * 256) + 2 * Hs * pl.W * 4 + 1024;
    pl.ph_tc = (pl.tc && pl.G == 4 && (pl.W == 32 || pl.W == 64 || pl.W == 128) && pl.Hkv >= 2 &&
                ph_smem + 1024 <= 227 * 1024) ? 1 : 0;
    pl.ph_slots = pl.ph_tc ? 4 * (pl.W / rs) : 0;
    pl.ph_ent_parts = pl.ph_tc ? 4 * ((n + 127) / 128) : pl.ncol_tiles;
    pl.off_ph_ent = take((size_t)(pl.ph_ent_parts + 1) * Hs * 4);   // + the per-head totals
    pl.off_ph_part = take((size_t)2 * pl.ph_slots * Hs * nn * 4);
    pl.off_ph_vec = take(Hs * 2 * nw * 4);
    pl.off_ph_ghi = take(nw * 4);
    pl.off_ph_gbuf = take(nw * 2 * 8 + nw * 4);
    pl.off_ph_bufs = take(Hs * 4 * nw * 8);
    pl.off_ph_ranks = take(Hs * 2 * nw * 4);
    pl.off_ph_bits = take(Hs * ((nw + 31) / 32) * 4);
  }
  pl.total = off;
  *out = pl;
  return CKV_OK;
}

static int check_layer(const ckv_layer* L) {
  if (!L || !L->q || !L->k || !L->v) return fail(CKV_ERR_ARG, "null layer or tensor pointer");
  const size_t es = L->dtype == CKV_FP32 ? 4 : 2;
  auto al = [&](const void* p, int64_t hs, int64_t ts) {
    return ((uintptr_t)p % 16 == 0) && ((hs * (int64_t)es) % 16 == 0) && ((ts * (int64_t)es) % 16 == 0);
  };
  if (!al(L->q, L->q_head_stride, L->q_tok_stride) || !al(L->k, L->k_head_stride, L->k_tok_stride) ||
      !al(L->v, L->v_head_stride, L->v_tok_stride))
    return fail(CKV_ERR_ARG, "tensor pointers and strides must be 16-byte aligned (contiguous head_dim rows)");
  return CKV_OK;
}

static int check_ws(const Plan& pl, void* ws, size_t bytes) {
  if (!ws || (uintptr_t)ws % 256 != 0) return fail(CKV_ERR_WORKSPACE, "workspace must be 256-byte aligned and non-null");
  if (bytes < pl.total) return fail(CKV_ERR_WORKSPACE, "workspace too small (see ckv_workspace_size)");
  return CKV_OK;
}

static int launch_gather_layer(const Plan& pl, const ckv_layer* L, const ckv_outputs* out,
                               const int32_t* idx, int identity, cudaStream_t st) {
  GatherArgs g;
  g.k = L->k; g.khs = L->k_head_stride; g.kts = L->k_tok_stride;
  g.v = L->v; g.vhs = L->v_head_stride; g.vts = L->v_tok_stride;
  g.out_k = out->out_k; g.out_v = out->out_v; g.idx = idx;
  g.n = pl.n; g.W = identity ? 0 : pl.W; g.H = pl.H; g.Hkv = pl.Hkv; g.G = pl.G; g.D = pl.D;
  g.out_len = pl.out_len; g.per_head = pl.per_head; g.identity = identity;
  g.distinct = out->distinct_kv_heads ? 1 : 0;
  const cudaError_t e = launch_gather(g, pl.dtype, st);
  return e == cudaSuccess ? CKV_OK : cuda_fail(e, "gather launch");
}

static int score_evict_one(const ckv_params* p, const ckv_layer* L, void* workspace,
                           size_t ws_bytes, const ckv_outputs* out, cudaStream_t st, bool marks = true) {
  if (!p || !out || !out->out_k || !out->out_v) return fail(CKV_ERR_ARG, "null params or outputs");
  if (out->distinct_kv_heads && p->per_head_eviction)
    return fail(CKV_ERR_UNSUPPORTED, "distinct_kv_heads outputs are for shared eviction");
  int rc = check_layer(L);
  if (rc) return rc;
  Plan pl;
  const char* why = "";
  rc = make_plan(*p, L->n, L->num_heads, L->num_kv_heads, L->head_dim, L->dtype, &pl, &why);
  if (rc) return fail(rc, why);
  if (L->n < p->max_capacity_prompt) return launch_gather_layer(pl, L, out, nullptr, 1, st);
  if (!out->out_idx) return fail(CKV_ERR_ARG, "out_idx is required");
  rc = check_ws(pl, workspace, ws_bytes);
  if (rc) return rc;
  char* ws = static_cast<char*>(workspace);
  cudaError_t e = cudaMemsetAsync(ws, 0, sizeof(Header), st);
  if (e != cudaSuccess) return cuda_fail(e, "workspace header reset");
  g_stage_next = marks ? 0 : g_stage_count;   // stage events only for single-layer calls
  stage_mark(st);
  WinArgs wa;
  wa.q = L->q; wa.qhs = L->q_head_stride; wa.qts = L->q_tok_stride;
  wa.k = L->k; wa.khs = L->k_head_stride; wa.kts = L->k_tok_stride;
  wa.ws = ws; wa.fixup_pass = 0; wa.p = *p; wa.pl = pl;
  wa.tc_min = 0; wa.force_exact = 0;
  if (pl.per_head) {   // PU:3296-3464: per-head importance and selection, per-head gather
    e = launch_window_stage(wa, 0, st);
    if (e != cudaSuccess) return cuda_fail(e, "window moments");
    stage_mark(st);
    e = launch_ph_pass(wa, st);
    if (e != cudaSuccess) return cuda_fail(e, "per-head pass");
    // stage marks as the shared path's: the per-head pass stands where the pooling pass
    // does; reduction, re-run, sweep and aux take no time here
    for (int i = 0; i < 6; ++i) stage_mark(st);
    PhArgs ph;
    ph.pl = pl; ph.p = *p; ph.ws = ws; ph.out_idx = out->out_idx;
    ph.eq = (float)pow((double)p->qi_gamma, pl.K / 2.0);
    ph.eh = (float)pow((double)p->hi_gamma, pl.K / 2.0);
    e = launch_ph_select(ph, st);
    if (e != cudaSuccess) return cuda_fail(e, "per-head selection");
    stage_mark(st);
    if (out->out_scores) {   // [H][2][n - W] ranked vectors, then [H] entropies
      const size_t nv = (size_t)pl.H * 2 * pl.ph_nw;
      e = cudaMemcpyAsync(out->out_scores, ws + pl.off_ph_vec, nv * 4, cudaMemcpyDeviceToDevice, st);
      if (e == cudaSuccess)
        e = cudaMemcpyAsync(out->out_scores + nv, ws + pl.off_ph_ent + (size_t)pl.ph_ent_parts * pl.H * 4,
                            (size_t)pl.H * 4, cudaMemcpyDeviceToDevice, st);
      if (e != cudaSuccess) return cuda_fail(e, "per-head score copy");
    }
    const int rc_g = launch_gather_layer(pl, L, out, out->out_idx, 0, st);
    stage_mark(st);
    return rc_g;
  }
  for (int s = 0; s < 3; ++s) {
    e = launch_window_stage(wa, s, st);
    if (e != cudaSuccess) {
      static const char* names[3] = {"window moments", "window pooling", "window pooling re-run"};
      return cuda_fail(e, names[s]);
    }
    stage_mark(st);
  }
  e = launch_sweep(pl, *p, ws, st);
  if (e != cudaSuccess) return cuda_fail(e, "sweep kernels");
  stage_mark(st);
  if (pl.mode == CKV_COMB_MAX || pl.mode == CKV_COMB_WEIGHTED ||
      (pl.mode == CKV_COMB_DIS && p->use_bridge_importance)) {
    e = launch_aux(pl, *p, ws, st);
    if (e != cudaSuccess) return cuda_fail(e, "aux kernel");
  }
  stage_mark(st);
  SelArgs sa;
  memset(&sa, 0, sizeof(sa));
  sa.pl = pl; sa.p = *p; sa.ws = ws; sa.out_idx = out->out_idx; sa.out_scores = out->out_scores;
  sa.narrow = marks ? 0 : 1;   // concurrent layers: the smaller cluster
  e = launch_select(sa, st);
  if (e != cudaSuccess) return cuda_fail(e, "select kernel");
  stage_mark(st);
  const int rc2 = launch_gather_layer(pl, L, out, out->out_idx, 0, st);
  stage_mark(st);
  return rc2;
}

}  // namespace ckv

using namespace ckv;

extern "C" {

void ckv_default_params(ckv_params* p) {
  if (!p) return;
  memset(p, 0, sizeof(*p));
  p->window_size = 64;
  p->max_capacity_prompt = 2048;
  p->sink_size = 4;
  p->neumann_iterations = 10;
  p->neumann_temperature = 1.0f;
  p->neumann_gamma = 1.0f;
  p->qi_gamma = 1.0f;
  p->hi_gamma = 1.0f;
  p->combination_mode = CKV_COMB_DIS;
  p->h2o_weight = 0.5f;
  p->qi_ratio = 0.5f;
  p->entropy_adaptive = 1;
  p->use_gaussian = 1;
  p->qi_kernel_size = 3;
  p->hi_kernel_size = 5;
  p->gaussian_sigma = 1.0f;
  p->entropy_aware = 1;
  p->top_k_heads = 10;
  p->hi_mass_threshold = 0.5f;
  p->bi_kernel_size = 5;
}

int ckv_output_len(const ckv_params* p, int32_t n, int32_t* out_len) {
  if (!p || !out_len) return fail(CKV_ERR_ARG, "null argument");
  Plan pl;
  const char* why = "";
  const int rc = make_plan(*p, n, 32, 8, 128, CKV_BF16, &pl, &why);
  if (rc) return fail(rc, why);
  *out_len = pl.out_len;
  return CKV_OK;
}

int ckv_workspace_size(const ckv_params* p, int32_t n, int32_t num_heads, int32_t num_kv_heads,
                       int32_t head_dim, size_t* bytes) {
  if (!p || !bytes) return fail(CKV_ERR_ARG, "null argument");
  size_t best = 0;
  for (int dt = 0; dt < 3; ++dt) {   // large enough for any dtype
    Plan pl;
    const char* why = "";
    const int rc = make_plan(*p, n, num_heads, num_kv_heads, head_dim, dt, &pl, &why);
    if (rc == CKV_OK && pl.total > best) best = pl.total;
    if (rc != CKV_OK && dt == 0) return fail(rc, why);
  }
  *bytes = best;
  return CKV_OK;
}

int ckv_score_evict(const ckv_params* p, const ckv_layer* layer, void* workspace,
                    size_t workspace_bytes, const ckv_outputs* out, ckv_stream_t stream) {
  return score_evict_one(p, layer, workspace, workspace_bytes, out, (cudaStream_t)stream);
}

// Side streams of the batched entry point, per device: the layers are independent,
// so their chains run concurrently on kLanes streams forked from and joined back to
// the caller's stream (inside a stream capture this records parallel graph branches).
// One layer's latency-bound steps (selection, reduction tails) then overlap another
// layer's tensor-core passes.
namespace {
constexpr int kLanes = 16;
constexpr int kMaxDevices = 64;
struct Lanes {
  cudaStream_t s[kLanes];
  cudaEvent_t fork;
  cudaEvent_t join[kLanes];
  bool ready;
};
std::mutex g_lanes_mu;
Lanes g_lanes[kMaxDevices];

cudaError_t lanes_for_device(Lanes** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  Lanes& L = g_lanes[dev];
  if (!L.ready) {
    for (int i = 0; i < kLanes && e == cudaSuccess; ++i) e = cudaStreamCreateWithFlags(&L.s[i], cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&L.fork, cudaEventDisableTiming);
    for (int i = 0; i < kLanes && e == cudaSuccess; ++i) e = cudaEventCreateWithFlags(&L.join[i], cudaEventDisableTiming);
    if (e != cudaSuccess) return e;
    L.ready = true;
  }
  *out = &L;
  return cudaSuccess;
}
}  // namespace

int ckv_score_evict_batched(const ckv_params* params, int32_t params_count, const ckv_layer* layers,
                            int32_t count, void* workspace, size_t workspace_bytes,
                            const ckv_outputs* outs, ckv_stream_t stream) {
  if (!params || !layers || !outs || count < 0) return fail(CKV_ERR_ARG, "null argument");
  if (params_count != 1 && params_count != count)
    return fail(CKV_ERR_ARG, "params_count must be 1 or count");
  auto par = [&](int i) { return params + (params_count == 1 ? 0 : i); };
  char* base = static_cast<char*>(workspace);
  cudaStream_t st = (cudaStream_t)stream;
  // validate every layer before anything is enqueued
  std::vector<size_t> offs((size_t)count + 1, 0);
  for (int i = 0; i < count; ++i) {
    size_t need = 0;
    int rc = ckv_workspace_size(par(i), layers[i].n, layers[i].num_heads, layers[i].num_kv_heads,
                                layers[i].head_dim, &need);
    if (rc) return rc;
    rc = check_layer(&layers[i]);
    if (rc) return rc;
    if (!outs[i].out_k || !outs[i].out_v || (layers[i].n >= par(i)->max_capacity_prompt && !outs[i].out_idx))
      return fail(CKV_ERR_ARG, "null output pointer");
    if (outs[i].distinct_kv_heads && par(i)->per_head_eviction)
      return fail(CKV_ERR_UNSUPPORTED, "distinct_kv_heads outputs are for shared eviction");
    offs[i + 1] = offs[i] + align256(need);
    if (offs[i + 1] > workspace_bytes) return fail(CKV_ERR_WORKSPACE, "batched workspace too small");
  }
  if (count == 0) return CKV_OK;
  Lanes* lanes = nullptr;
  if (count == 1 || lanes_for_device(&lanes) != cudaSuccess) {
    cudaGetLastError();
    for (int i = 0; i < count; ++i) {
      const int rc = score_evict_one(par(i), &layers[i], base + offs[i], offs[i + 1] - offs[i], &outs[i], st);
      if (rc) return rc;
    }
    return CKV_OK;
  }
  std::lock_guard<std::mutex> lock(g_lanes_mu);
  const int nl = count < kLanes ? count : kLanes;
  cudaError_t e = cudaEventRecord(lanes->fork, st);
  for (int l = 0; l < nl && e == cudaSuccess; ++l) e = cudaStreamWaitEvent(lanes->s[l], lanes->fork, 0);
  if (e != cudaSuccess) return cuda_fail(e, "batched fork");
  int rc = CKV_OK;
  for (int i = 0; i < count && rc == CKV_OK; ++i)
    rc = score_evict_one(par(i), &layers[i], base + offs[i], offs[i + 1] - offs[i], &outs[i], lanes->s[i % nl], false);
  // join every lane back, also after a failure, so a stream capture stays well formed
  for (int l = 0; l < nl; ++l) {
    cudaError_t ej = cudaEventRecord(lanes->join[l], lanes->s[l]);
    if (ej == cudaSuccess) ej = cudaStreamWaitEvent(st, lanes->join[l], 0);
    if (ej != cudaSuccess && rc == CKV_OK) rc = cuda_fail(ej, "batched join");
  }
  return rc;
}

int ckv_read_status(void* workspace, ckv_stream_t stream, int32_t* device_status) {
  if (!device_status) return fail(CKV_ERR_ARG, "null argument");
  if (!workspace) {   // the static scratch of ckv_select_scores_noalloc on this device
    const cudaError_t e = noalloc_scratch(&workspace);
    if (e != cudaSuccess) return cuda_fail(e, "static scratch address");
  }
  Header h;
  cudaError_t e = cudaMemcpyAsync(&h, workspace, sizeof(Header), cudaMemcpyDeviceToHost, (cudaStream_t)stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "read status");
  *device_status = h.status;
  const int32_t zero = 0;
  e = cudaMemcpyAsync(workspace, &zero, sizeof(zero), cudaMemcpyHostToDevice, (cudaStream_t)stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "clear status");
  return CKV_OK;
}

int ckv_select_scores(const ckv_params* p, int32_t n, const float* a, const float* b,
                      const float* c, void* workspace, size_t workspace_bytes, int32_t* out_idx,
                      float* out_scores, ckv_stream_t stream) {
  if (!p || !a || !b || !out_idx) return fail(CKV_ERR_ARG, "null argument");
  if (p->per_head_eviction)
    return fail(CKV_ERR_UNSUPPORTED, "per-head selection needs the window attention: use ckv_score_evict");
  Plan pl;
  const char* why = "";
  int rc = make_plan(*p, n, 32, 8, 128, CKV_BF16, &pl, &why);
  if (rc) return fail(rc, why);
  if (n < p->max_capacity_prompt) return fail(CKV_ERR_ARG, "n < max_capacity_prompt: nothing to select");
  rc = check_ws(pl, workspace, workspace_bytes);
  if (rc) return rc;
  char* ws = static_cast<char*>(workspace);
  cudaError_t e = cudaMemsetAsync(ws, 0, sizeof(Header), (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "workspace header reset");
  SelArgs sa;
  memset(&sa, 0, sizeof(sa));
  sa.pl = pl; sa.p = *p; sa.ws = ws; sa.out_idx = out_idx; sa.out_scores = out_scores;
  sa.given = 1; sa.ga = a; sa.gb = b; sa.gc = c;
  e = launch_select(sa, (cudaStream_t)stream);
  return e == cudaSuccess ? CKV_OK : cuda_fail(e, "select kernel");
}

int ckv_select_scores_noalloc(const ckv_params* p, int32_t n, const float* a, const float* b,
                              const float* c, int32_t* out_idx, float* out_scores,
                              ckv_stream_t stream) {
  const char* why = "";
  const int rc = select_scores_noalloc(p, n, a, b, c, out_idx, out_scores, (cudaStream_t)stream, &why);
  return rc ? fail(rc, why) : CKV_OK;
}

int ckv_neumann_rows(const ckv_params* p, int32_t n, const float* rows_qi, const float* rows_hi,
                     int32_t single_chain, void* workspace, size_t workspace_bytes, float* out_qi,
                     float* out_hi, int32_t* out_steps, ckv_stream_t stream) {
  if (!p || !rows_qi || !out_qi) return fail(CKV_ERR_ARG, "null argument");
  ckv_params q = *p;
  q.combination_mode = single_chain ? CKV_COMB_MAX : CKV_COMB_DIS;
  q.entropy_aware = (rows_hi != nullptr && !single_chain) ? 1 : 0;
  q.max_capacity_prompt = 0;   // only the solve: any n is scored
  if (q.max_capacity_prompt < q.sink_size + q.window_size) q.max_capacity_prompt = q.sink_size + q.window_size;
  Plan pl;
  const char* why = "";
  int rc = make_plan(q, n, 32, 8, 128, CKV_BF16, &pl, &why);
  if (rc) return fail(rc, why);
  rc = check_ws(pl, workspace, workspace_bytes);
  if (rc) return rc;
  // rows given by the caller: 64-column partial layout of the prep kernel
  pl.tc_pool = 0;
  pl.lanes_pool = 0;
  pl.rs_parts = pl.ncol_tiles;
  pl.g_slice = kColTile;
  pl.e_parts = pl.ncol_tiles;
  char* ws = static_cast<char*>(workspace);
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = cudaMemsetAsync(ws, 0, sizeof(Header), st);
  const int nrows = pl.hi_rows ? 2 : 1;
  for (int r = 0; r < nrows && e == cudaSuccess; ++r) {
    char* dst = ws + (r == 0 ? pl.off_rows_qi : pl.off_rows_hi);
    e = cudaMemsetAsync(dst, 0, (size_t)pl.W * pl.n_pad * 4, st);
    if (e == cudaSuccess)
      e = cudaMemcpy2DAsync(dst, (size_t)pl.n_pad * 4, r == 0 ? rows_qi : rows_hi, (size_t)n * 4,
                            (size_t)n * 4, pl.W, cudaMemcpyDeviceToDevice, st);
  }
  if (e == cudaSuccess) e = launch_rows_prep(pl, q, ws, st);
  if (e == cudaSuccess) e = launch_sweep(pl, q, ws, st);
  if (e != cudaSuccess) return cuda_fail(e, "neumann stage");
  // finished scores of both chains into a [2][n] scratch, then split
  float* fin = reinterpret_cast<float*>(ws + pl.off_sel) + 6 * (size_t)n;   // past the select vectors
  (void)fin;
  SelArgs sa;
  memset(&sa, 0, sizeof(sa));
  sa.pl = pl; sa.p = q; sa.ws = ws; sa.finish_only = 1;
  sa.out_scores = reinterpret_cast<float*>(ws + pl.off_sel) + 3 * (size_t)n;   // [2][n] in the sm area
  e = launch_select(sa, st);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(out_qi, sa.out_scores, (size_t)n * 4, cudaMemcpyDeviceToDevice, st);
  if (e == cudaSuccess && out_hi && pl.nchains > 1)
    e = cudaMemcpyAsync(out_hi, sa.out_scores + n, (size_t)n * 4, cudaMemcpyDeviceToDevice, st);
  if (e == cudaSuccess && out_steps)
    e = cudaMemcpyAsync(out_steps, &reinterpret_cast<Header*>(ws)->steps, 4, cudaMemcpyDeviceToDevice, st);
  return e == cudaSuccess ? CKV_OK : cuda_fail(e, "neumann stage output");
}

int ckv_window_pool(const ckv_params* p, const ckv_layer* layer, void* workspace,
                    size_t workspace_bytes, float* out_entropy, float* out_mass,
                    uint64_t* out_qi_heads, uint64_t* out_hi_heads, float* rows_qi, float* rows_hi,
                    ckv_stream_t stream) {
  if (!p) return fail(CKV_ERR_ARG, "null params");
  int rc = check_layer(layer);
  if (rc) return rc;
  ckv_params q = *p;
  if (q.max_capacity_prompt > layer->n) q.max_capacity_prompt = layer->n;
  Plan pl;
  const char* why = "";
  rc = make_plan(q, layer->n, layer->num_heads, layer->num_kv_heads, layer->head_dim, layer->dtype, &pl, &why);
  if (rc) return fail(rc, why);
  rc = check_ws(pl, workspace, workspace_bytes);
  if (rc) return rc;
  char* ws = static_cast<char*>(workspace);
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = cudaMemsetAsync(ws, 0, sizeof(Header), st);
  WinArgs wa;
  wa.q = layer->q; wa.qhs = layer->q_head_stride; wa.qts = layer->q_tok_stride;
  wa.k = layer->k; wa.khs = layer->k_head_stride; wa.kts = layer->k_tok_stride;
  wa.ws = ws; wa.fixup_pass = 0; wa.p = q; wa.pl = pl;
  wa.tc_min = 0; wa.force_exact = 1;   // the entropies and masses are outputs here
  for (int s = 0; s < 3 && e == cudaSuccess; ++s) {
    e = launch_window_stage(wa, s, st);
    if (e != cudaSuccess) {
      static const char* names[3] = {"window moments", "window pooling", "window pooling re-run"};
      return cuda_fail(e, names[s]);
    }
  }
  const float* exact = reinterpret_cast<const float*>(ws + pl.off_spec) + 2 * pl.H;
  Header* hdr = reinterpret_cast<Header*>(ws);
  if (e == cudaSuccess && out_entropy) e = cudaMemcpyAsync(out_entropy, exact, pl.H * 4, cudaMemcpyDeviceToDevice, st);
  if (e == cudaSuccess && out_mass) e = cudaMemcpyAsync(out_mass, exact + pl.H, pl.H * 4, cudaMemcpyDeviceToDevice, st);
  if (e == cudaSuccess && out_qi_heads) e = cudaMemcpyAsync(out_qi_heads, &hdr->qi_heads, 8, cudaMemcpyDeviceToDevice, st);
  if (e == cudaSuccess && out_hi_heads) e = cudaMemcpyAsync(out_hi_heads, &hdr->hi_heads, 8, cudaMemcpyDeviceToDevice, st);
  if (e == cudaSuccess && rows_qi)
    e = cudaMemcpy2DAsync(rows_qi, (size_t)pl.n * 4, ws + pl.off_rows_qi, (size_t)pl.n_pad * 4,
                          (size_t)pl.n * 4, pl.W, cudaMemcpyDeviceToDevice, st);
  if (e == cudaSuccess && rows_hi && pl.hi_rows)
    e = cudaMemcpy2DAsync(rows_hi, (size_t)pl.n * 4, ws + pl.off_rows_hi, (size_t)pl.n_pad * 4,
                          (size_t)pl.n * 4, pl.W, cudaMemcpyDeviceToDevice, st);
  return e == cudaSuccess ? CKV_OK : cuda_fail(e, "window stage");
}

static int check_walk(int32_t n, int32_t current_idx, int32_t num_walkers, int32_t max_steps,
                      int32_t sink_size, float temperature, float explore_temp, float explore_ratio,
                      int32_t rng_mode) {
  // the reference's argument checks (circuit_manager.cpp:1200-1226)
  if (n < 1) return fail(CKV_ERR_ARG, "seq_len must be >= 1");
  if (current_idx < 0 || current_idx >= n) return fail(CKV_ERR_ARG, "current_idx out of bounds");
  if (num_walkers < 1) return fail(CKV_ERR_ARG, "num_walkers must be >= 1");
  if (max_steps <= 0 || max_steps > 100) return fail(CKV_ERR_ARG, "max_steps must be in (0, 100]");
  if (sink_size < 0 || sink_size >= n) return fail(CKV_ERR_ARG, "sink_size out of bounds");
  if (!(temperature >= 0.1f && temperature <= 100.0f)) return fail(CKV_ERR_ARG, "temperature must be in [0.1, 100.0]");
  if (!(explore_temp >= 0.1f && explore_temp <= 100.0f)) return fail(CKV_ERR_ARG, "explore_temp must be in [0.1, 100.0]");
  if (!(explore_ratio >= 0.0f && explore_ratio <= 1.0f)) return fail(CKV_ERR_ARG, "explore_ratio must be in [0.0, 1.0]");
  if (rng_mode != CKV_RNG_PHILOX && rng_mode != CKV_RNG_PCG) return fail(CKV_ERR_ARG, "unknown rng_mode");
  return CKV_OK;
}

static WalkArgs walk_args(int32_t n, int32_t current_idx, int32_t num_walkers, int32_t max_steps,
                          int32_t sink_size, float temperature, float explore_temp, float explore_ratio,
                          int32_t rng_mode, uint64_t seed, uint64_t* rng_state, int32_t init_state,
                          float* visits, float* scores) {
  WalkArgs a;
  memset(&a, 0, sizeof(a));
  a.n = n; a.current_idx = current_idx; a.num_walkers = num_walkers; a.max_steps = max_steps;
  a.sink = sink_size;
  a.inv_temp = 1.0f / fmaxf(temperature, 0.1f);
  a.inv_explore_temp = 1.0f / fmaxf(explore_temp, 0.1f);
  a.explore_ratio = explore_ratio;
  a.rng_mode = rng_mode; a.seed = seed; a.rng_state = rng_state; a.init_state = init_state;
  a.visits = visits; a.scores = scores;
  return a;
}

int ckv_choose_heads(const ckv_params* p, int32_t num_heads, const float* entropy, const float* mass,
                     uint64_t* out_sets, int32_t* out_mode, ckv_stream_t stream) {
  if (!p || !entropy || !mass || !out_sets || !out_mode) return fail(CKV_ERR_ARG, "null argument");
  if (num_heads < 1 || num_heads > 32) return fail(CKV_ERR_UNSUPPORTED, "ckv_choose_heads: 1 to 32 heads");
  const cudaError_t e = launch_choose_heads(*p, num_heads, entropy, mass, out_sets, out_mode, (cudaStream_t)stream);
  return e == cudaSuccess ? CKV_OK : cuda_fail(e, "choose heads");
}

int ckv_pool_rows_given(const ckv_params* p, const ckv_layer* layer, int32_t head_offset, const uint64_t* sets,
                        const int32_t* mode, void* workspace, size_t workspace_bytes, float* rows_qi,
                        float* rows_hi, ckv_stream_t stream) {
  if (!p || !sets || !mode || !rows_qi) return fail(CKV_ERR_ARG, "null argument");
  int rc = check_layer(layer);
  if (rc) return rc;
  if (head_offset < 0 || head_offset + layer->num_heads > 64)
    return fail(CKV_ERR_ARG, "head_offset + num_heads must be at most 64");
  if (p->per_head_eviction) return fail(CKV_ERR_UNSUPPORTED, "head-sharded pooling is for shared eviction");
  ckv_params q = *p;
  if (q.max_capacity_prompt > layer->n) q.max_capacity_prompt = layer->n;
  Plan pl;
  const char* why = "";
  rc = make_plan(q, layer->n, layer->num_heads, layer->num_kv_heads, layer->head_dim, layer->dtype, &pl, &why);
  if (rc) return fail(rc, why);
  rc = check_ws(pl, workspace, workspace_bytes);
  if (rc) return rc;
  char* ws = static_cast<char*>(workspace);
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = cudaMemsetAsync(ws, 0, sizeof(Header), st);
  WinArgs wa;
  wa.q = layer->q; wa.qhs = layer->q_head_stride; wa.qts = layer->q_tok_stride;
  wa.k = layer->k; wa.khs = layer->k_head_stride; wa.kts = layer->k_tok_stride;
  wa.ws = ws; wa.fixup_pass = 0; wa.p = q; wa.pl = pl;
  wa.tc_min = 0; wa.force_exact = 0;
  if (e == cudaSuccess) e = launch_window_stage(wa, 0, st);   // row moments (log-sum-exp) of the local heads
  if (e == cudaSuccess) e = launch_set_heads(ws, head_offset, pl.H, sets, mode, st);
  if (e == cudaSuccess) e = launch_window_stage(wa, 1, st);   // pooling with the given sets
  if (e != cudaSuccess) return cuda_fail(e, "head-sharded pooling");
  e = cudaMemcpy2DAsync(rows_qi, (size_t)pl.n * 4, ws + pl.off_rows_qi, (size_t)pl.n_pad * 4, (size_t)pl.n * 4,
                        pl.W, cudaMemcpyDeviceToDevice, st);
  if (e == cudaSuccess && rows_hi && pl.hi_rows)
    e = cudaMemcpy2DAsync(rows_hi, (size_t)pl.n * 4, ws + pl.off_rows_hi, (size_t)pl.n_pad * 4,
                          (size_t)pl.n * 4, pl.W, cudaMemcpyDeviceToDevice, st);
  return e == cudaSuccess ? CKV_OK : cuda_fail(e, "head-sharded pooling output");
}

int ckv_graph_update(const void* query, const void* keys, int32_t dtype, int32_t n, int32_t head_dim,
                     int32_t current_idx, int32_t top_k, float* scratch, int32_t* adj_list, float* adj_weights,
                     ckv_stream_t stream) {
  if (!query || !keys || !scratch || !adj_list || !adj_weights) return fail(CKV_ERR_ARG, "null argument");
  if (dtype != CKV_BF16 && dtype != CKV_FP16 && dtype != CKV_FP32) return fail(CKV_ERR_DTYPE, "dtype must be bf16, fp16 or fp32");
  if (top_k <= 0 || top_k > 64) return fail(CKV_ERR_ARG, "top_k must be in (0, 64]");
  if (n <= 0 || head_dim <= 0 || head_dim > 1024 || current_idx < 0) return fail(CKV_ERR_ARG, "bad n, head_dim or current_idx");
  const cudaError_t e = launch_graph_update(query, keys, dtype, n, head_dim, current_idx, top_k, scratch, adj_list,
                                            adj_weights, (cudaStream_t)stream);
  return e == cudaSuccess ? CKV_OK : cuda_fail(e, "graph update");
}

int ckv_circuit_walk(const int32_t* adj_list, const float* adj_weights, int32_t n, int32_t top_k, int32_t source,
                     int32_t num_walkers, uint64_t* rng_state, int32_t* visits, int32_t clear_visits,
                     ckv_stream_t stream) {
  if (!adj_list || !adj_weights || !rng_state || !visits) return fail(CKV_ERR_ARG, "null argument");
  if (top_k <= 0 || top_k > 64 || n <= 0 || num_walkers <= 0) return fail(CKV_ERR_ARG, "bad n, top_k or num_walkers");
  if (source < 0 || source >= n) source = n - 1;   // as the reference's launcher
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = clear_visits ? cudaMemsetAsync(visits, 0, (size_t)n * sizeof(int32_t), st) : cudaSuccess;
  if (e == cudaSuccess) e = launch_circuit_walk(adj_list, adj_weights, visits, rng_state, source, n, top_k, num_walkers, st);
  return e == cudaSuccess ? CKV_OK : cuda_fail(e, "circuit walk");
}

int ckv_pcg_seed(uint64_t seed, int32_t num_walkers, uint64_t* rng_state, ckv_stream_t stream) {
  if (!rng_state || num_walkers <= 0) return fail(CKV_ERR_ARG, "bad arguments");
  const cudaError_t e = launch_pcg_init(rng_state, seed, num_walkers, (cudaStream_t)stream);
  return e == cudaSuccess ? CKV_OK : cuda_fail(e, "pcg seed");
}

int ckv_spectral_scores(const int32_t* adj_list, const float* adj_weights, int32_t n, int32_t top_k, int32_t iters,
                        float* v, float* scratch, ckv_stream_t stream) {
  if (!adj_list || !adj_weights || !v || !scratch) return fail(CKV_ERR_ARG, "null argument");
  if (n <= 0 || top_k <= 0 || top_k > 64 || iters < 0) return fail(CKV_ERR_ARG, "bad n, top_k or iters");
  if (iters == 0) return CKV_OK;   // the reference leaves the vector as it was
  const cudaError_t e = launch_spectral(adj_list, adj_weights, n, top_k, iters, v, scratch, (cudaStream_t)stream);
  return e == cudaSuccess ? CKV_OK : cuda_fail(e, "spectral scores");
}

int ckv_combine_scores(const int32_t* visits, float* spectral, float* walker_scores, float* combined, int32_t n,
                       ckv_stream_t stream) {
  if (!visits || !spectral || !walker_scores || !combined || n <= 0) return fail(CKV_ERR_ARG, "bad arguments");
  const cudaError_t e = launch_combine(visits, spectral, walker_scores, combined, n, (cudaStream_t)stream);
  return e == cudaSuccess ? CKV_OK : cuda_fail(e, "combine scores");
}

int ckv_landmark_workspace_size(int32_t n, size_t* bytes) {
  if (!bytes || n <= 0) return fail(CKV_ERR_ARG, "bad n or null pointer");
  *bytes = landmark_workspace_floats(n) * sizeof(float);
  return CKV_OK;
}

int ckv_landmark_walk(const float* attn, int32_t n, int32_t current_idx, int32_t mode, int32_t num_landmarks,
                      int32_t walkers_per_source, float query_boost, int32_t min_spacing, float position_alpha,
                      int32_t absorb_at_landmarks, uint64_t* rng_state, int32_t* visits, float* scores,
                      int32_t* positions, int32_t* count, void* workspace, size_t workspace_bytes,
                      ckv_stream_t stream) {
  if (!attn || !rng_state || !visits || !scores || !positions || !count || !workspace)
    return fail(CKV_ERR_ARG, "null argument");
  if (n <= 0 || current_idx < 0 || current_idx >= n) return fail(CKV_ERR_ARG, "bad n or current_idx");
  if (mode < CKV_LANDMARK_POSITIONAL || mode > CKV_LANDMARK_ABSORBING) return fail(CKV_ERR_ARG, "bad mode");
  if (num_landmarks < 1 || num_landmarks > 32) return fail(CKV_ERR_ARG, "num_landmarks must be in [1, 32]");
  if (walkers_per_source < 0 || (long long)(num_landmarks + 1) * walkers_per_source > INT32_MAX)
    return fail(CKV_ERR_ARG, "bad walkers_per_source");
  if (workspace_bytes < landmark_workspace_floats(n) * sizeof(float) || ((uintptr_t)workspace & 15u))
    return fail(CKV_ERR_WORKSPACE, "landmark workspace too small or misaligned");
  const cudaError_t e = launch_landmark_walk(attn, n, current_idx, mode, num_landmarks, walkers_per_source, query_boost,
                                             min_spacing, position_alpha, absorb_at_landmarks, rng_state, visits,
                                             scores, positions, count, static_cast<float*>(workspace),
                                             (cudaStream_t)stream);
  return e == cudaSuccess ? CKV_OK : cuda_fail(e, "landmark walk");
}

int ckv_influence_walk_dense(const float* attn, int32_t n, int32_t current_idx, int32_t num_walkers,
                             int32_t max_steps, int32_t sink_size, float temperature, float explore_temp,
                             float explore_ratio, int32_t rng_mode, uint64_t seed, uint64_t* rng_state,
                             int32_t init_state, float* visits, float* scores, ckv_stream_t stream) {
  if (!attn || !visits || !scores) return fail(CKV_ERR_ARG, "null argument");
  int rc = check_walk(n, current_idx, num_walkers, max_steps, sink_size, temperature, explore_temp,
                      explore_ratio, rng_mode);
  if (rc) return rc;
  WalkArgs a = walk_args(n, current_idx, num_walkers, max_steps, sink_size, temperature, explore_temp,
                         explore_ratio, rng_mode, seed, rng_state, init_state, visits, scores);
  a.attn = attn;
  const cudaError_t e = launch_walk_dense(a, (cudaStream_t)stream);
  return e == cudaSuccess ? CKV_OK : cuda_fail(e, "influence walker (dense)");
}

static size_t walk_ws_bytes(int32_t n, int32_t W) {
  const size_t n_p = n > W ? (size_t)(n - W) : 1;
  return align256(n_p * 4) + align256(n_p * 4) + align256((n_p + 1) * 2 * 8);
}

int ckv_walk_workspace_size(int32_t n, int32_t window, size_t* bytes) {
  if (!bytes || n < 1 || window < 1) return fail(CKV_ERR_ARG, "bad argument");
  *bytes = walk_ws_bytes(n, window);
  return CKV_OK;
}

int ckv_influence_walk(const float* rows, int32_t W, int32_t ld, int32_t n, int32_t current_idx,
                       int32_t num_walkers, int32_t max_steps, int32_t sink_size, float temperature,
                       float explore_temp, float explore_ratio, int32_t rng_mode, uint64_t seed,
                       uint64_t* rng_state, int32_t init_state, void* workspace, size_t workspace_bytes,
                       float* visits, float* scores, float* h2o, ckv_stream_t stream) {
  if (!rows || !visits || !scores || !h2o || !workspace) return fail(CKV_ERR_ARG, "null argument");
  if (W < 1 || W >= n || ld < n) return fail(CKV_ERR_ARG, "need 1 <= W < n and ld >= n");
  int rc = check_walk(n, current_idx, num_walkers, max_steps, sink_size, temperature, explore_temp,
                      explore_ratio, rng_mode);
  if (rc) return rc;
  if (workspace_bytes < walk_ws_bytes(n, W) || (uintptr_t)workspace % 256 != 0)
    return fail(CKV_ERR_WORKSPACE, "walker workspace too small or not 256-byte aligned");
  WalkArgs a = walk_args(n, current_idx, num_walkers, max_steps, sink_size, temperature, explore_temp,
                         explore_ratio, rng_mode, seed, rng_state, init_state, visits, scores);
  const size_t n_p = (size_t)(n - W);
  char* ws = static_cast<char*>(workspace);
  float* hbuf = reinterpret_cast<float*>(ws);
  float* cinv = reinterpret_cast<float*>(ws + align256(n_p * 4));
  double* pre = reinterpret_cast<double*>(ws + 2 * align256(n_p * 4));
  a.rows = rows; a.W = W; a.ld = ld; a.pre = pre; a.cinv = cinv; a.h2o = h2o;
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = launch_walk_prep(a, hbuf, cinv, pre, st);
  if (e == cudaSuccess) e = launch_walk_rows(a, st);
  return e == cudaSuccess ? CKV_OK : cuda_fail(e, "influence walker");
}

int ckv_rng_fill(int32_t mode, uint64_t seed, uint64_t stream_id, int32_t count, uint64_t* out,
                 ckv_stream_t stream) {
  if (!out || count < 0 || (mode != CKV_RNG_PHILOX && mode != CKV_RNG_PCG)) return fail(CKV_ERR_ARG, "bad argument");
  if (count == 0) return CKV_OK;
  const cudaError_t e = launch_rng_fill(mode, seed, stream_id, count, out, (cudaStream_t)stream);
  return e == cudaSuccess ? CKV_OK : cuda_fail(e, "rng fill");
}

int ckv_gather(const ckv_layer* layer, int32_t window, const int32_t* idx, int32_t kept, int32_t per_head,
               void* out_k, void* out_v, ckv_stream_t stream) {
  int rc = check_layer(layer);
  if (rc) return rc;
  if (!idx || !out_k || !out_v || kept < 0 || window < 0 || window > layer->n)
    return fail(CKV_ERR_ARG, "bad gather argument");
  if (layer->num_heads % layer->num_kv_heads != 0) return fail(CKV_ERR_ARG, "num_heads % num_kv_heads != 0");
  GatherArgs g;
  g.k = layer->k; g.khs = layer->k_head_stride; g.kts = layer->k_tok_stride;
  g.v = layer->v; g.vhs = layer->v_head_stride; g.vts = layer->v_tok_stride;
  g.out_k = out_k; g.out_v = out_v; g.distinct = 0; g.idx = idx;
  g.n = layer->n; g.W = window; g.H = layer->num_heads; g.Hkv = layer->num_kv_heads;
  g.G = layer->num_heads / layer->num_kv_heads; g.D = layer->head_dim;
  g.out_len = kept + window; g.per_head = per_head ? 1 : 0; g.identity = 0;
  const cudaError_t e = launch_gather(g, layer->dtype, (cudaStream_t)stream);
  return e == cudaSuccess ? CKV_OK : cuda_fail(e, "gather");
}

int ckv_copy_rows(void* dst, size_t dst_pitch, const void* src, size_t src_pitch, size_t row_bytes, int32_t rows,
                  ckv_stream_t stream) {
  if (!dst || !src || rows < 0 || row_bytes > dst_pitch || row_bytes > src_pitch)
    return fail(CKV_ERR_ARG, "bad copy geometry");
  if (rows == 0 || row_bytes == 0) return CKV_OK;
  const cudaError_t e = cudaMemcpy2DAsync(dst, dst_pitch, src, src_pitch, row_bytes, (size_t)rows, cudaMemcpyDefault,
                                          (cudaStream_t)stream);
  return e == cudaSuccess ? CKV_OK : cuda_fail(e, "strided row copy");
}

int ckv_device_accessible(const void* ptr, int32_t* accessible) {
  if (!accessible) return fail(CKV_ERR_ARG, "null argument");
  *accessible = 0;
  if (!ptr) return CKV_OK;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) { cudaGetLastError(); return CKV_OK; }
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, ptr) != cudaSuccess) { cudaGetLastError(); return CKV_OK; }
  if (at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged)
    *accessible = at.device == dev ? 1 : 0;
  else if (at.type == cudaMemoryTypeHost)   // page-locked: mapped at the same address under UVA
    *accessible = at.devicePointer == ptr ? 1 : 0;
  return CKV_OK;
}

int ckv_set_stage_events(void* const* events, int32_t count) {
  if (count < 0 || (count > 0 && !events)) return fail(CKV_ERR_ARG, "bad stage event list");
  g_stage_events = count ? reinterpret_cast<cudaEvent_t*>(const_cast<void**>(events)) : nullptr;
  g_stage_count = count;
  g_stage_next = 0;
  return CKV_OK;
}

const char* ckv_last_error_string(void) { return g_last_error.c_str(); }

const char* ckv_version(void) { return "circuitkv-b200 0.1.0"; }

}  // extern "C"
