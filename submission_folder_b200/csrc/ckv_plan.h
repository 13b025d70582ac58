// Host/device plan of one layer call: sizes, tiling and the workspace carve-up.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include "../../include/ckv.h"

namespace ckv {

constexpr int kColTile = 64;        // key columns per MMA tile
constexpr int kScanChunk = 1024;    // prefix positions per sweep chunk (one CTA)
constexpr int kSweepThreads = 256;  // threads per sweep CTA
constexpr int kSweepRun = kScanChunk / kSweepThreads;   // consecutive positions per thread
constexpr int kWarps = 8;           // warps of the window kernels

// Workspace header (first 512 bytes of every layer workspace).
struct alignas(16) Header {
  int32_t status;          // device failure bits (kStatus*)
  uint32_t cnt_stats;      // arrival counter of the stats kernel
  uint32_t cnt_pool;       // arrival counter of the pooling kernel
  int32_t fixup;           // 1: the speculative head sets were wrong, pooling re-runs
  uint64_t qi_heads;       // head set max-pooled into the QI rows
  uint64_t hi_heads;       // head set pooled into the HI rows
  int32_t hi_mode;         // 0 mean, 1 max, 2 HI reuses the QI rows
  int32_t n_hi;            // heads in the HI set
  int32_t steps;           // Neumann terms taken (early stop)
  int32_t kept;            // prefix positions kept (selection output count)
  uint32_t tile_ctr[2];    // next column tile of the tensor-core pooling launch (pass, re-run)
  int32_t need_exact;      // 1: the pooling pass recomputes the clamped entropy / mass exactly
  uint32_t cnt_sweep[2];   // arrival counters of the sweep's chunk kernel, per chain
  int32_t pad[47];
  uint32_t cnt_group[64];  // arrival counters per head group of the stats kernel
};
static_assert(sizeof(Header) == 512, "header must be 512 bytes");

struct Plan {
  // shapes
  int n, H, Hkv, G, D, W, s, K, dtype;
  int n_p;            // n - W: prefix rows (structured transitions)
  int out_len;        // tokens kept per head
  int kk;             // tokens chosen by top-k (out_len - s - W)
  int mode;           // combination mode
  int per_head;       // per-head eviction
  int nchains;        // 2 (QI, HI) or 1 (single-chain influence)
  int tc;             // 1: window moments on tcgen05 tensor cores (16-bit inputs, G*W a multiple of 128)
  int tc_pool;        // 1: pooling pass on tcgen05 with one cluster CTA per KV group
  int lanes_pool;     // 1: W = 32 / 128: keys-on-lanes tcgen05 pooling when the head sets are
                      //    settled; the exact recomputation runs on the SIMT / mma.sync pass
  int pool_blocks;    // row blocks of the keys-on-lanes column-sum partials (W / 16, at least 4)
  int tc_nclusters;   // clusters of the tensor-core pooling pass
  int e_parts;        // exact entropy / mass partials per row
  int rs_parts;       // row-sum partials per chain (tensor-core pooling: one per 32 keys)
  int g_slice;        // columns per g-total partial (64 or 8)
  int hi_rows;        // 1 when the HI chain has its own pooled rows
  // window tiling
  int rows_per_warp;  // 32 (16-bit MMA) or 16 (fp32 SIMT)
  int rows_per_batch; // kWarps * rows_per_warp
  int heads_per_batch;
  int nbatch;         // H / heads_per_batch
  int ktiles_per_batch;  // distinct KV heads one batch touches
  int ncol_tiles;     // ceil(n / kColTile)
  int nstat_chunks;   // column chunks of the stats kernel
  int tiles_per_chunk;
  int n_pad;          // ncol_tiles * kColTile
  // sweep tiling
  int nscan;          // ceil(n_p / kScanChunk)
  // workspace offsets (bytes from the layer workspace base)
  size_t off_stats, off_lse, off_lastlogit, off_spec, off_epart, off_mpart;
  size_t off_minx;    // [nstat_chunks][H][W] row minimum of the rounded logits (tensor-core moments)
  size_t off_rows_qi, off_rows_hi, off_colsum, off_gtile, off_rspart;
  size_t off_colpart;  // [2][pool_blocks][n_pad] column-sum partials of the keys-on-lanes pooling pass
  size_t off_wk, off_yk, off_ymax, off_bk, off_cg, off_agg, off_sin, off_cum, off_cmax;
  size_t off_sel, off_ph;
  // per-head eviction (PU:2208-2382, 3296-3464): only allocated in that mode
  size_t off_ph_q2w;   // [H][W] query row -> window columns
  size_t off_ph_qrow;  // [H][n] query row
  size_t off_ph_two;   // [H][n] two-hop attention through the window rows
  size_t off_ph_col;   // [H][n] column sums over the window rows
  size_t off_ph_ent;   // [ph_ent_parts][H] query-row entropy partials, then [H] totals
  size_t off_ph_part;  // tcgen05 per-head pass: [2][ph_slots][H][n] two-hop / column-sum partials
  size_t off_ph_vec;   // [H][2][nw] finished, truncated, smoothed QI / HI (or H2O)
  size_t off_ph_ghi;   // [nw] rank-normalised mean over heads of HI
  size_t off_ph_gbuf;  // [2][nw] u64 + [nw] int: ranking scratch of the mean HI
  size_t off_ph_bufs;  // [H][2][2][nw] u64: per-head ranking scratch
  size_t off_ph_ranks; // [H][2][nw] int
  size_t off_ph_bits;  // [H][ceil(nw / 32)] keep bits
  int ph_nw;           // n - W
  int ph_tc;           // 1: per-head pass on tcgen05 (keys-on-lanes form)
  int ph_slots;        // its partial slots per (head, key): 4 row blocks per 64-row half
  int ph_ent_parts;    // entropy partials per head: one per 32 keys (tcgen05) or per 64-key tile
  size_t sel_bytes;
  size_t total;
};

// Fills *pl for one layer; returns CKV_OK or an error status with a message.
int make_plan(const ckv_params& p, int n, int H, int Hkv, int D, int dtype, Plan* pl,
              const char** why);

}  // namespace ckv
