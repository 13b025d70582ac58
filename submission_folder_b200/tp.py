"""Head-sharded (tensor-parallel) scoring of one layer.

When a serving engine splits the KV heads of a layer over ranks (tensor parallelism),
no rank holds all heads, yet the reference's scoring ranks and pools ACROSS heads
(``KVCache-Factory/pyramidkv/pyramidkv_utils.py`` PU:2905-2999: the 10 lowest-entropy
heads are max-pooled into the QI rows, the heads with transient mass >= 0.5 averaged
into the HI rows).  The reference itself has no such mode (it scores a layer in one
process); this one gives the same result from sharded heads with two collectives on
the data path:

1. each rank computes its heads' exact entropy / transient mass (``ckv_window_pool``);
2. one all-gather of those ``[H_local]`` values; every rank derives the same head sets
   from all ``H`` of them (``ckv_choose_heads``);
3. each rank pools its heads with those sets (``ckv_pool_rows_given``): QI rows = max over
   its QI heads, HI rows = sum over its HI heads;
4. one all-reduce of the ``[W, n]`` rows: max for QI, sum for HI (max when HI pools by
   max), then HI is scaled by 1 / (HI head count) as the single-process mean is;
5. every rank scores and selects from the combined rows (``ckv_neumann_rows``,
   ``ckv_select_scores``) -- the same kept positions on every rank -- and gathers the K / V
   rows of its own heads (``ckv_gather``).

Combination modes "dis" (the CLI default) and "union" (scores that come from the pooled
rows alone); 32 query heads at most per layer.  Works over any
``torch.distributed`` backend (NCCL on GPUs; gloo in the CPU tests, with the oracle as
the ``backend``).
"""

from __future__ import annotations

import torch

from ._lib import COMB_CODES, Params


class CudaBackend:
    """The per-rank steps on the sm_100a kernels of ``libckv.so``."""

    def __init__(self):
        from . import ops
        self.ops = ops

    def head_stats(self, p: Params, q, k):
        ent, mass, _, _, _ = self.ops.window_pool(p, q, k)
        return ent, mass

    def choose_heads(self, p: Params, ent, mass):
        return self.ops.choose_heads(p, ent, mass)

    def hi_count(self, mode):
        return mode[1:2].float()

    def pool_rows(self, p: Params, q, k, head_offset: int, sets, mode):
        return self.ops.pool_rows_given(p, q, k, head_offset, sets, mode)

    def select(self, p: Params, rows_qi, rows_hi):
        qi, hi, _ = self.ops.neumann_rows(p, rows_qi, rows_hi)
        idx, scores = self.ops.select_scores(p, qi, hi, want_scores=True)
        return idx, scores

    def gather(self, q, k, v, window: int, idx):
        return self.ops.gather(q, k, v, window, idx)


def score_evict_head_sharded(p: Params, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, group=None,
                             backend=None):
    """One layer's eviction with this rank holding heads ``rank * H_local .. (rank + 1) *
    H_local - 1`` (``q`` ``[H_local, n, D]``, ``k`` / ``v`` ``[Hkv_local, n, D]``, every rank
    the same counts).  Returns ``(k_out, v_out, keep_idx, scores)``: this rank's heads'
    compressed K / V ``[H_local, out_len, D]``, the kept prefix positions (the same on every
    rank) and the two ranked score vectors ``[2, n]``."""
    import torch.distributed as dist

    if p.combination_mode not in (COMB_CODES["dis"], COMB_CODES["union"]):
        raise ValueError("head-sharded scoring supports combination modes dis and union")
    if p.per_head_eviction:
        raise ValueError("head-sharded scoring is for shared eviction")
    be = backend if backend is not None else CudaBackend()
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    h_local = q.shape[0]
    if h_local * world > 32:
        raise ValueError("at most 32 query heads per layer")
    n = q.shape[1]
    if n < p.max_capacity_prompt:   # the reference returns its inputs unchanged
        idx = torch.arange(max(n - p.window_size, 0), dtype=torch.int32, device=q.device)
        return k, v, idx, None
    # 1-2: exact per-head statistics, all-gathered; the same head sets on every rank
    ent, mass = be.head_stats(p, q, k)
    ent_all = torch.empty(h_local * world, dtype=ent.dtype, device=ent.device)
    mass_all = torch.empty_like(ent_all)
    dist.all_gather_into_tensor(ent_all, ent.contiguous(), group=group)
    dist.all_gather_into_tensor(mass_all, mass.contiguous(), group=group)
    sets, mode = be.choose_heads(p, ent_all, mass_all)
    # 3-4: this rank's partial rows, combined over the ranks
    rows_qi, rows_hi = be.pool_rows(p, q, k, rank * h_local, sets, mode)
    dist.all_reduce(rows_qi, op=dist.ReduceOp.MAX, group=group)
    hi_rows = bool(p.entropy_aware)   # without entropy-aware pooling the HI chain reuses the QI rows
    if hi_rows:
        if p.hi_pooling_mode == 1:
            dist.all_reduce(rows_hi, op=dist.ReduceOp.MAX, group=group)
        else:
            dist.all_reduce(rows_hi, op=dist.ReduceOp.SUM, group=group)
            rows_hi.mul_(1.0 / be.hi_count(mode))   # mean = sum * (1 / count), as the single-process path
    # 5: scores and selection (identical on every rank), then this rank's heads' K / V
    idx, scores = be.select(p, rows_qi, rows_hi if hi_rows else None)
    k_out, v_out = be.gather(q, k, v, p.window_size, idx)
    return k_out, v_out, idx, scores


def heads_for_rank(num_heads: int, num_kv_heads: int, rank: int, world: int):
    """Contiguous head split: (query heads, KV heads) slices of this rank; every rank must
    get whole KV groups."""
    if num_kv_heads % world or num_heads % world:
        raise ValueError("heads must split evenly over the ranks")
    hq, hk = num_heads // world, num_kv_heads // world
    return slice(rank * hq, (rank + 1) * hq), slice(rank * hk, (rank + 1) * hk)
