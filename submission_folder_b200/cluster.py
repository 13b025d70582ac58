"""Drop-in ``CircuitKVCluster`` / ``init_circuitkv`` for the KVCache-Factory hook.

Mirrors ``KVCache-Factory/pyramidkv/pyramidkv_utils.py``:
``CircuitKVCluster.__init__`` (PU:1244-1431, same keyword names and class
defaults), ``reset`` (PU:1432-1450), ``update_kv`` (PU:2775-3519) and
``init_circuitkv`` (PU:3829-3998, same ``config`` attribute names and
``hasattr`` / ``getattr`` defaults).  ``update_kv`` runs the sm_100a kernels of
``libckv.so`` on torch's current stream without a host synchronisation.

Differences from the reference, by design:
* no per-call ``print`` (PU:2861) and no debug log file (PU:1548-1838);
* batch size must be 1 (the reference averages attention over the batch and
  gathers one index set for all sequences, PU:2923/2998; independent sequences go
  through ``submission_folder_b200.ops`` / ``ckv_score_evict_batched``);
* host (CPU) tensors are moved to the current CUDA device and the results moved
  back -- the kernels never run on the CPU.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from . import _lib, ops
from ._lib import Params


class CircuitKVCluster:
    """Prefill KV eviction by absorbing-Markov importance (QI / HI), B200 kernels."""

    def __init__(
        self,
        window_size: int = 32,
        max_capacity_prompt: int = 2048,
        kernel_size: int = 5,
        pooling: str = 'avgpool',
        merge=None,
        sink_size: int = 4,
        top_k: int = 32,
        alpha: float = 0.85,
        num_walkers: int = 10000,
        num_steps: int = 100,
        max_steps: int = 10,
        decay: float = 0.95,
        observation_window: int = 1,
        bidirectional: bool = False,
        use_combined_scoring: bool = False,
        num_power_iterations: int = 10,
        num_landmarks: int = 8,
        min_spacing: int = 50,
        walkers_per_source: int = 100,
        query_boost: float = 2.0,
        position_alpha: float = 0.6,
        use_reachability: bool = False,
        absorb_at_landmarks: bool = True,
        debug: bool = False,
        use_instruction_anchors: bool = False,
        use_fundamental_norm: bool = False,
        use_multi_horizon: bool = True,
        tokenizer=None,
        use_neumann: bool = True,
        neumann_iterations: int = 10,
        neumann_temperature: float = 1.0,
        neumann_gamma: float = 1.0,
        qi_gamma: Optional[float] = None,
        hi_gamma: Optional[float] = None,
        h2o_weight: float = 0.5,
        combination_mode: str = "dis",
        dis_alpha: float = 0.5,
        qi_ratio: float = 0.5,
        ablate_qi: bool = False,
        ablate_hi: bool = False,
        per_head_eviction: bool = False,
        head_chunk_size: int = 8,
        true_hub_hi: bool = False,
        entropy_adaptive: bool = True,
        smoothing_kernel: int = 0,
        smooth_hi_only: bool = False,
        use_gaussian: bool = False,
        qi_kernel_size: int = 0,
        hi_kernel_size: int = 0,
        gaussian_sigma: float = 1.0,
        entropy_aware: bool = False,
        top_k_heads: int = 8,
        head_selection_mode: str = "entropy",
        hi_pooling_mode: str = "mean",
        hi_mass_threshold: float = 0.0,
        hi_top_k_heads: int = 0,
        hi_mass_cdf: float = 0.0,
        hi_log_head_stats: bool = False,
        use_bridge_importance: bool = False,
        bi_kernel_size: int = 5,
        distinct_kv_heads: bool = False,
    ):
        self.window_size = window_size
        self.max_capacity_prompt = max_capacity_prompt
        self.kernel_size = kernel_size
        self.pooling = pooling
        self.merge = merge
        self.sink_size = sink_size
        self.top_k = top_k
        self.alpha = alpha
        self.num_walkers = num_walkers
        self.num_steps = num_steps
        self.max_steps = max_steps
        self.decay = decay
        self.observation_window = observation_window
        self.bidirectional = bidirectional
        self.use_combined_scoring = use_combined_scoring
        self.num_power_iterations = num_power_iterations
        self.num_landmarks = num_landmarks
        self.min_spacing = min_spacing
        self.walkers_per_source = walkers_per_source
        self.query_boost = query_boost
        self.position_alpha = position_alpha
        self.use_reachability = use_reachability
        self.absorb_at_landmarks = absorb_at_landmarks
        self.debug = debug
        self.use_instruction_anchors = use_instruction_anchors
        self.use_fundamental_norm = use_fundamental_norm
        self.use_multi_horizon = use_multi_horizon
        self.tokenizer = tokenizer
        self.use_neumann = use_neumann
        self.neumann_iterations = neumann_iterations
        self.neumann_temperature = neumann_temperature
        self.neumann_gamma = neumann_gamma
        self.qi_gamma = qi_gamma if qi_gamma is not None else neumann_gamma
        self.hi_gamma = hi_gamma if hi_gamma is not None else neumann_gamma
        self.h2o_weight = h2o_weight
        self.combination_mode = combination_mode
        self.dis_alpha = dis_alpha
        self.qi_ratio = qi_ratio
        self.ablate_qi = ablate_qi
        self.ablate_hi = ablate_hi
        self.per_head_eviction = per_head_eviction
        self.head_chunk_size = head_chunk_size
        self.true_hub_hi = true_hub_hi
        self.entropy_adaptive = entropy_adaptive
        self.smoothing_kernel = smoothing_kernel
        self.smooth_hi_only = smooth_hi_only
        self.use_gaussian = use_gaussian
        self.qi_kernel_size = qi_kernel_size
        self.hi_kernel_size = hi_kernel_size
        self.gaussian_sigma = gaussian_sigma
        self.entropy_aware = entropy_aware
        self.top_k_heads = top_k_heads
        self.head_selection_mode = head_selection_mode
        self.hi_pooling_mode = hi_pooling_mode
        self.hi_mass_threshold = hi_mass_threshold
        self.hi_top_k_heads = hi_top_k_heads
        self.hi_mass_cdf = hi_mass_cdf
        self.hi_log_head_stats = hi_log_head_stats
        self.use_bridge_importance = use_bridge_importance
        self.bi_kernel_size = bi_kernel_size
        # not a reference kwarg: return each KV head once ([1, Hkv, B, D], no repeat_kv
        # copies) for a decode cache that keeps the distinct heads (cache.DistinctKVCache)
        self.distinct_kv_heads = distinct_kv_heads
        # state of the last call (for callers that want the kept positions)
        self.last_keep_indices: Optional[torch.Tensor] = None
        self._graph = None
        self._walk_rng = None         # influence-walker PCG states (use_neumann=False)
        self._walk_rng_init = True
        self._device = None

    def reset(self, window_size: int = 64, max_capacity_prompt: int = 2048, kernel_size: int = 5,
              pooling: str = 'avgpool', merge=None):
        """PU:1432-1450."""
        self.window_size = window_size
        self.max_capacity_prompt = max_capacity_prompt
        self.kernel_size = kernel_size
        self.pooling = pooling
        self.merge = merge
        self.last_keep_indices = None

    # -- parameters -----------------------------------------------------------
    def _budget(self, q_len: int) -> int:
        b = self.max_capacity_prompt
        if isinstance(b, float) and b <= 1.0 and self.combination_mode not in ("union", "union_da"):
            return int(q_len * b)          # dynamic budget (PU:2612-2614)
        return int(b)

    def params(self, q_len: int) -> Params:
        """The ``ckv_params`` of this cluster for a prefill of length ``q_len``."""
        p = Params()
        p.window_size = int(self.window_size)
        p.max_capacity_prompt = self._budget(q_len)
        p.sink_size = int(self.sink_size)
        p.neumann_iterations = int(self.neumann_iterations)
        p.neumann_temperature = float(self.neumann_temperature)
        p.neumann_gamma = float(self.neumann_gamma)
        p.qi_gamma = float(self.qi_gamma)
        p.hi_gamma = float(self.hi_gamma)
        mode = self.combination_mode
        if mode not in ("dis", "union", "union_da"):
            mode = "weighted" if mode == "weighted" else "max"
        p.combination_mode = _lib.COMB_CODES[mode]
        p.h2o_weight = float(self.h2o_weight)
        p.qi_ratio = float(self.qi_ratio)
        p.ablate_qi = int(bool(self.ablate_qi))
        p.ablate_hi = int(bool(self.ablate_hi))
        p.per_head_eviction = int(bool(self.per_head_eviction))
        p.true_hub_hi = int(bool(self.true_hub_hi))
        p.entropy_adaptive = int(bool(self.entropy_adaptive))
        p.smoothing_kernel = int(self.smoothing_kernel)
        p.smooth_hi_only = int(bool(self.smooth_hi_only))
        p.use_gaussian = int(bool(self.use_gaussian))
        p.qi_kernel_size = int(self.qi_kernel_size)
        p.hi_kernel_size = int(self.hi_kernel_size)
        p.gaussian_sigma = float(self.gaussian_sigma)
        p.entropy_aware = int(bool(self.entropy_aware))
        p.top_k_heads = int(self.top_k_heads)
        p.head_selection_mode = 1 if self.head_selection_mode == "mass" else 0
        p.hi_pooling_mode = 0 if self.hi_pooling_mode == "mean" else 1
        p.hi_mass_threshold = float(self.hi_mass_threshold)
        p.hi_top_k_heads = int(self.hi_top_k_heads)
        p.hi_mass_cdf = float(self.hi_mass_cdf)
        p.use_bridge_importance = int(bool(self.use_bridge_importance))
        p.bi_kernel_size = int(self.bi_kernel_size)
        return p

    # -- the hook ---------------------------------------------------------------
    def update_kv(self, key_states: torch.Tensor, query_states: torch.Tensor,
                  value_states: torch.Tensor, attention_mask, num_key_value_groups: int):
        """PU:2775: returns the compressed ``(key_states, value_states)``."""
        assert key_states.shape[-2] == query_states.shape[-2]
        bsz, num_heads, q_len, head_dim = query_states.shape
        if q_len < self.max_capacity_prompt:
            return key_states, value_states
        if bsz != 1:
            raise NotImplementedError("CircuitKVCluster.update_kv supports batch size 1 "
                                      "(independent sequences: ckv_score_evict_batched)")
        host = not query_states.is_cuda
        if host:
            if not torch.cuda.is_available():
                raise RuntimeError("the CircuitKV B200 kernels need a CUDA device")
            dev = torch.device("cuda", torch.cuda.current_device())
        else:
            dev = query_states.device
        groups = int(num_key_value_groups)
        q, k, v = self._views(query_states, key_states, value_states, groups, num_heads)
        if host:
            W = int(self.window_size)
            qd = torch.empty(q.shape, dtype=q.dtype, device=dev)   # only the window rows are read
            # the window rows of every head in one strided copy (per-head copies cost ~12 us each)
            if not ops.copy_rows_async(qd[:, q_len - W:], q[:, q_len - W:]):
                for h in range(q.shape[0]):
                    qd[h, q_len - W:].copy_(q[h, q_len - W:], non_blocking=True)
            q = qd
            k = _to_device_by_head(k, dev)
            # V is read only by the final gather (the kept rows): from a page-locked host
            # tensor the device reads those rows in place instead of copying all of V
            if not ops.device_readable(v):
                v = _to_device_by_head(v, dev)
        p = self.params(q_len)
        if not self.use_neumann and self.combination_mode not in ("dis", "union", "union_da"):
            k_out, v_out, idx = self._walker_path(p, q, k, v, q_len)
        else:
            k_out, v_out, idx, _ = ops.score_evict(p, q, k, v, distinct_kv_heads=self.distinct_kv_heads)
        self.last_keep_indices = idx
        k_out, v_out = k_out.unsqueeze(0), v_out.unsqueeze(0)
        if host:
            # one pass over the link each way at full rate: pinned outputs (torch's caching
            # host allocator), asynchronous copies, one wait
            kh = torch.empty(k_out.shape, dtype=k_out.dtype, pin_memory=True)
            vh = torch.empty(v_out.shape, dtype=v_out.dtype, pin_memory=True)
            kh.copy_(k_out, non_blocking=True)
            vh.copy_(v_out, non_blocking=True)
            torch.cuda.current_stream(dev).synchronize()
            k_out, v_out = kh, vh
        return k_out, v_out

    def _walker_path(self, p, q, k, v, q_len):
        if self.distinct_kv_heads:
            raise NotImplementedError("distinct_kv_heads with use_neumann=False")
        """use_neumann=False (PU:3244-3263): pooled window rows, the influence walker on
        the structured full_attn (its PCG states kept across calls like the reference's
        CircuitGraph, seeded once with 42 + 3000), H2O = full_attn column sums, rank MAX,
        keep mask, gather."""
        _, _, _, rows_qi, _ = ops.window_pool(p, q, k)
        if self._walk_rng is None or self._walk_rng.device != q.device:
            self._walk_rng = torch.zeros(2 * 10000, dtype=torch.int64, device=q.device)
            self._walk_rng_init = True
        scores, _, h2o = ops.influence_walk(rows_qi, q_len - 1, int(self.num_walkers), int(self.max_steps),
                                            int(self.sink_size), rng_state=self._walk_rng,
                                            init_state=self._walk_rng_init)
        self._walk_rng_init = False
        pm = self.params(q_len)
        pm.combination_mode = _lib.COMB_CODES["max"]
        idx, _ = ops.select_scores(pm, scores, h2o)
        k_out, v_out = ops.gather(q, k, v, int(self.window_size), idx)
        return k_out, v_out, idx

    @staticmethod
    def _views(query_states, key_states, value_states, groups, num_heads):
        q = query_states[0]
        if q.stride(-1) != 1:
            q = q.contiguous()

        def distinct(x):
            x = x[0]
            if x.stride(-1) != 1:
                x = x.contiguous()
            if x.shape[0] == num_heads and groups > 1:
                return x[::groups]          # repeat_kv layout: heads g*groups .. share a KV head
            return x
        return q, distinct(key_states), distinct(value_states)


def _to_device_by_head(x: torch.Tensor, dev: torch.device) -> torch.Tensor:
    """Copy a [heads, n, D] host view (heads possibly strided, e.g. every groups-th
    head of a repeat_kv'd tensor) as one strided asynchronous copy (one per head when a
    head's rows are not contiguous)."""
    out = torch.empty(x.shape, dtype=x.dtype, device=dev)
    if not ops.copy_rows_async(out, x):
        for h in range(x.shape[0]):
            out[h].copy_(x[h], non_blocking=True)
    return out


def init_circuitkv(self):
    """PU:3829-3998: build ``self.kv_cluster`` from ``self.config`` attributes."""
    if not hasattr(self, "kv_cluster"):
        c = self.config
        defaults = dict(window_size=64, max_capacity_prompt=2048, kernel_size=5, pooling='avgpool',
                        merge=None, sink_size=4, top_k=32, alpha=0.85, num_walkers=10000,
                        num_steps=100, max_steps=50, decay=0.99, bidirectional=False,
                        num_landmarks=8, min_spacing=50, walkers_per_source=100, query_boost=2.0,
                        position_alpha=0.6, use_reachability=False, absorb_at_landmarks=True,
                        circuitkv_debug=False, use_neumann=True, neumann_iterations=10,
                        neumann_temperature=1.0, h2o_weight=0.5, combination_mode="dis",
                        dis_alpha=0.5, ablate_qi=False, ablate_hi=False, per_head_eviction=False,
                        head_chunk_size=8, qi_ratio=0.5, smoothing_kernel=0, smooth_hi_only=False,
                        use_gaussian=False, qi_kernel_size=0, hi_kernel_size=0, gaussian_sigma=1.0)
        for name, val in defaults.items():
            if not hasattr(c, name):
                setattr(c, name, val)
    c = self.config
    self.kv_cluster = CircuitKVCluster(
        window_size=c.window_size, max_capacity_prompt=c.max_capacity_prompt,
        kernel_size=c.kernel_size, pooling=c.pooling, merge=c.merge, sink_size=c.sink_size,
        top_k=c.top_k, alpha=c.alpha, num_walkers=c.num_walkers, num_steps=c.num_steps,
        max_steps=c.max_steps, decay=c.decay, bidirectional=c.bidirectional,
        num_landmarks=c.num_landmarks, min_spacing=c.min_spacing,
        walkers_per_source=c.walkers_per_source, query_boost=c.query_boost,
        position_alpha=c.position_alpha, use_reachability=c.use_reachability,
        absorb_at_landmarks=c.absorb_at_landmarks, debug=c.circuitkv_debug,
        use_neumann=c.use_neumann, neumann_iterations=c.neumann_iterations,
        neumann_temperature=c.neumann_temperature,
        neumann_gamma=getattr(c, 'neumann_gamma', 1.0),
        qi_gamma=getattr(c, 'qi_gamma', None), hi_gamma=getattr(c, 'hi_gamma', None),
        h2o_weight=c.h2o_weight, combination_mode=c.combination_mode, dis_alpha=c.dis_alpha,
        ablate_qi=c.ablate_qi, ablate_hi=c.ablate_hi, per_head_eviction=c.per_head_eviction,
        head_chunk_size=c.head_chunk_size, true_hub_hi=getattr(c, 'true_hub_hi', False),
        entropy_adaptive=getattr(c, 'entropy_adaptive', True), qi_ratio=c.qi_ratio,
        smoothing_kernel=c.smoothing_kernel, smooth_hi_only=c.smooth_hi_only,
        use_gaussian=c.use_gaussian, qi_kernel_size=c.qi_kernel_size,
        hi_kernel_size=c.hi_kernel_size, gaussian_sigma=c.gaussian_sigma,
        entropy_aware=getattr(c, 'entropy_aware', False), top_k_heads=getattr(c, 'top_k_heads', 8),
        head_selection_mode=getattr(c, 'head_selection_mode', 'entropy'),
        hi_pooling_mode=getattr(c, 'hi_pooling_mode', 'mean'),
        hi_mass_threshold=getattr(c, 'hi_mass_threshold', 0.0),
        hi_top_k_heads=getattr(c, 'hi_top_k_heads', 0), hi_mass_cdf=getattr(c, 'hi_mass_cdf', 0.0),
        hi_log_head_stats=getattr(c, 'hi_log_head_stats', False),
        use_bridge_importance=getattr(c, 'use_bridge_importance', False),
        bi_kernel_size=getattr(c, 'bi_kernel_size', 5),
    )


def cli_cluster_kwargs(window_size: int = 64, max_capacity_prompt: int = 2048, **over) -> dict:
    """Keyword arguments KVCache-Factory's run_longbench.py passes by default (run_longbench.py:505-548)."""
    kw = dict(window_size=window_size, max_capacity_prompt=max_capacity_prompt, kernel_size=7,
              pooling='maxpool', sink_size=4, combination_mode='dis', entropy_aware=True,
              top_k_heads=10, hi_pooling_mode='mean', hi_mass_threshold=0.5, use_gaussian=True,
              qi_kernel_size=3, hi_kernel_size=5, gaussian_sigma=1.0, neumann_iterations=10,
              neumann_temperature=1.0, neumann_gamma=1.0, per_head_eviction=False)
    kw.update(over)
    return kw
