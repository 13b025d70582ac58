"""Configs and decode-time monitors of the ``circuit_kv`` package.

Same public names, fields, defaults and methods as the reference's
``CircuitKV/circuit_kv/engine.py`` (``CircuitKVConfig`` :20-46,
``LandmarkWalkerConfig`` :48-81, ``CircuitKVMonitor`` :84-349,
``LandmarkWalkerMonitor`` :351-526), so code written against the reference
imports and constructs them unchanged.

The monitors keep their host-side logic here: the prefill charge initialisation
from H2O column sums, the exponential moving average of the charge, the keep mask
(sinks and local window forced, top-k of the rest).  The walker steps they call
(``CircuitGraph.update_and_step_circuit``, ``update_and_step_landmark_walker``
and their score getters) are decode-time kernels that this library does not
provide: those calls raise ``NotImplementedError`` from ``circuit_kv._C``.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch


@dataclass
class CircuitKVConfig:
    """Fields and defaults of the reference's ``CircuitKVConfig``."""

    max_seq_len: int = 8192
    top_k: int = 32
    num_walkers: int = 1024
    alpha: float = 0.85
    num_steps: int = 100
    sink_size: int = 4
    local_window: int = 64
    decay: float = 0.95
    device: str = "cuda"
    dtype: torch.dtype = torch.float16


@dataclass
class LandmarkWalkerConfig:
    """Fields and defaults of the reference's ``LandmarkWalkerConfig``."""

    max_seq_len: int = 8192
    top_k: int = 32
    num_landmarks: int = 32
    min_spacing: int = 50
    walkers_per_source: int = 100
    query_boost: float = 2.0
    use_reachability: bool = False
    position_alpha: float = 0.6
    sink_size: int = 4
    local_window: int = 64
    device: str = "cuda"


def _keep_mask(scores: torch.Tensor, budget_ratio: float, seq_len: int, sink: int, local: int) -> torch.Tensor:
    """Sinks ``[0, sink)`` and the last ``local`` positions forced, then the largest
    remaining scores up to ``int(seq_len * budget_ratio)`` kept positions in total."""
    scores = scores[:seq_len]
    budget = int(seq_len * budget_ratio)
    keep = torch.zeros(seq_len, dtype=torch.bool, device=scores.device)
    keep[:sink] = True
    keep[max(0, seq_len - local):] = True
    remaining = max(0, budget - int(keep.sum().item()))
    if remaining > 0:
        masked = scores.clone()
        masked[keep] = float("-inf")
        keep[masked.topk(remaining).indices] = True
    return keep


class _MonitorBase:
    _graph: Optional[object]

    def _make_graph(self, top_k: int, alpha: float, num_walkers: int, num_steps: int):
        from . import get_extension
        return get_extension().CircuitGraph(self.config.max_seq_len, top_k, alpha, num_walkers, num_steps)

    def synchronize(self) -> None:
        if self._graph is not None:
            self._graph.synchronize()


class CircuitKVMonitor(_MonitorBase):
    """Capacitive charge monitor: H2O charge at the end of prefill, then an EMA of
    the circuit walker's current at every generated token."""

    def __init__(self, config: CircuitKVConfig):
        self.config = config
        self._graph = None
        self._initialized = False
        self._accumulated_charge: Optional[torch.Tensor] = None
        self._prefill_initialized = False

    def _lazy_init(self) -> None:
        if not self._initialized:
            c = self.config
            self._graph = self._make_graph(c.top_k, c.alpha, c.num_walkers, c.num_steps)
            self._initialized = True

    def initialize_from_prefill(self, attention_matrix: torch.Tensor, seq_len: Optional[int] = None) -> None:
        """Charge = H2O column sums of the prefill attention, divided by their maximum.

        Accepts column sums ``[N]``, a matrix ``[N, N]``, ``[B, H, N]`` (averaged over
        batch and heads) or ``[B, H, N, N]`` (averaged, then column-summed)."""
        self._lazy_init()
        a = attention_matrix
        if a.dim() == 1:
            h2o = a
        elif a.dim() == 2:
            h2o = a.sum(dim=0)
        elif a.dim() == 4:
            h2o = a.mean(dim=(0, 1)).sum(dim=0)
        else:
            h2o = a.mean(dim=(0, 1))
        top = h2o.max()
        if top > 0:
            h2o = h2o / top
        n = seq_len if seq_len is not None else h2o.shape[0]
        self._accumulated_charge = torch.zeros(self.config.max_seq_len, device=h2o.device, dtype=torch.float32)
        self._accumulated_charge[:n] = h2o[:n].float()
        self._prefill_initialized = True

    def update(self, query: torch.Tensor, keys: torch.Tensor, current_idx: int) -> None:
        """One generation step: circuit walk from ``current_idx`` and the charge EMA
        ``charge = decay * charge + (1 - decay) * current / max(current)``."""
        self._lazy_init()
        if query.dim() == 1:
            query = query.unsqueeze(0)
        self._graph.update_and_step_circuit(query.contiguous(), keys.contiguous(), current_idx)
        current = self._graph.get_scores()
        top = current[:current_idx + 1].max()
        norm = current / top if top > 0 else current
        if self._accumulated_charge is None:
            self._accumulated_charge = torch.zeros(self.config.max_seq_len, device=current.device,
                                                   dtype=torch.float32)
        d = self.config.decay
        self._accumulated_charge = d * self._accumulated_charge + (1 - d) * norm.float()

    def get_scores(self) -> torch.Tensor:
        self._lazy_init()
        if self._accumulated_charge is not None:
            return self._accumulated_charge
        return self._graph.get_scores()

    def get_instant_current(self) -> torch.Tensor:
        self._lazy_init()
        return self._graph.get_scores()

    def get_keep_mask(self, budget_ratio: float, seq_len: int) -> torch.Tensor:
        return _keep_mask(self.get_scores(), budget_ratio, seq_len, self.config.sink_size,
                          self.config.local_window)

    def reset(self) -> None:
        if self._graph is not None:
            self._graph.reset()
        self._accumulated_charge = None
        self._prefill_initialized = False


class LandmarkWalkerMonitor(_MonitorBase):
    """Multi-source (landmarks + query) walker monitor over a dense attention matrix."""

    def __init__(self, config: LandmarkWalkerConfig):
        self.config = config
        self._graph = None
        self._initialized = False
        self._current_scores: Optional[torch.Tensor] = None

    def _lazy_init(self) -> None:
        if not self._initialized:
            # the landmark walker ignores alpha / walkers / steps of the graph object
            self._graph = self._make_graph(self.config.top_k, 0.85, 1024, 100)
            self._initialized = True

    def update(self, attention_matrix: torch.Tensor, current_idx: int) -> None:
        self._lazy_init()
        a = attention_matrix.float() if attention_matrix.dtype != torch.float32 else attention_matrix
        c = self.config
        self._graph.update_and_step_landmark_walker(a.contiguous(), current_idx, c.num_landmarks,
                                                    c.walkers_per_source, c.query_boost, c.min_spacing,
                                                    c.position_alpha, c.use_reachability)
        self._current_scores = self._graph.get_landmark_scores()

    def get_scores(self) -> torch.Tensor:
        self._lazy_init()
        if self._current_scores is not None:
            return self._current_scores
        return torch.zeros(self.config.max_seq_len, device=self.config.device)

    def get_keep_mask(self, budget_ratio: float, seq_len: int) -> torch.Tensor:
        return _keep_mask(self.get_scores(), budget_ratio, seq_len, self.config.sink_size,
                          self.config.local_window)

    def reset(self) -> None:
        if self._graph is not None:
            self._graph.reset()
        self._current_scores = None
