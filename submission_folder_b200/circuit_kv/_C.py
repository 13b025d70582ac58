"""``circuit_kv._C`` for the prefill eviction path: ``CircuitGraph`` with the
reference's constructor and influence-walker methods (CircuitKV/csrc/pybind.cpp:44-64,
263-300; circuit_manager.cpp:26-84, 562-590, 1190-1330), on the sm_100a walker of
``libckv.so``.

Like the reference, the object owns the walker buffers: PCG states for up to 10000
walkers, seeded once with ``seed + 3000`` (walker w: ``pcg_init(seed + 3000, w)``)
and carried across calls, the raw visit counts and the normalised scores.  Methods of
the decode-time monitors (circuit / landmark walkers, spectral scoring) are not part of
this path and raise ``NotImplementedError``.
"""

from __future__ import annotations

import torch

from .. import _lib, ops

__version__ = "4.3.0"

_INFLUENCE_MAX_WALKERS = 10000


class CircuitGraph:
    def __init__(self, max_seq_len: int, top_k: int, alpha: float, num_walkers: int, num_steps: int,
                 query_window: int = 64, seed: int = 42):
        if not max_seq_len > 0:
            raise RuntimeError("max_seq_len must be positive")
        if not (0 < top_k <= 64):
            raise RuntimeError("top_k must be in (0, 64]")
        if not num_walkers > 0:
            raise RuntimeError("num_walkers must be positive")
        if not torch.cuda.is_available():
            raise RuntimeError("CircuitGraph needs a CUDA device")
        self.max_seq_len = int(max_seq_len)
        self.top_k, self.alpha, self.num_walkers, self.num_steps = top_k, alpha, num_walkers, num_steps
        self.query_window, self.seed = query_window, int(seed)
        self.rng_mode = _lib.RNG_PCG          # CircuitGraph-compatible generator; _lib.RNG_PHILOX also works
        dev = torch.device("cuda", torch.cuda.current_device())
        self._dev = dev
        self._rng_state = torch.zeros(2 * _INFLUENCE_MAX_WALKERS, dtype=torch.int64, device=dev)
        self._rng_initialized = False
        self._visits = torch.zeros(self.max_seq_len, dtype=torch.float32, device=dev)
        self._scores = torch.zeros(self.max_seq_len, dtype=torch.float32, device=dev)
        self._seq_len = 0

    # -- influence walker (the prefill path) -------------------------------------
    def update_and_step_influence_walker(self, attention_matrix: torch.Tensor, current_idx: int,
                                         num_walkers: int = 10000, max_steps: int = 10, sink_size: int = 4,
                                         temperature: float = 2.0, explore_temp: float = 10.0,
                                         explore_ratio: float = 0.3) -> None:
        a = attention_matrix
        if not a.is_cuda:
            raise RuntimeError("attention_matrix must be a CUDA tensor")
        if not a.is_contiguous():
            raise RuntimeError("attention_matrix must be contiguous")
        if a.dtype != torch.float32:
            raise RuntimeError("attention_matrix must be float32")
        if a.dim() != 2:
            raise RuntimeError("attention_matrix must be 2D [seq_len, seq_len]")
        n = a.shape[0]
        if a.shape[1] != n:
            raise RuntimeError("attention_matrix must be square")
        if not (0 <= current_idx < n):
            raise RuntimeError("current_idx out of bounds")
        if n > self.max_seq_len:
            raise RuntimeError("seq_len exceeds max_seq_len")
        if num_walkers > _INFLUENCE_MAX_WALKERS:
            raise RuntimeError("num_walkers exceeds influence_max_walkers")
        self._seq_len = n
        ops.influence_walk_dense(a, int(current_idx), int(num_walkers), int(max_steps), int(sink_size),
                                 float(temperature), float(explore_temp), float(explore_ratio),
                                 rng_mode=self.rng_mode, seed=self.seed + 3000, rng_state=self._rng_state,
                                 init_state=not self._rng_initialized, visits=self._visits[:n],
                                 scores=self._scores[:n])
        self._rng_initialized = True

    def get_influence_scores(self) -> torch.Tensor:
        self.synchronize()
        return self._scores[:self._seq_len].clone()

    def get_influence_raw_visits(self) -> torch.Tensor:
        self.synchronize()
        return self._visits[:self._seq_len].clone()

    def reset(self) -> None:
        self.synchronize()
        self._visits.zero_()
        self._seq_len = 0

    def synchronize(self) -> None:
        torch.cuda.current_stream(self._dev).synchronize()

    # -- decode-time monitor methods: not on the prefill eviction path ------------
    def _not_here(self, *args, **kwargs):
        raise NotImplementedError("decode-time monitor method: not part of the prefill eviction path")

    update_and_step_circuit = get_scores = update_and_step_circuit_combined = get_combined_scores = _not_here
    update_and_step_landmark_walker = get_landmark_scores = _not_here
    update_and_step_landmark_absorbing_walker = get_landmark_absorbing_scores = _not_here
    get_landmark_absorbing_raw_visits = get_landmark_positions = _not_here
