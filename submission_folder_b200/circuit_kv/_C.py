"""``circuit_kv._C``: ``CircuitGraph`` with the reference's constructor, its
influence-walker methods (the prefill path's legacy branch) and the decode-time graph
methods behind ``CircuitKVMonitor`` (CircuitKV/csrc/pybind.cpp:44-300;
circuit_manager.cpp:26-84, 433-1330), on the sm_100a kernels of ``libckv.so``.

Like the reference, the object owns its buffers: the sparse attention graph
(``[max_seq_len, top_k]`` neighbours, -1 where empty, and weights), PCG states for
``num_walkers`` circuit walkers seeded once with ``seed``, for up to 10000 influence
walkers seeded once with ``seed + 3000`` and for (32 + 1) x 500 landmark walkers seeded once
with ``seed + 1000`` or ``seed + 2000`` (whichever landmark method runs first; walker w:
``pcg_init(seed, w)``), all carried across calls, visit counts (shared by the circuit and
landmark walkers, as the reference's), spectral / walker / combined / landmark scores.
"""

from __future__ import annotations

import ctypes

import torch

from .. import _lib, ops

__version__ = "4.3.0"

_INFLUENCE_MAX_WALKERS = 10000
_LANDMARK_MAX = 32
_LANDMARK_MAX_WALKERS = (_LANDMARK_MAX + 1) * 500
_GRAPH_DTYPES = {torch.float16: 1, torch.float32: 2, torch.bfloat16: 0}


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
        # decode-time graph (circuit walker, spectral and combined scores)
        self._adj = torch.full((self.max_seq_len, self.top_k), -1, dtype=torch.int32, device=dev)
        self._adj_w = torch.zeros(self.max_seq_len, self.top_k, dtype=torch.float32, device=dev)
        self._counts = torch.zeros(self.max_seq_len, dtype=torch.int32, device=dev)
        self._circuit_rng = torch.zeros(2 * self.num_walkers, dtype=torch.int64, device=dev)
        self._spectral = torch.zeros(self.max_seq_len, dtype=torch.float32, device=dev)
        self._spectral_tmp = torch.zeros(self.max_seq_len, dtype=torch.float32, device=dev)
        self._walker_scores = torch.zeros(self.max_seq_len, dtype=torch.float32, device=dev)
        self._combined = torch.zeros(self.max_seq_len, dtype=torch.float32, device=dev)
        self._graph_scratch = torch.zeros(self.max_seq_len, dtype=torch.float32, device=dev)
        self._num_power_iterations = 10
        # landmark walkers: PCG states for (32 + 1) x 500 walkers, landmark positions and count
        self._lm_rng = torch.zeros(2 * _LANDMARK_MAX_WALKERS, dtype=torch.int64, device=dev)
        self._lm_rng_initialized = False
        self._lm_positions = torch.zeros(_LANDMARK_MAX, dtype=torch.int32, device=dev)
        self._lm_count = torch.zeros(1, dtype=torch.int32, device=dev)
        self._lm_scores = torch.zeros(self.max_seq_len, dtype=torch.float32, device=dev)
        self._lm_ws = None
        lib = _lib.load()
        _lib.check(lib.ckv_pcg_seed(int(self.seed), self.num_walkers, self._circuit_rng.data_ptr(),
                                    ops._stream(dev)), "ckv_pcg_seed")

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

    # -- decode-time graph: circuit walker, spectral and combined scores ---------
    def _graph_step(self, query: torch.Tensor, keys: torch.Tensor, current_idx: int) -> int:
        for t, nm in ((query, "query"), (keys, "keys")):
            if not t.is_cuda:
                raise RuntimeError(f"{nm} must be a CUDA tensor")
            if not t.is_contiguous():
                raise RuntimeError(f"{nm} must be contiguous")
        if query.dtype not in _GRAPH_DTYPES or keys.dtype != query.dtype:
            raise RuntimeError("Unsupported dtype. Use float16 or float32.")
        n, d = keys.shape[0], keys.shape[1]
        if not (0 <= current_idx < self.max_seq_len):
            raise RuntimeError("current_idx out of bounds")
        if n > self.max_seq_len:
            raise RuntimeError("seq_len exceeds max_seq_len")
        self._seq_len = n
        lib = _lib.load()
        _lib.check(lib.ckv_graph_update(query.data_ptr(), keys.data_ptr(), _GRAPH_DTYPES[query.dtype], n, d,
                                        int(current_idx), self.top_k, self._graph_scratch.data_ptr(),
                                        self._adj.data_ptr(), self._adj_w.data_ptr(), ops._stream(self._dev)),
                   "ckv_graph_update")
        return n

    def update_and_step_circuit(self, query: torch.Tensor, keys: torch.Tensor, current_idx: int) -> None:
        """Row ``current_idx`` of the graph from the query, then the circuit walkers from it
        (visit counts cleared first: the current of this query only)."""
        n = self._graph_step(query, keys, current_idx)
        self._counts.zero_()
        _lib.check(_lib.load().ckv_circuit_walk(self._adj.data_ptr(), self._adj_w.data_ptr(), n, self.top_k,
                                                int(current_idx), self.num_walkers, self._circuit_rng.data_ptr(),
                                                self._counts.data_ptr(), 0, ops._stream(self._dev)),
                   "ckv_circuit_walk")

    def get_scores(self) -> torch.Tensor:
        """Visit counts of the last circuit walk as floats, ``[max_seq_len]``."""
        self.synchronize()
        return self._counts.float()

    def update_and_step_circuit_combined(self, query: torch.Tensor, keys: torch.Tensor, current_idx: int,
                                         num_iterations: int = 10) -> None:
        """The graph row, the circuit walk, ``num_iterations`` power iterations, and both
        scores divided by their maxima and combined by an element-wise maximum."""
        n = self._graph_step(query, keys, current_idx)
        self._num_power_iterations = int(num_iterations)
        lib, st = _lib.load(), ops._stream(self._dev)
        _lib.check(lib.ckv_circuit_walk(self._adj.data_ptr(), self._adj_w.data_ptr(), n, self.top_k,
                                        int(current_idx), self.num_walkers, self._circuit_rng.data_ptr(),
                                        self._counts.data_ptr(), 1, st), "ckv_circuit_walk")
        _lib.check(lib.ckv_spectral_scores(self._adj.data_ptr(), self._adj_w.data_ptr(), n, self.top_k,
                                           self._num_power_iterations, self._spectral.data_ptr(),
                                           self._spectral_tmp.data_ptr(), st), "ckv_spectral_scores")
        _lib.check(lib.ckv_combine_scores(self._counts.data_ptr(), self._spectral.data_ptr(),
                                          self._walker_scores.data_ptr(), self._combined.data_ptr(), n, st),
                   "ckv_combine_scores")

    def get_combined_scores(self) -> torch.Tensor:
        self.synchronize()
        return self._combined.clone()

    def reset(self) -> None:
        self.synchronize()
        self._visits.zero_()
        self._adj.fill_(-1)
        self._counts.zero_()
        self._seq_len = 0

    def synchronize(self) -> None:
        torch.cuda.current_stream(self._dev).synchronize()

    # -- landmark walkers ----------------------------------------------------------------
    def _landmark_step(self, attention_matrix: torch.Tensor, current_idx: int, num_landmarks: int,
                       walkers_per_source: int, query_boost: float, min_spacing: int, mode: int,
                       position_alpha: float, absorb_at_landmarks: bool, seed_offset: int) -> None:
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
        if num_landmarks > _LANDMARK_MAX:
            raise RuntimeError("num_landmarks exceeds MAX_LANDMARKS")
        if (num_landmarks + 1) * walkers_per_source > _LANDMARK_MAX_WALKERS:
            raise RuntimeError("total_walkers exceeds max_landmark_walkers")
        if num_landmarks < 1:
            raise RuntimeError("num_landmarks must be at least 1")
        if walkers_per_source < 0:
            raise RuntimeError("walkers_per_source must be non-negative")
        lib, st = _lib.load(), ops._stream(self._dev)
        if self._lm_ws is None:
            sz = ctypes.c_size_t()
            _lib.check(lib.ckv_landmark_workspace_size(self.max_seq_len, ctypes.byref(sz)),
                       "ckv_landmark_workspace_size")
            self._lm_ws = torch.empty(sz.value, dtype=torch.uint8, device=self._dev)
        if not self._lm_rng_initialized:
            _lib.check(lib.ckv_pcg_seed(int(self.seed + seed_offset), _LANDMARK_MAX_WALKERS,
                                        self._lm_rng.data_ptr(), st), "ckv_pcg_seed")
            self._lm_rng_initialized = True
        self._seq_len = n
        _lib.check(lib.ckv_landmark_walk(a.data_ptr(), n, int(current_idx), mode, int(num_landmarks),
                                         int(walkers_per_source), float(query_boost), int(min_spacing),
                                         float(position_alpha), 1 if absorb_at_landmarks else 0,
                                         self._lm_rng.data_ptr(), self._counts.data_ptr(),
                                         self._lm_scores.data_ptr(), self._lm_positions.data_ptr(),
                                         self._lm_count.data_ptr(), self._lm_ws.data_ptr(), self._lm_ws.numel(), st),
                   "ckv_landmark_walk")

    def update_and_step_landmark_walker(self, attention_matrix: torch.Tensor, current_idx: int,
                                        num_landmarks: int = 32, walkers_per_source: int = 100,
                                        query_boost: float = 2.0, min_spacing: int = 50,
                                        position_alpha: float = 0.6, use_reachability: bool = False) -> None:
        """Walkers from stratified landmarks and the query; scores normalised by position
        (visits / (1 / d^alpha + 1e-8)) or, with use_reachability, by the walkers able to reach
        each position.  Landmark PCG states seeded once with seed + 1000 (shared with the
        absorbing form, whichever runs first)."""
        mode = _lib.LANDMARK_REACHABILITY if use_reachability else _lib.LANDMARK_POSITIONAL
        self._landmark_step(attention_matrix, current_idx, num_landmarks, walkers_per_source, query_boost,
                            min_spacing, mode, position_alpha, False, 1000)

    def get_landmark_scores(self) -> torch.Tensor:
        self.synchronize()
        return self._lm_scores[:self._seq_len].clone()

    def update_and_step_landmark_absorbing_walker(self, attention_matrix: torch.Tensor, current_idx: int,
                                                  num_landmarks: int = 8, walkers_per_source: int = 100,
                                                  query_boost: float = 2.0, min_spacing: int = 50,
                                                  absorb_at_landmarks: bool = True) -> None:
        """Landmarks as sources and (with probability 0.1) sinks; reachability with 0.9
        pass-through per landmark.  Landmark PCG states seeded once with seed + 2000 (shared
        with the plain landmark walker, whichever runs first)."""
        self._landmark_step(attention_matrix, current_idx, num_landmarks, walkers_per_source, query_boost,
                            min_spacing, _lib.LANDMARK_ABSORBING, 0.0, absorb_at_landmarks, 2000)

    def get_landmark_absorbing_scores(self) -> torch.Tensor:
        self.synchronize()
        return self._lm_scores[:self._seq_len].clone()

    def get_landmark_absorbing_raw_visits(self) -> torch.Tensor:
        self.synchronize()
        return self._counts[:self._seq_len].clone()

    def get_landmark_positions(self) -> torch.Tensor:
        self.synchronize()
        k = int(self._lm_count.item())
        return self._lm_positions[:max(k, 0)].clone()
