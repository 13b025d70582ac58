"""``circuit_kv._C``: ``CircuitGraph`` with the reference's constructor, its
influence-walker methods (the prefill path's legacy branch) and the decode-time graph
methods behind ``CircuitKVMonitor`` (CircuitKV/csrc/pybind.cpp:44-300;
circuit_manager.cpp:26-84, 433-766, 1190-1330), on the sm_100a kernels of ``libckv.so``.

Like the reference, the object owns its buffers: the sparse attention graph
(``[max_seq_len, top_k]`` neighbours, -1 where empty, and weights), PCG states for
``num_walkers`` circuit walkers seeded once with ``seed`` and for up to 10000 influence
walkers seeded once with ``seed + 3000`` (walker w: ``pcg_init(seed, w)``), all carried
across calls, visit counts, spectral / walker / combined scores.  The landmark walkers
(``update_and_step_landmark_walker`` and the absorbing variant) raise
``NotImplementedError``.
"""

from __future__ import annotations

import torch

from .. import _lib, ops

__version__ = "4.3.0"

_INFLUENCE_MAX_WALKERS = 10000
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

    # -- landmark walkers: not built ------------------------------------------------
    def _not_here(self, *args, **kwargs):
        raise NotImplementedError("the landmark walkers of CircuitGraph are not built in this library")

    update_and_step_landmark_walker = get_landmark_scores = _not_here
    update_and_step_landmark_absorbing_walker = get_landmark_absorbing_scores = _not_here
    get_landmark_absorbing_raw_visits = get_landmark_positions = _not_here
