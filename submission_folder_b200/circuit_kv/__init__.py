"""Mirror of the reference's ``circuit_kv`` package for the prefill eviction path.

``circuit_kv._C.CircuitGraph`` provides the constructor and the influence-walker
pair that ``CircuitKVCluster`` calls when ``use_neumann=False``
(CircuitKV/csrc/pybind.cpp:44-64, 263-300), running the sm_100a walker of
``libckv.so``.  The package exports the reference's names
(CircuitKV/circuit_kv/__init__.py:14-28): ``CircuitKVMonitor``, ``CircuitKVConfig``,
``LandmarkWalkerMonitor``, ``LandmarkWalkerConfig`` (``engine.py``) and ``set_seed``;
``get_extension`` keeps its reference behaviour.
"""

import random

import numpy as np
import torch

from . import _C
from .engine import CircuitKVConfig, CircuitKVMonitor, LandmarkWalkerConfig, LandmarkWalkerMonitor

__version__ = "3.0.0"
__all__ = [
    "CircuitKVMonitor",
    "CircuitKVConfig",
    "LandmarkWalkerMonitor",
    "LandmarkWalkerConfig",
    "set_seed",
]


def set_seed(seed: int) -> None:
    """Seed Python, NumPy and PyTorch (CPU and CUDA) generators (CircuitKV/circuit_kv/utils.py)."""
    random.seed(seed)
    np.random.seed(seed)
    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed(seed)
        torch.cuda.manual_seed_all(seed)
        torch.backends.cudnn.deterministic = True
        torch.backends.cudnn.benchmark = False


def get_extension():
    """The native module (here: ``circuit_kv._C`` backed by ``libckv.so``)."""
    return _C
