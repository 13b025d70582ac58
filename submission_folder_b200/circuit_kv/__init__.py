"""Mirror of the reference's ``circuit_kv`` package for the prefill eviction path.

``circuit_kv._C.CircuitGraph`` provides the constructor and the influence-walker
pair that ``CircuitKVCluster`` calls when ``use_neumann=False``
(CircuitKV/csrc/pybind.cpp:44-64, 263-300), running the sm_100a walker of
``libckv.so``.  The package-level helpers ``set_seed`` and ``get_extension`` keep
their reference behaviour (CircuitKV/circuit_kv/__init__.py, utils.py).
"""

import random

import numpy as np
import torch

from . import _C

__version__ = "3.0.0"
__all__ = ["set_seed", "get_extension"]


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
