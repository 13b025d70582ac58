"""B200-native CircuitKV prefill scoring + eviction.

Drop-in for KVCache-Factory's ``CircuitKVCluster.update_kv`` hook
(``pyramidkv/pyramidkv_utils.py``) and the ``circuit_kv`` package API, running
hand-written sm_100a CUDA kernels through the C ABI in ``include/ckv.h``.
"""

from .cluster import CircuitKVCluster, cli_cluster_kwargs, init_circuitkv  # noqa: F401

__version__ = "0.1.0"
