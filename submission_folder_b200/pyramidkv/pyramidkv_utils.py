"""Mirror of ``pyramidkv.pyramidkv_utils`` for the CircuitKV method: the cluster and its init hook.

``from submission_folder_b200.pyramidkv.pyramidkv_utils import CircuitKVCluster, init_circuitkv``
replaces the reference import of the same names.
"""

from ..cluster import CircuitKVCluster, init_circuitkv  # noqa: F401
