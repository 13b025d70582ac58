"""score_evict_pipelined: a cache held in host memory scored layer after layer with uploads,
scoring and downloads overlapped; results equal one update_kv call per layer."""

import numpy as np
import pytest
import torch

from submission_folder_b200 import ops
from submission_folder_b200.cluster import CircuitKVCluster, cli_cluster_kwargs
from submission_folder_b200.pipeline import score_evict_pipelined
from submission_folder_b200.synth import make_layer, repeat_kv

pytestmark = pytest.mark.gpu


def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def test_pipelined_equals_per_layer_calls():
    dev = _cuda()
    W, B = 64, 512
    lengths = [3000, 4100, 2600, 400, 3333]          # 400 < B: every row kept
    layers, host = [], []
    for i, n in enumerate(lengths):
        q, k, v = make_layer(n, seed=7, layer=i, window=W, dtype="bf16")
        Q, K, V = q[None], repeat_kv(k, 4), repeat_kv(v, 4)
        pin = i != 2                                     # one layer in pageable memory
        if pin:
            Q, K, V = Q.pin_memory(), K.pin_memory(), V.pin_memory()
        host.append((Q, K, V))
        layers.append((Q[0], K[0, ::4], V[0, ::4]))
    params = [CircuitKVCluster(**cli_cluster_kwargs(W, B)).params(n) for n in lengths]
    out = score_evict_pipelined(params, layers)
    assert len(out) == len(lengths)
    for i, (n, (Q, K, V)) in enumerate(zip(lengths, host)):
        cl = CircuitKVCluster(**cli_cluster_kwargs(W, B))
        kref, vref = cl.update_kv(K, Q, V, None, 4)
        ko, vo, idx = out[i]
        assert not ko.is_cuda and ko.is_pinned()
        if n < B:
            assert torch.equal(kref, K) and torch.equal(ko, K[0]) and torch.equal(vo, V[0])
            assert torch.equal(idx.cpu(), torch.arange(n - W, dtype=torch.int32))
            continue
        assert torch.equal(ko, kref[0]) and torch.equal(vo, vref[0]), i
        assert np.array_equal(idx.cpu().numpy(), cl.last_keep_indices.cpu().numpy()), i
    # again into caller-provided page-locked buffers: the same results
    bufs = [(torch.zeros_like(ko).pin_memory(), torch.zeros_like(vo).pin_memory()) for ko, vo, _ in out]
    again = score_evict_pipelined(params, layers, out=bufs)
    for (ko, vo, idx), (k2, v2, i2), (bk, bv) in zip(out, again, bufs):
        assert k2 is bk and v2 is bv
        assert torch.equal(ko, k2) and torch.equal(vo, v2) and torch.equal(idx, i2)
    assert ops.read_status(dev) == 0
