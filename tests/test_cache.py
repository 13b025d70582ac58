"""Decode-side cache with distinct KV heads (``submission_folder_b200.cache``) and the
hook's ``distinct_kv_heads`` output (each KV head written once)."""

import numpy as np
import pytest
import torch

from submission_folder_b200.cache import DistinctKVCache
from submission_folder_b200.synth import repeat_kv


def test_cache_keeps_distinct_heads():
    torch.manual_seed(0)
    k, v = torch.randn(8, 100, 128), torch.randn(8, 100, 128)
    K, V = repeat_kv(k, 4), repeat_kv(v, 4)            # the reference's layout, 32 heads
    c = DistinctKVCache(8, 4)
    ko, vo = c.update(K, V, 0)
    assert ko.shape == (1, 8, 100, 128) and torch.equal(ko[0], k) and torch.equal(vo[0], v)
    # a decode step: one token, repeated heads again
    k1, v1 = torch.randn(8, 1, 128), torch.randn(8, 1, 128)
    ko, vo = c.update(repeat_kv(k1, 4), repeat_kv(v1, 4), 0)
    assert ko.shape == (1, 8, 101, 128) and torch.equal(ko[0, :, -1:], k1)
    assert c.get_seq_length(0) == 101 and c.get_usable_length(1, 0) == 101 and c._seen_tokens == 101
    assert c.nbytes() == 2 * 8 * 101 * 128 * 4           # a quarter of the repeated cache
    # inputs already distinct (CircuitKVCluster(distinct_kv_heads=True)) are stored as they are
    c2 = DistinctKVCache(8, 4, repeat=True)
    c2.update(k[None], v[None], 0)
    kr, vr = c2.update(repeat_kv(k1, 4), repeat_kv(v1, 4), 0)
    assert kr.shape == (1, 32, 101, 128)
    assert torch.equal(kr, repeat_kv(torch.cat([k, k1], dim=1), 4))
    # layers held elsewhere (pipeline / layer sharding) stay empty
    c3 = DistinctKVCache(8, 4)
    c3.update(K, V, 2)
    assert len(c3) == 3 and c3.get_seq_length(0) == 0 and c3.get_seq_length(2) == 100
    with pytest.raises(ValueError):
        c3.update(torch.zeros(1, 5, 1, 128), torch.zeros(1, 5, 1, 128), 2)


@pytest.mark.gpu
def test_hook_distinct_kv_heads_output():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from submission_folder_b200.cluster import CircuitKVCluster, cli_cluster_kwargs
    from submission_folder_b200.synth import make_layer
    dev = torch.device("cuda", 0)
    n, W, B = 4096, 64, 512
    q, k, v = make_layer(n, seed=17, window=W, planted=16, dtype="bf16")
    K, V, Q = repeat_kv(k, 4).to(dev), repeat_kv(v, 4).to(dev), q[None].to(dev)
    full = CircuitKVCluster(**cli_cluster_kwargs(W, B))
    ko, vo = full.update_kv(K, Q, V, None, 4)
    dist = CircuitKVCluster(**cli_cluster_kwargs(W, B), distinct_kv_heads=True)
    kd, vd = dist.update_kv(K, Q, V, None, 4)
    torch.cuda.synchronize()
    assert kd.shape == (1, 8, B, 128) and vd.shape == (1, 8, B, 128)
    assert torch.equal(kd, ko[:, ::4]) and torch.equal(vd, vo[:, ::4])
    assert torch.equal(dist.last_keep_indices, full.last_keep_indices)
    cache = DistinctKVCache(8, 4)
    kc, vc = cache.update(kd, vd, 0)
    assert torch.equal(kc, kd) and cache.nbytes() * 4 == ko.numel() * 2 * 2
