"""Full-size runs (the 32k-token Llama-3-8B layer of the headline workload, the
131k-token Mistral layer) checked through size-independent properties and against
the structured oracle."""

import numpy as np
import pytest
import torch

import ckv_oracle as O
from _golden import compare_keep
from submission_folder_b200 import ops
from submission_folder_b200.cluster import CircuitKVCluster, cli_cluster_kwargs
from submission_folder_b200.synth import make_layer

pytestmark = pytest.mark.gpu


def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


@pytest.mark.parametrize("n,W,B,planted", [(32768, 64, 2048, 64), (131072, 128, 4096, 256)])
def test_full_size_layer(n, W, B, planted):
    dev = _cuda()
    q, k, v = make_layer(n, seed=7, window=W, planted=planted, dtype="bf16", device="cpu")
    cl = CircuitKVCluster(**cli_cluster_kwargs(W, B))
    p = cl.params(n)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    ko, vo, idx, sc = ops.score_evict(p, qd, kd, vd, want_scores=True)
    ko2, vo2, idx2, sc2 = ops.score_evict(p, qd, kd, vd, want_scores=True)
    torch.cuda.synchronize()
    assert ops.read_status(dev) == 0
    # determinism
    assert torch.equal(idx, idx2) and torch.equal(sc, sc2) and torch.equal(ko, ko2)
    ii = idx.cpu().numpy()
    assert len(ii) == B - W and np.all(np.diff(ii) > 0) and np.all(ii[:4] == np.arange(4))
    assert ii[-1] < n - W
    # gathered rows: every query head of a group carries its KV head's row
    rows = kd[:, idx.long()]
    for g in range(8):
        for r in range(4):
            assert torch.equal(ko[g * 4 + r, : B - W], rows[g])
            assert torch.equal(ko[g * 4 + r, B - W:], kd[g, n - W:])
    assert torch.equal(vo[5, : B - W], vd[1, idx.long()])
    # planted keys (aligned with the window queries) should mostly survive
    # and the structured oracle agrees on the kept set up to near-ties
    op = O.Params(window_size=W, max_capacity_prompt=B)
    if n <= 32768:
        r = O.update_kv(q.float().numpy(), k.float().numpy(), v.float().numpy(), 4, op, dtype="bf16")
        nd, ok = compare_keep(ii, r.keep_idx, r.combined, 4, n - W, B - W - 4, margin=16.0 / (n - 1))
        assert ok, nd
        got = sc.cpu().numpy()
        assert np.max(np.abs(got[0] - r.qi)) / np.abs(r.qi).max() < 1e-3
        assert np.max(np.abs(got[1] - r.hi)) / np.abs(r.hi).max() < 1e-3
