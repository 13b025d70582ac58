"""Full-size runs (the 32k-token Llama-3-8B layer of the headline workload, the
131k-token Mistral layer) checked through size-independent properties and against
the structured oracle."""

import numpy as np
import pytest
import torch

import ckv_oracle as O
from _golden import check_kept
from submission_folder_b200 import ops
from submission_folder_b200.cluster import CircuitKVCluster, cli_cluster_kwargs
from submission_folder_b200.synth import make_layer

pytestmark = pytest.mark.gpu


def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


@pytest.mark.parametrize("n,W,B,planted,band", [(32768, 64, 2048, 64, 256), (131072, 128, 4096, 256, 1024)])
def test_full_size_layer(n, W, B, planted, band, parity_report):
    """The 32k layer of the 32-layer cache and the 131k Mistral-shaped layer (window
    128, 256 planted keys, locality band 1024): determinism, gathered rows, and the kept
    set against the structured oracle (the reference itself cannot hold the n x n
    matrices at 131k)."""
    dev = _cuda()
    q, k, v = make_layer(n, seed=7, window=W, planted=planted, locality=band, dtype="bf16", device="cpu")
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
    # the structured oracle: exact selection on our vectors, vectors within 1e-3
    op = O.Params(window_size=W, max_capacity_prompt=B)
    r = O.update_kv(q.float().numpy(), k.float().numpy(), v.float().numpy(), 4, op, dtype="bf16")
    check_kept(f"fullsize_n{n}_w{W}", ii, sc.cpu().numpy(), r.keep_idx, r.combined, r.qi, r.hi, op, n, False,
               parity_report)


def test_ragged_batch_of_sequences(parity_report):
    """A ragged batch of 16 sequences, n_i ~ U[2048, 32768] (seeded), window 32, budget
    int(0.1 n_i), bf16, as independent units in one batched call: bit-identical to one
    call per sequence, valid kept sets, and every sequence against the structured oracle."""
    from submission_folder_b200 import sharding
    dev = _cuda()
    rng = np.random.default_rng(2024)
    lengths = rng.integers(2048, 32769, size=16).tolist()
    W = 32
    layers, params, cpu = [], [], []
    for i, n in enumerate(lengths):
        q, k, v = make_layer(n, seed=500 + i, window=W, planted=16, dtype="bf16", device="cpu")
        cpu.append((q, k, v))
        layers.append((q.to(dev), k.to(dev), v.to(dev)))
        params.append(CircuitKVCluster(**cli_cluster_kwargs(W, int(0.1 * n))).params(n))
    batched = ops.score_evict_batched(params, layers, want_scores=True)
    # the units one rank of eight would own: its slice of the batch alone gives the same results
    mine = sharding.sequences_for_rank(lengths, 3, 8)
    part = ops.score_evict_batched([params[i] for i in mine], [layers[i] for i in mine])
    torch.cuda.synchronize()
    assert ops.read_status(dev) == 0
    for j, i in enumerate(mine):
        assert torch.equal(part[j][2], batched[i][2])
    for i, n in enumerate(lengths):
        ko, vo, idx, sc = batched[i]
        assert torch.isfinite(sc).all(), (i, n)
        one = ops.score_evict(params[i], *layers[i], want_scores=True)
        for x, y in zip(one, batched[i]):
            assert torch.equal(x, y), i
        B = int(0.1 * n)
        ii = idx.cpu().numpy()
        assert len(ii) == B - W and np.all(np.diff(ii) > 0) and np.all(ii[:4] == np.arange(4)) and ii[-1] < n - W
        kd = layers[i][1]
        assert torch.equal(ko[0, : B - W], kd[0, idx.long()]) and torch.equal(ko[31, B - W:], kd[7, n - W:])
    for i in range(16):
        n, (q, k, v) = lengths[i], cpu[i]
        op = O.Params(window_size=W, max_capacity_prompt=int(0.1 * n))
        r = O.update_kv(q.float().numpy(), k.float().numpy(), v.float().numpy(), 4, op, dtype="bf16")
        check_kept(f"ragged_seq{i}_n{n}", batched[i][2].cpu().numpy(), batched[i][3].cpu().numpy(), r.keep_idx,
                   r.combined, r.qi, r.hi, op, n, False, parity_report)
