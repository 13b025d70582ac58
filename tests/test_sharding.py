"""Multi-rank host logic on CPU: unit assignment over ranks and the one collective
(all-gather of kept positions), run as world_size-2 gloo process groups; each rank
scores its own units with the oracle (the GPU path is the same host code over NCCL)."""

import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from submission_folder_b200 import sharding

LENGTHS = [700, 300, 900, 450, 450, 620]


def test_layers_round_robin():
    for world in (1, 2, 4, 8):
        parts = [sharding.layers_for_rank(32, r, world) for r in range(world)]
        assert sorted(sum(parts, [])) == list(range(32))
        assert all(len(p) == 32 // world for p in parts)
    with pytest.raises(ValueError):
        sharding.layers_for_rank(4, 2, 2)


def test_sequences_balanced_partition():
    rng = np.random.default_rng(0)
    lengths = rng.integers(2048, 32769, size=16).tolist()
    for world in (1, 2, 4, 8):
        parts = [sharding.sequences_for_rank(lengths, r, world) for r in range(world)]
        assert sorted(sum(parts, [])) == list(range(16))
        loads = [sum(lengths[i] for i in p) for p in parts]
        # longest-first greedy: within the largest sequence of the optimum
        assert max(loads) - min(loads) <= max(lengths)
        assert max(loads) <= sum(lengths) / world + max(lengths)


def test_pack_round_trip():
    local = {3: torch.tensor([0, 1, 5, 9], dtype=torch.int32),
             7: torch.arange(12, dtype=torch.int32).reshape(3, 4),
             8: torch.arange(5, dtype=torch.int32).reshape(1, 5),
             1: torch.zeros(0, dtype=torch.int32)}
    out = {}
    sharding._unpack(sharding._pack(local), out)
    assert set(out) == {1, 3, 7, 8}
    for u in (3, 7, 8):
        assert torch.equal(out[u], local[u])
    assert out[1].numel() == 0


def _oracle_keep(i):
    import ckv_oracle as O
    from submission_folder_b200.synth import make_layer
    n = LENGTHS[i]
    q, k, v = make_layer(n, seed=40 + i, window=32, planted=8, dtype="fp32", device="cpu")
    p = O.Params(window_size=32, max_capacity_prompt=n // 4, per_head_eviction=(i == 2))
    r = O.update_kv(q.numpy(), k.numpy(), v.numpy(), 4, p, dtype="fp32")
    return torch.from_numpy(np.asarray(r.keep_idx, dtype=np.int32))


def _worker(rank, world, port, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    for p in (os.path.dirname(here), os.path.join(os.path.dirname(here), "oracle")):
        sys.path.insert(0, p)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        mine = sharding.sequences_for_rank(LENGTHS, rank, world)
        local = {i: _oracle_keep(i) for i in mine}
        allk = sharding.gather_kept(local)
        slowest = sharding.max_over_ranks(float(rank + 1))
        # the fixed-size exchange: shapes and owners known to every rank up front
        shapes = {i: ((32, n // 4 - 32) if i == 2 else (n // 4 - 32,)) for i, n in enumerate(LENGTHS)}
        owner = {i: r for r in range(world) for i in sharding.sequences_for_rank(LENGTHS, r, world)}
        ex = sharding.KeptExchange(shapes, owner, rank, world)
        assert ex.units_of(rank) == mine
        for i in mine:
            ex.out(i).copy_(local[i])
        ex.exchange()
        fixed = {i: ex.result(i).clone() for i in range(len(LENGTHS))}
        if rank == 0:
            torch.save({"kept": allk, "fixed": fixed, "slowest": slowest, "mine": mine}, out_path)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_gloo_ranks_gather_kept(world):
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "r0.pt")
        mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, join=True,
                           start_method="spawn")
        res = torch.load(out)
    assert res["slowest"] == float(world)
    kept = res["kept"]
    assert sorted(kept) == list(range(len(LENGTHS)))
    for i in range(len(LENGTHS)):
        assert torch.equal(kept[i], _oracle_keep(i)), i
        assert torch.equal(res["fixed"][i], kept[i]), i
    assert kept[2].dim() == 2 and kept[0].dim() == 1       # per-head unit keeps its [H, kept] shape
