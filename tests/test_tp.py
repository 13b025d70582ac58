"""Head-sharded (tensor-parallel) scoring: the host protocol of
``submission_folder_b200.tp`` over world_size-2 gloo process groups on CPU, with the
oracle as each rank's backend, against the single-process oracle on all heads; and on
the GPU, the two kernel entry points it uses (``ckv_choose_heads``,
``ckv_pool_rows_given``) with the two ranks' reductions done in one process."""

import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import ckv_oracle as O
from submission_folder_b200 import tp
from submission_folder_b200.cluster import CircuitKVCluster, cli_cluster_kwargs
from submission_folder_b200.synth import make_layer

N, W, B, G = 2048, 64, 256, 4


class OracleBackend:
    """Each rank's steps restated on the CPU (the oracle), for the protocol test."""

    def __init__(self, op, dtype):
        self.op, self.dtype = op, dtype

    def _attn(self, q, k):
        return O.window_attention(q.float().numpy(), k.float().numpy(), self.op.window_size, G, self.dtype)

    def head_stats(self, p, q, k):
        a = self._attn(q, k)
        return (torch.from_numpy(O.head_entropy(a)), torch.from_numpy(O.head_transient_mass(a, self.op.sink_size)))

    def choose_heads(self, p, ent, mass):
        ch = O.choose_heads_from(ent.numpy(), mass.numpy(), self.op)
        return ch, None

    def hi_count(self, mode):
        return float(self._hi_count)

    def pool_rows(self, p, q, k, off, ch, mode):
        a = self._attn(q, k)
        hl = a.shape[0]
        mine_q = [h - off for h in ch.qi_heads if off <= h < off + hl]
        rq = a[mine_q].max(axis=0) if mine_q else np.zeros(a.shape[1:], dtype=np.float32)
        rh = np.zeros(a.shape[1:], dtype=np.float32)
        if ch.hi_heads is not None:
            self._hi_count = len(ch.hi_heads)
            for h in ch.hi_heads:
                if off <= h < off + hl:
                    rh = (rh + a[h - off]).astype(np.float32) if ch.hi_mode == "mean" else np.maximum(rh, a[h - off])
        return torch.from_numpy(np.ascontiguousarray(rq)), torch.from_numpy(rh)

    def select(self, p, rq, rh):
        op = self.op
        n = rq.shape[1]
        rows_hi = rh.numpy() if rh is not None else rq.numpy()
        (qi, hi), _, _ = O.neumann_structured([O.Chain(rq.numpy(), "query"), O.Chain(rows_hi, "uniform")], n - 1,
                                              op.sink_size, op.neumann_iterations, op.neumann_temperature,
                                              op.neumann_gamma)
        qi = O.smooth(qi, op.qi_kernel_size, op.use_gaussian, op.gaussian_sigma * 0.5)
        hi = O.smooth(hi, op.hi_kernel_size, op.use_gaussian, op.gaussian_sigma)
        idx = O.select_from_vectors(qi, hi, op, n)
        return torch.from_numpy(idx.astype(np.int32)), torch.from_numpy(np.stack([qi, hi]))

    def gather(self, q, k, v, window, idx):
        return None, None


def _worker(rank, world, port, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        q, k, v = make_layer(N, seed=91, window=W, planted=16, dtype="bf16")
        hq, hk = tp.heads_for_rank(32, 8, rank, world)
        op = O.Params(window_size=W, max_capacity_prompt=B)
        p = CircuitKVCluster(**cli_cluster_kwargs(W, B)).params(N)
        _, _, idx, sc = tp.score_evict_head_sharded(p, q[hq], k[hk], v[hk], backend=OracleBackend(op, "bf16"))
        if rank == 0:
            torch.save({"idx": idx, "scores": sc}, out_path)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_head_sharded_protocol_two_ranks_gloo():
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "r0.pt")
        mp.start_processes(_worker, args=(2, _free_port(), out), nprocs=2, join=True, start_method="spawn")
        res = torch.load(out)
    q, k, v = make_layer(N, seed=91, window=W, planted=16, dtype="bf16")
    r = O.update_kv(q.float().numpy(), k.float().numpy(), v.float().numpy(), G,
                    O.Params(window_size=W, max_capacity_prompt=B), dtype="bf16")
    np.testing.assert_array_equal(res["idx"].numpy(), r.keep_idx)
    np.testing.assert_allclose(res["scores"][0].numpy(), r.qi, rtol=1e-5, atol=1e-8)
    np.testing.assert_allclose(res["scores"][1].numpy(), r.hi, rtol=1e-5, atol=1e-8)


def test_heads_for_rank_split():
    assert tp.heads_for_rank(32, 8, 1, 2) == (slice(16, 32), slice(4, 8))
    assert tp.heads_for_rank(32, 8, 3, 8) == (slice(12, 16), slice(3, 4))
    with pytest.raises(ValueError):
        tp.heads_for_rank(32, 8, 0, 3)


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4])
def test_head_sharded_kernels_match_single_call(world, parity_report):
    """The kernel steps of head-sharded scoring, with the ranks' all-gather / all-reduce done
    in one process: the kept positions equal the single-call path's (up to exact ties of the
    combined score), and the ranked vectors agree within 1e-5."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from submission_folder_b200 import ops
    dev = torch.device("cuda", 0)
    n, Wn, Bn = 8192, 64, 1024
    q, k, v = (x.to(dev) for x in make_layer(n, seed=93, window=Wn, planted=32, dtype="bf16"))
    p = CircuitKVCluster(**cli_cluster_kwargs(Wn, Bn)).params(n)
    _, _, idx1, sc1 = ops.score_evict(p, q, k, v, want_scores=True)
    shards = [tp.heads_for_rank(32, 8, r, world) for r in range(world)]
    stats = [ops.window_pool(p, q[hq], k[hk])[:2] for hq, hk in shards]
    ent = torch.cat([s[0] for s in stats])
    mass = torch.cat([s[1] for s in stats])
    ent1, mass1, _, _, _ = ops.window_pool(p, q, k)
    torch.testing.assert_close(ent, ent1, rtol=1e-5, atol=1e-6)
    sets, mode = ops.choose_heads(p, ent, mass)
    parts = [ops.pool_rows_given(p, q[hq], k[hk], hq.start, sets, mode) for hq, hk in shards]
    rq = torch.stack([x[0] for x in parts]).amax(0)
    rh = torch.stack([x[1] for x in parts]).sum(0) * (1.0 / mode[1:2].float())
    qi, hi, _ = ops.neumann_rows(p, rq, rh)
    idx, sc = ops.select_scores(p, qi, hi, want_scores=True)
    torch.cuda.synchronize()
    s1, s2 = sc1.cpu().numpy(), sc.cpu().numpy()
    for a, b in zip(s1, s2):
        assert np.max(np.abs(a - b)) / np.abs(a).max() < 1e-5
    op = O.Params(window_size=Wn, max_capacity_prompt=Bn)
    np.testing.assert_array_equal(O.select_from_vectors(s2[0], s2[1], op, n), idx.cpu().numpy())
    d = set(idx.cpu().numpy().tolist()) ^ set(idx1.cpu().numpy().tolist())
    parity_report[f"head_sharded_{world}_ranks"] = {"n": n, "kept": int(idx.numel()), "differ_from_single_call": len(d)}
    assert not d, sorted(d)[:10]


@pytest.mark.gpu
def test_head_sharded_over_nccl_on_two_gpus(tmp_path):
    """With two or more GPUs: two ranks (one per GPU, NCCL) score a layer's heads in halves;
    both hold the kept positions of the single-process path, and rank 0's heads' K / V are
    the single-process rows."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    out = tmp_path / "tp.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(here, "_tp_nccl_worker.py"), str(out)]
    subprocess.run(["timeout", "-k", "30", "300"] + cmd, check=True, env=env)
    import json
    res = json.loads(out.read_text())
    assert res["same_on_all_ranks"] and res["differ_from_single_call"] == 0, res
    assert res["score_max_rel_err"] < 1e-5 and res["kv_match"], res
