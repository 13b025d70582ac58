"""One rank of the head-sharded scoring check over NCCL (run by tests/test_tp.py under
torch.distributed.run on 2 or more GPUs): every rank scores its share of the KV heads of
one layer with ``tp.score_evict_head_sharded``; rank 0 compares the kept positions and
its heads' compressed K / V with the single-process path on all heads and writes the
verdict to the file named on the command line."""

import datetime
import json
import os
import sys

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

from submission_folder_b200 import ops, tp  # noqa: E402
from submission_folder_b200.cluster import CircuitKVCluster, cli_cluster_kwargs  # noqa: E402
from submission_folder_b200.synth import make_layer  # noqa: E402


def main():
    out_path = sys.argv[1]
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    rank, world = dist.get_rank(), dist.get_world_size()
    res = {}
    try:
        n, W, B = 8192, 64, 1024
        q, k, v = (x.to(dev) for x in make_layer(n, seed=97, window=W, planted=32, dtype="bf16"))
        p = CircuitKVCluster(**cli_cluster_kwargs(W, B)).params(n)
        hq, hk = tp.heads_for_rank(32, 8, rank, world)
        ko, vo, idx, sc = tp.score_evict_head_sharded(p, q[hq].contiguous(), k[hk].contiguous(), v[hk].contiguous())
        torch.cuda.synchronize()
        # every rank holds the same kept positions
        allidx = [torch.empty_like(idx) for _ in range(world)]
        dist.all_gather(allidx, idx)
        same = all(torch.equal(a, idx) for a in allidx)
        if rank == 0:
            k1, v1, idx1, sc1 = ops.score_evict(p, q, k, v, want_scores=True)
            torch.cuda.synchronize()
            d = set(idx.cpu().tolist()) ^ set(idx1.cpu().tolist())
            err = max(float(((a - b).abs().max() / a.abs().max()).item()) for a, b in zip(sc1, sc))
            res = {"world": world, "same_on_all_ranks": same, "differ_from_single_call": len(d),
                   "score_max_rel_err": err,
                   "kv_match": bool(torch.equal(ko, k1[hq]) and torch.equal(vo, v1[hq])) if not d else None}
            with open(out_path, "w") as f:
                json.dump(res, f)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
