"""Generate the golden fixtures from the reference implementation itself.

Runs KVCache-Factory's own ``CircuitKVCluster.update_kv`` (imported unmodified
from the reference checkout) on seeded synthetic inputs and records, per case:
the kept prefix positions, the QI / HI vectors returned by
``_compute_dual_importance_scores`` (or the influence / H2O pair), the combined
scores handed to ``_get_keep_mask``, the per-head entropy / transient mass and
a checksum of the returned K.  Inputs are not stored: they are regenerated from
the recorded seed by ``submission_folder_b200.synth.make_layer`` (CPU generator,
deterministic for a given torch build).

Usage (in a checkout that has the reference source; its root is given by --ref or
the CKV_REFERENCE_ROOT environment variable -- there is no default):
    python tests/golden/make_golden.py --ref /path/to/reference [--only NAME]

``--only`` regenerates the matching cases and merges them into ``cases.json``.
Each case also records the wall time of the reference's ``update_kv`` call and
the host threads it used (``ref_seconds``, ``ref_threads``).
"""

from __future__ import annotations

import argparse
import contextlib
import io
import json
import math
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from submission_folder_b200.cluster import cli_cluster_kwargs  # noqa: E402
from submission_folder_b200.synth import make_layer, repeat_kv  # noqa: E402

# (name, n, dtype, W, B, planted, qk_scale, seed, overrides)
CASES = [
    ("cfg1_fp32_n4096", 4096, "fp32", 32, 512, 16, 1.0, 11, {}),
    ("bf16_n2048_default", 2048, "bf16", 64, 256, 16, 1.0, 12, {}),
    ("fp16_n2048_w32", 2048, "fp16", 32, 256, 16, 1.0, 13, {}),
    ("bf16_literal_scale", 2048, "bf16", 64, 256, 16, 1.0 / math.sqrt(128), 14, {}),
    ("bf16_max", 2048, "bf16", 64, 256, 16, 1.0, 15, {"combination_mode": "max"}),
    ("bf16_weighted", 2048, "bf16", 64, 256, 16, 1.0, 16, {"combination_mode": "weighted"}),
    ("bf16_union", 2048, "bf16", 64, 256, 16, 1.0, 17, {"combination_mode": "union"}),
    ("bf16_union_da", 2048, "bf16", 64, 256, 16, 1.0, 18, {"combination_mode": "union_da"}),
    ("bf16_no_entropy", 2048, "bf16", 64, 256, 16, 1.0, 19, {"entropy_aware": False}),
    ("bf16_bridge", 2048, "bf16", 64, 256, 16, 1.0, 20, {"use_bridge_importance": True}),
    ("bf16_temp07", 2048, "bf16", 64, 256, 16, 1.0, 21, {"neumann_temperature": 0.7}),
    ("bf16_gamma09", 2048, "bf16", 64, 256, 16, 1.0, 22, {"neumann_gamma": 0.9}),
    ("bf16_mass_sel", 2048, "bf16", 64, 256, 16, 1.0, 23, {"head_selection_mode": "mass"}),
    ("bf16_hi_max", 2048, "bf16", 64, 256, 16, 1.0, 24, {"hi_pooling_mode": "max"}),
    ("bf16_hi_topk", 2048, "bf16", 64, 256, 16, 1.0, 25, {"hi_top_k_heads": 6}),
    ("bf16_hi_cdf", 2048, "bf16", 64, 256, 16, 1.0, 26, {"hi_mass_cdf": 0.85}),
    ("bf16_ablate_qi", 2048, "bf16", 64, 256, 16, 1.0, 27, {"ablate_qi": True}),
    ("bf16_ablate_hi", 2048, "bf16", 64, 256, 16, 1.0, 28, {"ablate_hi": True}),
    ("bf16_boxcar5", 2048, "bf16", 64, 256, 16, 1.0, 29,
     {"smoothing_kernel": 5, "qi_kernel_size": 0, "hi_kernel_size": 0, "use_gaussian": False}),
    ("bf16_iters3", 2048, "bf16", 64, 256, 16, 1.0, 30, {"neumann_iterations": 3}),
    ("bf16_sink8", 2048, "bf16", 64, 256, 16, 1.0, 31, {"sink_size": 8}),
    ("bf16_w128", 2048, "bf16", 128, 384, 32, 1.0, 32, {}),
    ("bf16_perhead", 2048, "bf16", 64, 256, 16, 1.0, 33, {"per_head_eviction": True}),
    ("bf16_perhead_hub", 2048, "bf16", 64, 256, 16, 1.0, 34,
     {"per_head_eviction": True, "true_hub_hi": True}),
    ("bf16_n8192_cfg2", 8192, "bf16", 64, 1024, 64, 1.0, 35, {}),
    # the 32k layer of the 32-layer cache (window 64, budget 2048, 64 planted keys per
    # head), once with unit-variance logits and once with the literal N(0,1)/sqrt(128)
    # components; and per-head eviction at 8k
    ("cfg3_bf16_n32768", 32768, "bf16", 64, 2048, 64, 1.0, 36, {}),
    ("cfg3_literal_n32768", 32768, "bf16", 64, 2048, 64, 1.0 / math.sqrt(128), 37, {}),
    ("bf16_perhead_n8192", 8192, "bf16", 64, 1024, 64, 1.0, 38, {"per_head_eviction": True}),
    # exact-arithmetic inputs (Q, K on a 0.25 grid): the logits are the same bits on every
    # device, so the GPU's kept sets are compared with these without any allowance
    ("grid_bf16_n2048", 2048, "bf16", 64, 256, 16, 1.0, 40, {}),
    ("grid_fp32_n4096_w32", 4096, "fp32", 32, 512, 16, 1.0, 41, {}),
    ("grid_bf16_n8192", 8192, "bf16", 64, 1024, 64, 1.0, 42, {}),
    ("grid_bf16_union", 2048, "bf16", 64, 256, 16, 1.0, 43, {"combination_mode": "union"}),
    ("grid_bf16_w128", 2048, "bf16", 128, 384, 32, 1.0, 44, {}),
    ("grid_bf16_perhead", 2048, "bf16", 64, 256, 16, 1.0, 45, {"per_head_eviction": True}),
    ("grid_bf16_n32768", 32768, "bf16", 64, 2048, 64, 1.0, 46, {}),
]

GRID_STEP = 0.25   # cases whose name starts with "grid_"


def run_case(CircuitKVCluster, case):
    name, n, dtype, W, B, planted, scale, seed, over = case
    grid = GRID_STEP if name.startswith("grid_") else 0.0
    q, k, v = make_layer(n, seed=seed, window=W, planted=planted, qk_scale=scale, dtype=dtype, grid_step=grid)
    kw = cli_cluster_kwargs(W, B, **over)
    cl = CircuitKVCluster(**kw)
    rec = {}
    orig = {}

    def wrap(attr, store):
        fn = getattr(cl, attr)
        orig[attr] = fn

        def inner(*a, **k):
            out = fn(*a, **k)
            store(a, k, out)
            return out
        setattr(cl, attr, inner)

    wrap("_compute_head_entropy", lambda a, k, o: rec.setdefault("entropy", o.float().numpy()))
    wrap("_compute_head_transient_mass", lambda a, k, o: rec.setdefault("mass", o.float().numpy()))
    wrap("_compute_dual_importance_scores",
         lambda a, k, o: rec.update(qi=o[0].numpy().copy(), hi=o[1].numpy().copy()))
    wrap("_compute_influence_neumann", lambda a, k, o: rec.update(influence=o.numpy().copy()))
    wrap("_get_keep_mask", lambda a, k, o: rec.update(combined=a[0].numpy().copy(),
                                                       mask=o.numpy().copy()))
    wrap("_get_union_keep_mask", lambda a, k, o: rec.update(union_qi=a[0].numpy().copy(),
                                                             union_hi=a[1].numpy().copy(),
                                                             mask=o.numpy().copy()))
    K, Q, V = repeat_kv(k, 4), q[None], repeat_kv(v, 4)
    with contextlib.redirect_stdout(io.StringIO()):
        t0 = time.perf_counter()
        ko, vo = cl.update_kv(K, Q, V, None, 4)
        secs = time.perf_counter() - t0
    del K, V
    ko = ko[0].float().numpy()
    out = {"k_checksum": np.float64(ko.astype(np.float64).sum())}
    if over.get("per_head_eviction"):
        # recover the per-head index sets from the returned rows
        kk = np.repeat(k.float().numpy(), 4, axis=0)
        idx = []
        for h in range(ko.shape[0]):
            lut = {kk[h, j].tobytes(): j for j in range(n)}
            idx.append([lut[ko[h, i].tobytes()] for i in range(ko.shape[1] - W)])
        out["keep_per_head"] = np.array(idx, dtype=np.int32)
    else:
        mask = rec["mask"].copy()
        mask[n - W:] = False
        out["keep"] = np.nonzero(mask)[0].astype(np.int32)
    for key in ("entropy", "mass", "qi", "hi", "influence", "combined", "union_qi", "union_hi"):
        if key in rec:
            out[key] = rec[key].astype(np.float32)
    meta = {"name": name, "n": n, "dtype": dtype, "window": W, "budget": B, "planted": planted,
            "qk_scale": scale, "seed": seed, "grid_step": grid, "overrides": over, "kwargs": kw,
            "ref_seconds": round(secs, 3), "ref_threads": torch.get_num_threads()}
    return meta, out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("CKV_REFERENCE_ROOT"))
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    if not args.ref:
        ap.error("give the reference checkout with --ref or CKV_REFERENCE_ROOT")
    sys.path.insert(0, os.path.join(args.ref, "KVCache-Factory"))
    from pyramidkv.pyramidkv_utils import CircuitKVCluster  # the reference, unmodified
    torch.set_num_threads(max(1, len(os.sched_getaffinity(0))))
    index = []
    for case in CASES:
        if args.only and args.only not in case[0]:
            continue
        meta, out = run_case(CircuitKVCluster, case)
        np.savez_compressed(os.path.join(HERE, meta["name"] + ".npz"), **out)
        index.append(meta)
        print(meta["name"], "kept", len(out.get("keep", out.get("keep_per_head", []))))
    path = os.path.join(HERE, "cases.json")
    if args.only and os.path.exists(path):
        with open(path) as f:
            old = json.load(f)["cases"]
        fresh = {m["name"]: m for m in index}
        names = [c[0] for c in CASES]
        merged = {c["name"]: c for c in old}
        merged.update(fresh)
        index = [merged[nm] for nm in names if nm in merged]
    meta_info = {"torch": torch.__version__, "generator": "tests/golden/make_golden.py",
                 "reference": "KVCache-Factory/pyramidkv/pyramidkv_utils.py CircuitKVCluster.update_kv",
                 "cases": index}
    with open(path, "w") as f:
        json.dump(meta_info, f, indent=1)


if __name__ == "__main__":
    main()
