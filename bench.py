#!/usr/bin/env python3
"""Benchmark of the CircuitKV prefill scoring + eviction path on B200.

Workload (one "step"): score and evict every layer of a Llama-3-8B-shaped
prefill cache -- 32 layers x 32 query / 8 KV heads, head_dim 128, bf16,
32768 tokens, observation window 64, budget 2048 per layer (``--pyramid``: the
budget falls linearly from 4096 at layer 0 to 512 at layer 31).  The timed step
is one ``ckv_score_evict_batched`` call over the 32 layers (each layer with the
semantics of CircuitKVCluster.update_kv; the library runs the layers on four
concurrent lanes) on device-resident inputs, captured in one CUDA graph.  The
per-stage breakdown and the roofline of the dominant kernel come from the serial
form of the step (one ``ckv_score_evict`` call per layer), timed separately.
Inputs are seeded synthetic tensors (``submission_folder_b200.synth``).

``value`` = tokens scored per second over all ranks (layers x tokens per step /
step time, max over ranks).  ``e2e`` = the same metric through the public hook
(``CircuitKVCluster.update_kv``) with pinned host buffers: the host->device copy
of each layer's window queries and distinct K / V heads and the device->host copy
of the compressed K / V are inside its timed region.

Multi-GPU: one process per GPU (torchrun); every rank scores its own 32-layer
cache (weak scaling), then the kept-index metadata of all ranks is all-gathered
over NCCL (the only collective).  ``--impl reference`` times the CPU oracle port
of the reference's path on the host cores (rank 0 only).
"""

from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

MEASURED = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
METRIC = "tokens scored/s (per-layer CircuitKV scoring+eviction, 32-layer Llama-3-8B cache, 32k ctx)"
STAGES = ["window_moments", "window_pool", "pool_reduce", "window_pool_rerun", "sweep_maps",
          "sweep_terms", "aux", "select", "gather"]


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--n", type=int, default=32768)
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--window", type=int, default=64)
    ap.add_argument("--budget", type=int, default=2048)
    ap.add_argument("--pyramid", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=3)
    return ap.parse_args()


def peaks():
    try:
        with open(MEASURED) as f:
            m = json.load(f)
        return {"hbm_gbs": float(m["hbm_gbs"]), "bf16_tflops": float(m["bf16_tflops"]),
                "bf16_tflops_sustained": float(m.get("bf16_tflops_sustained", m["bf16_tflops"])),
                "source": "measured"}
    except Exception:
        d = dict(FALLBACK_PEAKS)
        d["bf16_tflops_sustained"] = 1400.0
        d["source"] = "fallback"
        return d


def budgets(args):
    if args.pyramid:
        L = args.layers
        return [int(round(4096 - 3584 * l / max(1, L - 1))) for l in range(L)]
    return [args.budget] * args.layers


def layer_bytes(n, W, B, e=2, H=32, Hkv=8, D=128):
    """Algorithmic bytes of one layer call: K read once (distinct heads), window Q,
    kept K/V read, compacted K/V written."""
    return e * (Hkv * n * D + H * W * D + 2 * Hkv * B * D + 2 * H * B * D)


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.out = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.out,
                stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.out.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx.append(float(parts[2]))
                except ValueError:
                    continue
                for nm, val in zip(names, parts[5:9]):
                    if val.lower() == "active":
                        reasons.add(nm)
        os.unlink(self.path)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "samples": len(sm),
                "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------
# CPU oracle (baseline / reference arm)
# ---------------------------------------------------------------------------
def cpu_oracle_sample(args, seconds_cap=30.0):
    """The oracle port on the host cores: one full layer of the workload per sample."""
    import numpy as np
    import torch
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import ckv_oracle as O
    from submission_folder_b200.synth import make_layer
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    q, k, v = make_layer(args.n, seed=0, window=args.window, planted=64, dtype="bf16")
    qn, kn, vn = (x.float().numpy() for x in (q, k, v))
    p = O.Params(window_size=args.window, max_capacity_prompt=budgets(args)[0])
    times = []
    t_all = time.perf_counter()
    while True:
        t0 = time.perf_counter()
        O.update_kv(qn, kn, vn, 4, p, dtype="bf16", solver="structured")
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_all > seconds_cap or len(times) >= 3:
            break
    t = statistics.median(times)
    return {"value": args.n / t, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{len(times)} x one {args.n}-token layer (structured numpy restatement of the "
                      f"reference path), median {t:.2f} s/layer"}


def workload_config(args, world):
    """The ``config`` object of both arms' JSON lines."""
    bl = budgets(args)
    return {"workload": "32-layer Llama-3-8B cache, 32 q / 8 kv heads, head_dim 128, bf16, "
                        f"n={args.n}, window {args.window}, budget "
                        f"{'pyramid 4096->512' if args.pyramid else bl[0]}",
            "layers": args.layers, "n": args.n, "window": args.window,
            "budget": "pyramid" if args.pyramid else bl[0],
            "parallelism": f"layers of one cache per rank, {world} rank(s)",
            "l2": "inputs larger than L2 (32 x 64 MiB distinct K per step)"}


def run_reference(args, rank):
    if rank != 0:
        return
    cpu = cpu_oracle_sample(args)
    line = {"impl": "reference", "metric": METRIC, "value": cpu["value"], "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic", "config": workload_config(args, args.gpus),
            "cpu_baseline": cpu,
            "e2e": {"value": cpu["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args, rank, world):
    import torch
    import torch.distributed as dist
    from submission_folder_b200 import _lib, ops
    from submission_folder_b200.cluster import CircuitKVCluster, cli_cluster_kwargs
    from submission_folder_b200.synth import make_layer, repeat_kv

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    lib = _lib.load()
    n, W, L = args.n, args.window, args.layers
    bl = budgets(args)
    H, Hkv, D, G = 32, 8, 128, 4

    # ---- inputs: the caller's layout ([1,32,n,128] Q and repeat_kv'd K / V) ----
    Q, K, V = [], [], []
    for l in range(L):
        q, k, v = make_layer(n, seed=1000 * rank + 1, layer=l, window=W, planted=64, dtype="bf16",
                             device=str(dev))
        Q.append(q[None])
        K.append(repeat_kv(k, G))
        V.append(repeat_kv(v, G))
        del q, k, v
    torch.cuda.synchronize()

    params, structs, outs, idxs = [], [], [], []
    ws_size, ws_total = 0, 0
    for l in range(L):
        cl = CircuitKVCluster(**cli_cluster_kwargs(W, bl[l]))
        p = cl.params(n)
        params.append(p)
        one = ops.workspace_size(p, n, H, Hkv, D)
        ws_size = max(ws_size, one)
        ws_total += (one + 255) // 256 * 256
    # one workspace slice per layer: the batched call runs the layers concurrently
    ws = torch.empty(ws_total, dtype=torch.uint8, device=dev)
    for l in range(L):
        lay = ops.make_layer(Q[l][0], K[l][0, ::G], V[l][0, ::G])
        olen = ops.output_len(params[l], n)
        ko = torch.empty(H, olen, D, dtype=torch.bfloat16, device=dev)
        vo = torch.empty(H, olen, D, dtype=torch.bfloat16, device=dev)
        idx = torch.empty(olen - W, dtype=torch.int32, device=dev)
        o = _lib.Outputs()
        o.out_k, o.out_v, o.out_idx, o.out_scores = ko.data_ptr(), vo.data_ptr(), idx.data_ptr(), None
        structs.append(lay)
        outs.append((o, ko, vo))
        idxs.append(idx)
    wsp = ctypes.c_void_p(ws.data_ptr())

    nev = len(STAGES) + 1
    events = [[torch.cuda.Event(enable_timing=True) for _ in range(nev)] for _ in range(L)]
    for row in events:
        for e in row:
            e.record()
    torch.cuda.synchronize()
    ev_arrays = [(ctypes.c_void_p * nev)(*[e.cuda_event for e in row]) for row in events]

    P_arr = (_lib.Params * L)(*params)
    L_arr = (_lib.Layer * L)(*structs)
    O_arr = (_lib.Outputs * L)(*[o[0] for o in outs])

    def step_serial(with_events=True):
        """One ckv_score_evict call per layer; per-stage event records (graph capture only)."""
        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        for l in range(L):
            if with_events:
                lib.ckv_set_stage_events(ev_arrays[l], nev)
            rc = lib.ckv_score_evict(ctypes.byref(params[l]), ctypes.byref(structs[l]), wsp, ws_size,
                                     ctypes.byref(outs[l][0]), st)
            if rc != 0:
                raise RuntimeError(lib.ckv_last_error_string().decode())
        lib.ckv_set_stage_events(None, 0)

    def step():
        """The timed step: every layer in one batched call (concurrent lanes)."""
        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        rc = lib.ckv_score_evict_batched(P_arr, L, L_arr, L, wsp, ws.numel(), O_arr, st)
        if rc != 0:
            raise RuntimeError(lib.ckv_last_error_string().decode())

    def capture(fn):
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                fn()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        return g

    # eager warm-up (kernel attributes and the library's lanes are set up on first
    # use), then capture both forms of the step
    step()
    step_serial(with_events=False)
    torch.cuda.synchronize()
    graph_serial = capture(step_serial)
    graph = capture(step)

    # per-stage breakdown from the serial form (not the timed region)
    for _ in range(2):
        graph_serial.replay()
    torch.cuda.synchronize()
    stage_ms = [0.0] * (nev - 1)
    for l in range(L):
        for i in range(nev - 1):
            stage_ms[i] += events[l][i].elapsed_time(events[l][i + 1])
    t0s = torch.cuda.Event(enable_timing=True)
    t1s = torch.cuda.Event(enable_timing=True)
    t0s.record()
    graph_serial.replay()
    t1s.record()
    torch.cuda.synchronize()
    serial_ms = t0s.elapsed_time(t1s)

    pg = dist.is_initialized()
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    if pg:
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if pg:
        dist.barrier()
    t0.record()
    for _ in range(args.steps):
        graph.replay()
    t1.record()
    torch.cuda.synchronize()
    if pg:
        dist.barrier()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1) / args.steps
    # kept-index metadata of every rank (the only collective of the data path)
    gathered = None
    if pg:
        from submission_folder_b200 import sharding
        ms = sharding.max_over_ranks(ms, device=dev)
        allk = sharding.gather_kept({rank * L + l: idxs[l] for l in range(L)}, device=dev)
        gathered = int(sum(t.numel() for t in allk.values()))

    # device status of every layer's workspace slice (outside the timed region)
    st = ctypes.c_int32()
    status_all = 0
    off = 0
    for l in range(L):
        lib.ckv_read_status(ctypes.c_void_p(ws.data_ptr() + off),
                            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), ctypes.byref(st))
        status_all |= st.value
        off += (ops.workspace_size(params[l], n, H, Hkv, D) + 255) // 256 * 256

    tokens = L * n
    value = tokens * world / (ms / 1000.0)
    e = 2
    alg_bytes = sum(layer_bytes(n, W, b) for b in bl)
    pk = peaks()
    # the dominant kernel and its roofline: the larger of the two window passes.  They are
    # the only stages that fill every SM (one CTA per SM), so they hold most of the batched
    # step's SM-time; the sweep, selection and reduction kernels run on a few dozen CTAs
    # and overlap other layers' passes (serially the selection is as long as the pooling
    # pass, but it occupies 16 SMs).
    dom = max((STAGES.index("window_moments"), STAGES.index("window_pool")), key=lambda i: stage_ms[i])
    dom_ms = stage_ms[dom] / L
    flops = 2.0 * H * W * n * D
    kbytes = e * (Hkv * n * D + H * W * D)
    if STAGES[dom] in ("window_moments", "window_pool"):
        wbytes = kbytes + (2 * W * n * 4 if STAGES[dom] == "window_pool" else 0)
        t_tensor = flops / (pk["bf16_tflops"] * 1e12)
        t_hbm = wbytes / (pk["hbm_gbs"] * 1e9)
        if t_tensor >= t_hbm:
            roof = {"bound": "tensor", "achieved": flops / (dom_ms / 1e3) / 1e12, "peak": pk["bf16_tflops"],
                    "unit": "TFLOP/s"}
        else:
            roof = {"bound": "hbm", "achieved": wbytes / (dom_ms / 1e3) / 1e9, "peak": pk["hbm_gbs"],
                    "unit": "GB/s"}
    else:
        b = layer_bytes(n, W, bl[0])
        roof = {"bound": "hbm", "achieved": b / (dom_ms / 1e3) / 1e9, "peak": pk["hbm_gbs"], "unit": "GB/s"}
    roof["frac"] = roof["achieved"] / roof["peak"]
    roof["kernel"] = STAGES[dom]
    roof["peak_source"] = pk["source"]
    roof["avg_launch_us"] = dom_ms * 1e3
    roof["traffic"] = traffic_for(STAGES[dom])
    path_gbs = alg_bytes / (ms / 1e3) / 1e9
    # stats; the pooling pass (one kernel, either form) and its reduction; the re-run pair
    # (returns at once unless the speculated head sets were wrong); two sweep kernels;
    # selection; gather
    kernels_per_layer = 9
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": workload_config(args, world),
        "per_layer_us": ms * 1e3 / L,
        "serial_per_layer_us": serial_ms * 1e3 / L,
        "path_hbm_gbs": path_gbs, "path_hbm_frac": path_gbs / pk["hbm_gbs"],
        "stage_us_per_layer": {STAGES[i]: stage_ms[i] * 1e3 / L for i in range(len(stage_ms))},
        "roofline": roof,
        "clocks": clk,
        "gpu_launches": kernels_per_layer * L * args.steps,
        "device_status": status_all,
    }
    if gathered is not None:
        line["allgather_indices"] = gathered

    # ---- end to end through the public hook with pinned host buffers ----
    if not args.no_e2e:
        line["e2e"] = e2e(args, rank, world, dev, bl, CircuitKVCluster, cli_cluster_kwargs, make_layer,
                          repeat_kv, pg)
    if rank == 0 and world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_oracle_sample(args)
    del graph, graph_serial
    if rank == 0:
        print(json.dumps(line), flush=True)


def traffic_for(stage):
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(stage)
    except Exception:
        return None


def e2e(args, rank, world, dev, bl, CircuitKVCluster, cli_cluster_kwargs, make_layer, repeat_kv, pg):
    import torch
    import torch.distributed as dist
    n, W, L = args.n, args.window, args.layers
    G = 4
    host = []
    for l in range(2):
        q, k, v = make_layer(n, seed=1000 * rank + 2, layer=l, window=W, planted=64, dtype="bf16",
                             device=str(dev))
        host.append(tuple(x.cpu().pin_memory() for x in (q[None], repeat_kv(k, G), repeat_kv(v, G))))
        del q, k, v
    clusters = [CircuitKVCluster(**cli_cluster_kwargs(W, b)) for b in bl]
    # host -> device per layer: the window queries and K are copied; the gather reads V's
    # kept rows (8 KV heads x budget rows) from the pinned host tensor in place
    h2d = sum(2 * (32 * W * 128 + 8 * n * 128 + 8 * b * 128) for b in bl)
    d2h = sum(2 * 2 * 32 * b * 128 for b in bl)

    def one_step():
        for l in range(L):
            qh, kh, vh = host[l % 2]
            ko, vo = clusters[l].update_kv(kh, qh, vh, None, G)
        return ko

    one_step()
    torch.cuda.synchronize()
    if pg:
        dist.barrier()
    t = time.perf_counter()
    for _ in range(args.e2e_steps):
        one_step()
    torch.cuda.synchronize()
    sec = (time.perf_counter() - t) / args.e2e_steps
    if pg:
        from submission_folder_b200 import sharding
        sec = sharding.max_over_ranks(sec, device=dev)
    return {"value": L * n * world / sec, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "s_per_step": sec,
            "api": "CircuitKVCluster.update_kv on pinned host tensors"}


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    try:
        run_ours(args, rank, world)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
