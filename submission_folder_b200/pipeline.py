"""Scoring a whole cache that lives in host memory, with the host link busy both ways.

``CircuitKVCluster.update_kv`` on host tensors must hand back finished host tensors, so one
layer's download of its compacted K / V cannot overlap the next layer's upload.  A caller that
holds every layer of an offloaded cache (page-locked host tensors) can instead score them all
in one call: ``score_evict_pipelined`` uploads layer i + 1 (the window queries and the distinct
K heads, one strided DMA each) on one stream while layer i is scored on a second and layer
i - 1's outputs come down on a third (the link is full duplex), with two device buffer sets in
turn.  V's kept rows are read in place from page-locked memory by the final gather.  Results
equal those of one ``update_kv`` call per layer.  No reference counterpart: the reference scores
a layer at a time inside the model's forward.
"""

from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence, Tuple

import torch

from . import _lib, ops
from ._lib import Outputs, Params, check


def score_evict_pipelined(params, layers: Sequence[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]],
                          device: Optional[torch.device] = None,
                          out: Optional[Sequence[Tuple[torch.Tensor, torch.Tensor]]] = None
                          ) -> List[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]]:
    """``layers``: per layer ``(q [H, n, D], k [Hkv, n, D], v [Hkv, n, D])`` host tensors
    (views with contiguous rows per head, e.g. every ``groups``-th head of a repeat_kv'd
    tensor; page-locked for full link speed, V page-locked to be read in place);
    ``params``: one ``Params`` or one per layer.  Returns per layer ``(k_out, v_out, keep_idx)``:
    ``[H, out_len, D]`` page-locked host tensors and the kept positions (device tensors),
    all complete on return.  ``out``: per layer ``(k_out, v_out)`` host tensors to fill instead
    (contiguous, page-locked: a caller that scores caches repeatedly keeps them, which spares
    the page-locked allocations; the first allocation of page-locked memory is slow)."""
    plist = list(params) if isinstance(params, (list, tuple)) else [params] * len(layers)
    if len(plist) != len(layers):
        raise ValueError("params: one struct or one per layer")
    if out is not None and len(out) != len(layers):
        raise ValueError("out: one (k_out, v_out) pair per layer")
    if not layers:
        return []
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    lib = _lib.load()
    H, _, D = layers[0][0].shape
    Hkv = layers[0][1].shape[0]
    dt = layers[0][0].dtype
    for q, k, v in layers:
        if q.is_cuda or k.is_cuda or q.shape[0] != H or k.shape[0] != Hkv or q.dtype != dt:
            raise ValueError("host tensors of one head layout and dtype expected")
    nmax = max(q.shape[1] for q, _, _ in layers)
    omax = max(ops.output_len(p, q.shape[1]) for p, (q, _, _) in zip(plist, layers))
    need_v = any(not ops.device_readable(v) for _, _, v in layers)
    # two device buffer sets, used by layers i and i + 1 in turn
    qd = [torch.empty(H, nmax, D, dtype=dt, device=dev) for _ in range(2)]
    kd = [torch.empty(Hkv, nmax, D, dtype=dt, device=dev) for _ in range(2)]
    vd = [torch.empty(Hkv, nmax, D, dtype=dt, device=dev) for _ in range(2)] if need_v else None
    kod = [torch.empty(H * omax * D, dtype=dt, device=dev) for _ in range(2)]   # contiguous [H, out_len, D]
    vod = [torch.empty(H * omax * D, dtype=dt, device=dev) for _ in range(2)]
    ws = ops.workspace(max(ops.workspace_size(p, q.shape[1], H, Hkv, D) for p, (q, _, _) in zip(plist, layers)), dev)
    s_in, s_cmp, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    cur = torch.cuda.current_stream(dev)
    for s in (s_in, s_cmp, s_out):
        s.wait_stream(cur)
    ev_in = [torch.cuda.Event() for _ in layers]
    ev_cmp = [torch.cuda.Event() for _ in layers]
    ev_out = [torch.cuda.Event() for _ in layers]
    results = []
    for i, (p, (q, k, v)) in enumerate(zip(plist, layers)):
        b = i & 1
        n = q.shape[1]
        W = int(p.window_size)
        olen = ops.output_len(p, n)
        # upload: the window queries of every head and the distinct K heads (and V when it
        # cannot be read in place), once layer i - 2 no longer reads this buffer set
        with torch.cuda.stream(s_in):
            if i >= 2:
                s_in.wait_event(ev_cmp[i - 2])
            qv, kv = qd[b][:, :n], kd[b][:, :n]
            if not ops.copy_rows_async(qv[:, n - W:], q[:, n - W:]):
                qv[:, n - W:].copy_(q[:, n - W:], non_blocking=True)
            if not ops.copy_rows_async(kv, k):
                kv.copy_(k, non_blocking=True)
            if ops.device_readable(v):
                vv = v
            else:
                vv = vd[b][:, :n]
                vv.copy_(v, non_blocking=True)
            ev_in[i].record(s_in)
        # scoring, once the upload is in and layer i - 2's outputs have left this buffer set
        with torch.cuda.stream(s_cmp):
            s_cmp.wait_event(ev_in[i])
            if i >= 2:
                s_cmp.wait_event(ev_out[i - 2])
            ko = kod[b][:H * olen * D].view(H, olen, D)
            vo = vod[b][:H * olen * D].view(H, olen, D)
            idx = ops._index_tensor(p, H, olen, dev)
            L = ops.make_layer(qv, kv, vv)
            O = Outputs()
            O.out_k, O.out_v, O.out_idx, O.out_scores = ko.data_ptr(), vo.data_ptr(), idx.data_ptr(), None
            O.distinct_kv_heads = 0
            check(lib.ckv_score_evict(ctypes.byref(p), ctypes.byref(L), ctypes.c_void_p(ws.data_ptr()),
                                      ws.numel(), ctypes.byref(O), ops._stream(dev)), "ckv_score_evict")
            if n < p.max_capacity_prompt:   # shorter than the budget: every row kept
                idx = torch.arange(max(n - W, 0), dtype=torch.int32, device=dev)
            ev_cmp[i].record(s_cmp)
        # download of the compacted K / V into page-locked host tensors
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_cmp[i])
            if out is not None:
                kh, vh = out[i]
                if kh.shape != (H, olen, D) or vh.shape != (H, olen, D) or not (kh.is_contiguous() and vh.is_contiguous()):
                    raise ValueError(f"out[{i}]: contiguous [{H}, {olen}, {D}] host tensors expected")
            else:
                kh = torch.empty(H, olen, D, dtype=dt, pin_memory=True)
                vh = torch.empty(H, olen, D, dtype=dt, pin_memory=True)
            kh.copy_(ko, non_blocking=True)
            vh.copy_(vo, non_blocking=True)
            ev_out[i].record(s_out)
        results.append((kh, vh, idx))
    s_out.synchronize()
    s_cmp.synchronize()
    cur.wait_stream(s_cmp)
    return results
