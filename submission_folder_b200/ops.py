"""Torch-facing wrappers of the C ABI (device memory and streams come from torch).

Every function here runs the sm_100a kernels of ``libckv.so`` on the tensors'
CUDA device and the current torch stream.  Host (CPU) tensors are copied to
the GPU first and results copied back; nothing runs on the CPU.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from . import _lib
from ._lib import Layer, Outputs, Params, check

_DT = {torch.bfloat16: "bf16", torch.float16: "fp16", torch.float32: "fp32"}

_workspaces = {}


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """A cached uint8 workspace of at least ``nbytes`` on ``device`` (256-byte aligned)."""
    key = (device.type, device.index)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    return ws


def workspace_size(p: Params, n: int, heads: int, kv_heads: int, head_dim: int) -> int:
    out = ctypes.c_size_t()
    check(_lib.load().ckv_workspace_size(ctypes.byref(p), n, heads, kv_heads, head_dim,
                                         ctypes.byref(out)), "ckv_workspace_size")
    return out.value


def output_len(p: Params, n: int) -> int:
    out = ctypes.c_int32()
    check(_lib.load().ckv_output_len(ctypes.byref(p), n, ctypes.byref(out)), "ckv_output_len")
    return out.value


def device_readable(t: torch.Tensor) -> bool:
    """Whether the current CUDA device can read ``t`` in place (its own memory, or
    page-locked host memory mapped at the same address)."""
    if t.is_cuda:
        return True
    if not t.is_pinned() or not torch.cuda.is_available():
        return False
    ok = ctypes.c_int32(0)
    check(_lib.load().ckv_device_accessible(ctypes.c_void_p(t.data_ptr()), ctypes.byref(ok)), "ckv_device_accessible")
    return ok.value == 1


def copy_rows_async(dst: torch.Tensor, src: torch.Tensor) -> bool:
    """``dst.copy_(src)`` for ``[R, ...]`` tensors whose every ``[r]`` slice is contiguous
    (e.g. one head's rows of a host tensor with heads far apart) as ONE strided DMA on the
    current stream; returns False (nothing copied) when the layout does not allow it."""
    if dst.shape != src.shape or dst.dtype != src.dtype or dst.dim() < 2 or dst.shape[0] == 0:
        return False
    if not (dst[0].is_contiguous() and src[0].is_contiguous()):
        return False
    e = dst.element_size()
    row = dst[0].numel() * e
    if dst.shape[0] > 1 and (dst.stride(0) * e < row or src.stride(0) * e < row):
        return False
    dev = dst.device if dst.is_cuda else src.device
    check(_lib.load().ckv_copy_rows(ctypes.c_void_p(dst.data_ptr()), dst.stride(0) * e,
                                     ctypes.c_void_p(src.data_ptr()), src.stride(0) * e, row, dst.shape[0],
                                     _stream(dev)), "ckv_copy_rows")
    return True


def _require_readable(v: torch.Tensor) -> None:
    """V is read only by the final gather: device memory, or page-locked host memory the
    device reads in place."""
    if not torch.cuda.is_available():
        raise RuntimeError("the CircuitKV B200 kernels need a CUDA device; none is available")
    if not device_readable(v):
        raise RuntimeError("v must be on the CUDA device or in page-locked host memory it can read")


def _require_cuda(*ts: torch.Tensor) -> None:
    if not torch.cuda.is_available():
        raise RuntimeError("the CircuitKV B200 kernels need a CUDA device; none is available")
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("tensor is not on a CUDA device")


def make_layer(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> Layer:
    """``q`` ``[H, n, D]``, ``k``/``v`` ``[Hkv, n, D]`` views (head_dim contiguous)."""
    if q.dtype not in _DT or k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError("q, k, v must share one dtype among bf16 / fp16 / fp32")
    for t in (q, k, v):
        if t.dim() != 3 or t.stride(-1) != 1:
            raise ValueError("expected [heads, n, head_dim] views with contiguous head_dim")
    L = Layer()
    L.q, L.q_head_stride, L.q_tok_stride = q.data_ptr(), q.stride(0), q.stride(1)
    L.k, L.k_head_stride, L.k_tok_stride = k.data_ptr(), k.stride(0), k.stride(1)
    L.v, L.v_head_stride, L.v_tok_stride = v.data_ptr(), v.stride(0), v.stride(1)
    L.n, L.num_heads, L.num_kv_heads, L.head_dim = q.shape[1], q.shape[0], k.shape[0], q.shape[2]
    L.dtype = _lib.DTYPE_CODES[_DT[q.dtype]]
    return L


def _index_tensor(p: Params, heads: int, out_len: int, dev: torch.device) -> torch.Tensor:
    """Kept-position output: ``[out_len - W]`` (shared) or ``[H, out_len - W]`` (per head)."""
    nidx = max(out_len - p.window_size, 1)
    if p.per_head_eviction:
        return torch.empty(heads, nidx, dtype=torch.int32, device=dev)
    return torch.empty(nidx, dtype=torch.int32, device=dev)


def score_evict(p: Params, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                want_scores: bool = False, distinct_kv_heads: bool = False) -> Tuple[torch.Tensor, torch.Tensor,
                                                                                    torch.Tensor,
                                                                                    Optional[torch.Tensor]]:
    """One layer: returns ``(k_out [H,B,D], v_out [H,B,D], keep_idx, scores)``; ``keep_idx``
    is ``[B-W]`` int32 (shared eviction) or ``[H, B-W]`` (per-head eviction).

    ``scores`` (when requested) is ``[2, n]`` fp32: the two vectors ranked by the
    selection (QI / HI after smoothing for "dis"; influence / H2O for "max"); with per-head
    eviction ``(vectors [H, 2, n - W], entropies [H])``.
    ``distinct_kv_heads``: K / V outputs hold each KV head once, ``[Hkv, B, D]``.
    """
    _require_cuda(q, k)
    _require_readable(v)
    H, n, D = q.shape
    L = make_layer(q, k, v)
    out_len = output_len(p, n)
    dev = q.device
    ho = k.shape[0] if distinct_kv_heads else H
    k_out = torch.empty(ho, out_len, D, dtype=q.dtype, device=dev)
    v_out = torch.empty(ho, out_len, D, dtype=q.dtype, device=dev)
    idx = _index_tensor(p, H, out_len, dev)
    per_head = bool(p.per_head_eviction) and n >= p.max_capacity_prompt
    nsc = H * 2 * (n - p.window_size) + H if per_head else 2 * n
    scores = torch.empty(nsc, dtype=torch.float32, device=dev) if want_scores else None
    ws = workspace(workspace_size(p, n, H, k.shape[0], D), dev)
    O = Outputs()
    O.out_k, O.out_v, O.out_idx, O.out_scores = k_out.data_ptr(), v_out.data_ptr(), idx.data_ptr(), _ptr(scores)
    O.distinct_kv_heads = 1 if distinct_kv_heads else 0
    check(_lib.load().ckv_score_evict(ctypes.byref(p), ctypes.byref(L), ctypes.c_void_p(ws.data_ptr()),
                                      ws.numel(), ctypes.byref(O), _stream(dev)), "ckv_score_evict")
    if n < p.max_capacity_prompt:
        idx = torch.arange(max(n - p.window_size, 0), dtype=torch.int32, device=dev)
    return k_out, v_out, idx, _shape_scores(scores, p, H, n)


def _shape_scores(scores: Optional[torch.Tensor], p: Params, H: int, n: int):
    """The flat out_scores buffer as ``[2, n]``, or per head ``([H, 2, n - W], [H])``."""
    if scores is None:
        return None
    if bool(p.per_head_eviction) and n >= p.max_capacity_prompt:
        nw = n - p.window_size
        return scores[:H * 2 * nw].view(H, 2, nw), scores[H * 2 * nw:]
    return scores.view(2, n)


def score_evict_batched(params, layers, want_scores: bool = False):
    """Many independent layers / sequences in one call (ragged ``n`` allowed).

    ``params``: one ``Params`` for every layer or a list with one per layer;
    ``layers``: list of ``(q [H,n,D], k [Hkv,n,D], v [Hkv,n,D])``.  Returns a list of
    ``score_evict`` results in the same order.  The layers run concurrently on the
    library's internal streams; outputs are ready in stream order after the call.
    """
    plist = list(params) if isinstance(params, (list, tuple)) else [params]
    if len(plist) not in (1, len(layers)):
        raise ValueError("params: one struct or one per layer")
    if not layers:
        return []
    dev = layers[0][0].device
    Ls = (Layer * len(layers))()
    Os = (Outputs * len(layers))()
    results = []
    total = 0
    for i, (q, k, v) in enumerate(layers):
        _require_cuda(q, k, v)
        p = plist[0] if len(plist) == 1 else plist[i]
        H, n, D = q.shape
        Ls[i] = make_layer(q, k, v)
        out_len = output_len(p, n)
        k_out = torch.empty(H, out_len, D, dtype=q.dtype, device=dev)
        v_out = torch.empty(H, out_len, D, dtype=q.dtype, device=dev)
        idx = _index_tensor(p, H, out_len, dev)
        per_head = bool(p.per_head_eviction) and n >= p.max_capacity_prompt
        nsc = H * 2 * (n - p.window_size) + H if per_head else 2 * n
        scores = torch.empty(nsc, dtype=torch.float32, device=dev) if want_scores else None
        Os[i].out_k, Os[i].out_v, Os[i].out_idx, Os[i].out_scores = (k_out.data_ptr(), v_out.data_ptr(),
                                                                     idx.data_ptr(), _ptr(scores))
        results.append([k_out, v_out, idx, scores, n, p])
        total += (workspace_size(p, n, H, k.shape[0], D) + 255) // 256 * 256
    ws = workspace(total, dev)
    P = (Params * len(plist))(*plist)
    check(_lib.load().ckv_score_evict_batched(P, len(plist), Ls, len(layers), ctypes.c_void_p(ws.data_ptr()),
                                              ws.numel(), Os, _stream(dev)), "ckv_score_evict_batched")
    out = []
    for k_out, v_out, idx, scores, n, p in results:
        if n < p.max_capacity_prompt:
            idx = torch.arange(max(n - p.window_size, 0), dtype=torch.int32, device=dev)
        out.append((k_out, v_out, idx, _shape_scores(scores, p, k_out.shape[0], n)))
    return out


def read_status(dev: torch.device) -> int:
    """Device status word of the cached workspace (synchronises)."""
    ws = _workspaces.get((dev.type, dev.index))
    if ws is None:
        return 0
    st = ctypes.c_int32()
    check(_lib.load().ckv_read_status(ctypes.c_void_p(ws.data_ptr()), _stream(dev), ctypes.byref(st)),
          "ckv_read_status")
    return st.value


def select_scores(p: Params, a: torch.Tensor, b: torch.Tensor, c: Optional[torch.Tensor] = None,
                  want_scores: bool = False):
    """Selection stage alone from fp32 score vectors on the GPU; returns (keep_idx, scores)."""
    _require_cuda(a, b, c)
    n = a.numel()
    dev = a.device
    out_len = output_len(p, n)
    idx = torch.empty(max(out_len - p.window_size, 1), dtype=torch.int32, device=dev)
    scores = torch.empty(2, n, dtype=torch.float32, device=dev) if want_scores else None
    ws = workspace(workspace_size(p, n, 32, 8, 128), dev)
    a, b = a.float().contiguous(), b.float().contiguous()
    c = None if c is None else c.float().contiguous()
    check(_lib.load().ckv_select_scores(ctypes.byref(p), n, a.data_ptr(), b.data_ptr(), _ptr(c),
                                        ctypes.c_void_p(ws.data_ptr()), ws.numel(), idx.data_ptr(),
                                        _ptr(scores), _stream(dev)), "ckv_select_scores")
    return idx, scores


def neumann_rows(p: Params, rows_qi: torch.Tensor, rows_hi: Optional[torch.Tensor],
                 single_chain: bool = False):
    """Absorption solve alone from pooled rows ``[W, n]``; returns (qi, hi, steps tensor)."""
    _require_cuda(rows_qi, rows_hi)
    W, n = rows_qi.shape
    dev = rows_qi.device
    out_qi = torch.empty(n, dtype=torch.float32, device=dev)
    out_hi = torch.empty(n, dtype=torch.float32, device=dev)
    steps = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = workspace(workspace_size(p, n, 32, 8, 128), dev)
    rq = rows_qi.float().contiguous()
    rh = None if rows_hi is None else rows_hi.float().contiguous()
    check(_lib.load().ckv_neumann_rows(ctypes.byref(p), n, rq.data_ptr(), _ptr(rh), int(single_chain),
                                       ctypes.c_void_p(ws.data_ptr()), ws.numel(), out_qi.data_ptr(),
                                       out_hi.data_ptr(), steps.data_ptr(), _stream(dev)),
          "ckv_neumann_rows")
    return out_qi, out_hi, steps


def window_pool(p: Params, q: torch.Tensor, k: torch.Tensor):
    """Window statistics + pooling alone: (entropy [H], mass [H], qi_set, hi_set, rows_qi, rows_hi)."""
    _require_cuda(q, k)
    H, n, D = q.shape
    dev = q.device
    L = make_layer(q, k, k)
    ent = torch.empty(H, dtype=torch.float32, device=dev)
    mass = torch.empty(H, dtype=torch.float32, device=dev)
    sets = torch.zeros(2, dtype=torch.int64, device=dev)
    rq = torch.empty(p.window_size, n, dtype=torch.float32, device=dev)
    rh = torch.empty(p.window_size, n, dtype=torch.float32, device=dev)
    ws = workspace(workspace_size(p, max(n, p.max_capacity_prompt), H, k.shape[0], D), dev)
    check(_lib.load().ckv_window_pool(ctypes.byref(p), ctypes.byref(L), ctypes.c_void_p(ws.data_ptr()),
                                      ws.numel(), ent.data_ptr(), mass.data_ptr(), sets.data_ptr(),
                                      sets.data_ptr() + 8, rq.data_ptr(), rh.data_ptr(), _stream(dev)),
          "ckv_window_pool")
    return ent, mass, sets, rq, rh


def choose_heads(p: Params, entropy: torch.Tensor, mass: torch.Tensor):
    """Head sets of a layer from all its heads' entropy / mass: (sets int64 [2] = QI, HI
    bit masks; mode int32 [2] = HI mode, HI head count), on the device."""
    _require_cuda(entropy, mass)
    dev = entropy.device
    e, m = entropy.float().contiguous(), mass.float().contiguous()
    sets = torch.zeros(2, dtype=torch.int64, device=dev)
    mode = torch.zeros(2, dtype=torch.int32, device=dev)
    check(_lib.load().ckv_choose_heads(ctypes.byref(p), e.numel(), e.data_ptr(), m.data_ptr(), sets.data_ptr(),
                                       mode.data_ptr(), _stream(dev)), "ckv_choose_heads")
    return sets, mode


def pool_rows_given(p: Params, q: torch.Tensor, k: torch.Tensor, head_offset: int, sets: torch.Tensor,
                    mode: torch.Tensor):
    """This rank's pooled rows for given head sets: (rows_qi [W, n] = max over its QI heads,
    rows_hi [W, n] = sum over its HI heads).  ``q`` / ``k``: the rank's heads."""
    _require_cuda(q, k, sets, mode)
    H, n, D = q.shape
    dev = q.device
    L = make_layer(q, k, k)
    rq = torch.empty(p.window_size, n, dtype=torch.float32, device=dev)
    rh = torch.zeros(p.window_size, n, dtype=torch.float32, device=dev)
    ws = workspace(workspace_size(p, max(n, p.max_capacity_prompt), H, k.shape[0], D), dev)
    check(_lib.load().ckv_pool_rows_given(ctypes.byref(p), ctypes.byref(L), int(head_offset), sets.data_ptr(),
                                          mode.data_ptr(), ctypes.c_void_p(ws.data_ptr()), ws.numel(),
                                          rq.data_ptr(), rh.data_ptr(), _stream(dev)), "ckv_pool_rows_given")
    return rq, rh


# ---------------------------------------------------------------------------
# influence walker (legacy use_neumann=False path) and stand-alone gather
# ---------------------------------------------------------------------------
def walk_workspace_size(n: int, window: int) -> int:
    out = ctypes.c_size_t()
    check(_lib.load().ckv_walk_workspace_size(n, window, ctypes.byref(out)), "ckv_walk_workspace_size")
    return out.value


def _check_rng_state(rng_state: Optional[torch.Tensor], rng_mode: int, num_walkers: int) -> None:
    if rng_state is None:
        return
    need = 2 * num_walkers if rng_mode == _lib.RNG_PCG else 1
    if rng_state.dtype != torch.int64 or not rng_state.is_contiguous() or rng_state.numel() < need:
        raise ValueError(f"rng_state must be a contiguous int64 tensor of at least {need} elements")


def influence_walk(rows: torch.Tensor, current_idx: int, num_walkers: int = 10000, max_steps: int = 10,
                   sink_size: int = 4, temperature: float = 2.0, explore_temp: float = 10.0,
                   explore_ratio: float = 0.3, rng_mode: int = _lib.RNG_PCG, seed: int = 42 + 3000,
                   rng_state: Optional[torch.Tensor] = None, init_state: bool = False):
    """Walker on the full_attn defined by pooled window rows ``[W, n]`` fp32 (structured,
    never materialised).  Returns ``(scores [n], visits [n], h2o [n])``."""
    _require_cuda(rows, rng_state)
    _check_rng_state(rng_state, rng_mode, num_walkers)
    rows = rows.float().contiguous()
    W, n = rows.shape
    dev = rows.device
    ws = torch.empty((walk_workspace_size(n, W) + 255) // 256 * 256 + 256, dtype=torch.uint8, device=dev)
    base = (ws.data_ptr() + 255) // 256 * 256
    scores = torch.empty(n, dtype=torch.float32, device=dev)
    visits = torch.empty(n, dtype=torch.float32, device=dev)
    h2o = torch.empty(n, dtype=torch.float32, device=dev)
    check(_lib.load().ckv_influence_walk(rows.data_ptr(), W, n, n, current_idx, num_walkers, max_steps, sink_size,
                                         temperature, explore_temp, explore_ratio, rng_mode, seed,
                                         _ptr(rng_state), int(init_state), ctypes.c_void_p(base),
                                         ws.numel() - (base - ws.data_ptr()), visits.data_ptr(),
                                         scores.data_ptr(), h2o.data_ptr(), _stream(dev)),
          "ckv_influence_walk")
    return scores, visits, h2o


def influence_walk_dense(attn: torch.Tensor, current_idx: int, num_walkers: int = 10000, max_steps: int = 10,
                         sink_size: int = 4, temperature: float = 2.0, explore_temp: float = 10.0,
                         explore_ratio: float = 0.3, rng_mode: int = _lib.RNG_PCG, seed: int = 42 + 3000,
                         rng_state: Optional[torch.Tensor] = None, init_state: bool = False,
                         visits: Optional[torch.Tensor] = None, scores: Optional[torch.Tensor] = None):
    """Walker on a dense ``[n, n]`` fp32 attention matrix; returns ``(scores, visits)``."""
    _require_cuda(attn, rng_state)
    _check_rng_state(rng_state, rng_mode, num_walkers)
    if attn.dtype != torch.float32 or attn.dim() != 2 or attn.shape[0] != attn.shape[1] or not attn.is_contiguous():
        raise ValueError("attn must be a contiguous square float32 matrix")
    n = attn.shape[0]
    dev = attn.device
    scores = torch.empty(n, dtype=torch.float32, device=dev) if scores is None else scores
    visits = torch.empty(n, dtype=torch.float32, device=dev) if visits is None else visits
    check(_lib.load().ckv_influence_walk_dense(attn.data_ptr(), n, current_idx, num_walkers, max_steps,
                                               sink_size, temperature, explore_temp, explore_ratio, rng_mode,
                                               seed, _ptr(rng_state), int(init_state), visits.data_ptr(),
                                               scores.data_ptr(), _stream(dev)), "ckv_influence_walk_dense")
    return scores, visits


def rng_fill(mode: int, seed: int, stream_id: int, count: int, device: torch.device) -> torch.Tensor:
    """Raw generator outputs (uint64 values in an int64 tensor)."""
    out = torch.empty(max(count, 1), dtype=torch.int64, device=device)
    check(_lib.load().ckv_rng_fill(mode, seed, stream_id, count, out.data_ptr(), _stream(device)), "ckv_rng_fill")
    return out[:count]


def gather(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, window: int, idx: torch.Tensor):
    """K / V of the kept positions ``idx`` (``[kept]`` or ``[H, kept]``) then the last
    ``window`` rows: ``[H, kept + window, D]`` each."""
    _require_cuda(q, k, idx)
    _require_readable(v)
    H, n, D = q.shape
    L = make_layer(q, k, v)
    idx = idx.to(torch.int32).contiguous()
    kept = idx.shape[-1]
    k_out = torch.empty(H, kept + window, D, dtype=k.dtype, device=k.device)
    v_out = torch.empty(H, kept + window, D, dtype=k.dtype, device=k.device)
    check(_lib.load().ckv_gather(ctypes.byref(L), window, idx.data_ptr(), kept, int(idx.dim() == 2),
                                 k_out.data_ptr(), v_out.data_ptr(), _stream(k.device)), "ckv_gather")
    return k_out, v_out
