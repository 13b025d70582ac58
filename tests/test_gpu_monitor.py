"""Decode-time graph scoring of ``circuit_kv._C.CircuitGraph`` on the GPU (through the
C ABI): the graph update, the absorbing circuit walker, the spectral power iteration and
the combined scores against the reference's own kernels (graph_update.cu,
circuit_walker.cu, spectral_power.cu compiled from their sources into oracle/_ref by
oracle/Makefile) on the same inputs and PCG states -- bit for bit -- and the monitor API
on top of them."""

import ctypes
import os

import numpy as np
import pytest
import torch

from submission_folder_b200 import _lib
from submission_folder_b200.circuit_kv import CircuitKVConfig, CircuitKVMonitor, _C

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_SO = os.path.join(ROOT, "oracle", "_ref", "libref_monitor.so")


def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _ref():
    if not os.path.exists(REF_SO):
        pytest.skip("the reference's kernels are not built (oracle/Makefile)")
    lib = ctypes.CDLL(REF_SO)
    vp, i32, u64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_uint64
    lib.ref_graph_update.argtypes = [vp, vp, i32, i32, i32, i32, i32, vp, vp, vp]
    lib.ref_init_rng.argtypes = [vp, u64, i32, vp]
    lib.ref_circuit_walk.argtypes = [vp, vp, vp, vp, i32, i32, i32, i32, vp]
    lib.ref_spectral_combined.argtypes = [vp, vp, vp, i32, i32, i32, vp, vp, vp, vp, vp, vp]
    f32 = ctypes.c_float
    lib.ref_landmark_walk.argtypes = [vp, i32, i32, i32, i32, i32, f32, i32, f32, i32, vp, vp, vp, vp, vp, vp, vp]
    return lib


def _st(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _graph(dev, n, top_k, dtype, seed, positive=True):
    """Rows 4 .. n-1 each from its own query over the keys up to that row (a causal graph),
    built by both implementations."""
    g = torch.Generator().manual_seed(seed)
    keys = torch.rand(n, 128, generator=g) if positive else torch.randn(n, 128, generator=g)
    qs = torch.rand(n, 128, generator=g) if positive else torch.randn(n, 128, generator=g)
    keys, qs = keys.to(dtype).to(dev), qs.to(dtype).to(dev)
    code = {torch.float16: 1, torch.float32: 2}[dtype]
    lib, ref = _lib.load(), _ref()
    adj = torch.full((n, top_k), -1, dtype=torch.int32, device=dev)
    w = torch.zeros(n, top_k, dtype=torch.float32, device=dev)
    radj, rw = adj.clone(), w.clone()
    scratch = torch.empty(n, dtype=torch.float32, device=dev)
    for row in range(4, n):
        m = row + 1
        assert lib.ckv_graph_update(qs[row].data_ptr(), keys.data_ptr(), code, m, 128, row, top_k,
                                    scratch.data_ptr(), adj.data_ptr(), w.data_ptr(), _st(dev)) == 0
        assert ref.ref_graph_update(qs[row].data_ptr(), keys.data_ptr(), code, m, 128, row, top_k,
                                    radj.data_ptr(), rw.data_ptr(), _st(dev)) == 0
    torch.cuda.synchronize()
    return adj, w, radj, rw


@pytest.mark.parametrize("dtype,top_k", [(torch.float16, 32), (torch.float32, 8), (torch.float16, 64)])
def test_graph_update_matches_reference(dtype, top_k):
    dev = _cuda()
    adj, w, radj, rw = _graph(dev, 300, top_k, dtype, seed=top_k)
    assert torch.equal(w, rw)
    assert torch.equal(adj, radj)
    # short rows: fewer keys than top_k leave -1 / 0 entries
    assert int(adj[4, 5].item()) == -1 and float(w[4, 5].item()) == 0.0


def test_circuit_walk_spectral_and_combined_match_reference():
    dev = _cuda()
    n, top_k, walkers = 700, 16, 2048
    adj, w, radj, rw = _graph(dev, n, top_k, torch.float16, seed=3)
    assert torch.equal(adj, radj) and torch.equal(w, rw)
    lib, ref = _lib.load(), _ref()
    st = torch.zeros(2 * walkers, dtype=torch.int64, device=dev)
    rst = torch.zeros_like(st)
    assert lib.ckv_pcg_seed(42, walkers, st.data_ptr(), _st(dev)) == 0
    assert ref.ref_init_rng(rst.data_ptr(), 42, walkers, _st(dev)) == 0
    torch.cuda.synchronize()
    assert torch.equal(st, rst)
    visits = torch.zeros(n, dtype=torch.int32, device=dev)
    rvisits = torch.zeros_like(visits)
    for call in range(3):   # states carried across calls, visits cleared each time
        assert lib.ckv_circuit_walk(adj.data_ptr(), w.data_ptr(), n, top_k, n - 1, walkers, st.data_ptr(),
                                    visits.data_ptr(), 1, _st(dev)) == 0
        rvisits.zero_()
        assert ref.ref_circuit_walk(radj.data_ptr(), rw.data_ptr(), rvisits.data_ptr(), rst.data_ptr(), n - 1, n,
                                    top_k, walkers, _st(dev)) == 0
        torch.cuda.synchronize()
        assert torch.equal(visits, rvisits), call
        assert torch.equal(st, rst), call
    assert int(visits[:4].sum().item()) > 0 and int(visits[n - 1].item()) == walkers
    # spectral scores and the combination
    v, vt, ws, comb = (torch.zeros(n, dtype=torch.float32, device=dev) for _ in range(4))
    rv, rvt, rws, rcomb = (torch.zeros(n, dtype=torch.float32, device=dev) for _ in range(4))
    scratch = torch.zeros(257, dtype=torch.float32, device=dev)
    assert lib.ckv_spectral_scores(adj.data_ptr(), w.data_ptr(), n, top_k, 10, v.data_ptr(), vt.data_ptr(),
                                   _st(dev)) == 0
    assert lib.ckv_combine_scores(visits.data_ptr(), v.data_ptr(), ws.data_ptr(), comb.data_ptr(), n, _st(dev)) == 0
    assert ref.ref_spectral_combined(radj.data_ptr(), rw.data_ptr(), rvisits.data_ptr(), n, top_k, 10, rv.data_ptr(),
                                     rvt.data_ptr(), rws.data_ptr(), rcomb.data_ptr(), scratch.data_ptr(),
                                     _st(dev)) == 0
    torch.cuda.synchronize()
    assert torch.equal(v, rv)
    assert torch.equal(ws, rws)
    assert torch.equal(comb, rcomb)
    assert float(comb.max().item()) == 1.0


def test_circuit_graph_and_monitor_api():
    dev = _cuda()
    n = 256
    g = _C.CircuitGraph(512, 16, 0.85, 1024, 100)
    torch.manual_seed(0)
    keys = torch.rand(n, 128, device=dev, dtype=torch.float16)
    for idx in range(4, n):
        g.update_and_step_circuit(torch.rand(128, device=dev, dtype=torch.float16), keys[: idx + 1], idx)
    sc = g.get_scores()
    assert sc.shape == (512,) and float(sc[n - 1].item()) == 1024.0 and float(sc[:4].sum().item()) > 0
    g.update_and_step_circuit_combined(torch.rand(128, device=dev, dtype=torch.float16), keys, n - 1, 10)
    comb = g.get_combined_scores()
    assert comb.shape == (512,) and abs(float(comb[:n].max().item()) - 1.0) < 1e-6
    g.reset()
    assert float(g.get_scores().sum().item()) == 0.0
    with pytest.raises(RuntimeError):
        g.update_and_step_circuit(torch.rand(128, device=dev), keys[:10].float().cpu(), 9)
    # the monitor on top: prefill charge, then the EMA of the circuit current
    mon = CircuitKVMonitor(CircuitKVConfig(max_seq_len=512, top_k=16, num_walkers=512))
    attn = torch.rand(n, n, device=dev)
    mon.initialize_from_prefill(attn)
    before = mon.get_scores().clone()
    mon.update(torch.rand(128, device=dev, dtype=torch.float16), keys, n - 1)
    after = mon.get_scores()
    cur = mon.get_instant_current()
    expect = 0.95 * before + 0.05 * (cur / cur[:n].max())
    torch.testing.assert_close(after, expect)
    m = mon.get_keep_mask(0.5, n)
    assert int(m.sum().item()) == n // 2 and bool(m[:4].all()) and bool(m[n - 64:].all())


def _causal_attention(dev, n, seed, zero_cols=0, negative=False):
    """Softmax rows of random logits under a causal mask (row i over keys [0, i]); optionally
    the first zero_cols columns zeroed (rows without mass there, so walkers jump) or a few
    negative entries (running sums not monotone)."""
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(n, n, generator=g) * 2.0
    logits = logits.masked_fill(torch.ones(n, n, dtype=torch.bool).triu(1), float("-inf"))
    a = torch.softmax(logits, dim=-1)
    if zero_cols:
        a[:, :zero_cols] = 0.0
    if negative:
        idx = torch.randint(0, n, (n // 4, 2), generator=g)
        a[idx[:, 0], idx[:, 1]] = -1e-3
    return a.contiguous().to(dev)


LANDMARK_CASES = [
    # n, mode (0 positional, 1 reachability, 2 absorbing), landmarks, walkers/source, boost, spacing, alpha, absorb, kind
    (700, 0, 32, 100, 2.0, 50, 0.6, 0, "plain"),
    (900, 1, 16, 37, 1.3, 20, 0.6, 0, "plain"),
    (1024, 2, 8, 100, 2.0, 50, 0.0, 1, "plain"),
    (800, 2, 12, 50, 3.7, 10, 0.0, 0, "plain"),
    (600, 1, 8, 64, 2.0, 50, 0.6, 0, "zero_cols"),
    (640, 0, 8, 64, 2.5, 30, 0.8, 0, "negative"),
    (80, 1, 8, 64, 2.0, 50, 0.6, 0, "plain"),          # shorter than 89: no landmarks
    (701, 1, 8, 37, 1.3, 20, 0.6, 0, "plain"),         # n not a multiple of 4: scalar row reads
    (2309, 2, 16, 64, 2.0, 50, 0.0, 1, "plain"),       # several 128-column blocks, ragged edge
]


@pytest.mark.parametrize("case", LANDMARK_CASES, ids=[f"n{c[0]}_m{c[1]}_{c[8]}" for c in LANDMARK_CASES])
def test_landmark_walk_matches_reference(case):
    n, mode, L, wps, boost, spacing, alpha, absorb, kind = case
    dev = _cuda()
    lib, ref = _lib.load(), _ref()
    a = _causal_attention(dev, n, seed=n + mode, zero_cols=40 if kind == "zero_cols" else 0,
                          negative=kind == "negative")
    walkers = (L + 1) * wps
    st = torch.zeros(2 * walkers, dtype=torch.int64, device=dev)
    assert lib.ckv_pcg_seed(42 + 1000, walkers, st.data_ptr(), _st(dev)) == 0
    rst = st.clone()
    sz = ctypes.c_size_t()
    assert lib.ckv_landmark_workspace_size(n, ctypes.byref(sz)) == 0
    ws = torch.zeros(sz.value, dtype=torch.uint8, device=dev)
    mine = dict(v=torch.zeros(n, dtype=torch.int32, device=dev), s=torch.zeros(n, device=dev),
                p=torch.zeros(32, dtype=torch.int32, device=dev), c=torch.zeros(1, dtype=torch.int32, device=dev))
    theirs = {k: torch.zeros_like(t) for k, t in mine.items()}
    rh2o = torch.zeros(n, device=dev)
    for call in range(2):   # PCG states carried over
        assert lib.ckv_landmark_walk(a.data_ptr(), n, n - 1, mode, L, wps, boost, spacing, alpha, absorb,
                                     st.data_ptr(), mine["v"].data_ptr(), mine["s"].data_ptr(), mine["p"].data_ptr(),
                                     mine["c"].data_ptr(), ws.data_ptr(), ws.numel(), _st(dev)) == 0
        assert ref.ref_landmark_walk(a.data_ptr(), n, n - 1, mode, L, wps, boost, spacing, alpha, absorb,
                                     rst.data_ptr(), theirs["v"].data_ptr(), theirs["s"].data_ptr(),
                                     theirs["p"].data_ptr(), theirs["c"].data_ptr(), rh2o.data_ptr(), _st(dev)) == 0
        torch.cuda.synchronize()
        k = int(theirs["c"].item())
        assert int(mine["c"].item()) == k, call
        assert torch.equal(mine["p"][:k], theirs["p"][:k]), call
        assert torch.equal(ws[: 4 * n].view(torch.float32), rh2o), call      # H2O scores
        assert torch.equal(mine["v"], theirs["v"]), (call, int((mine["v"] != theirs["v"]).sum()))
        assert torch.equal(st, rst), call
        assert torch.equal(mine["s"], theirs["s"]), call
    if n >= 89:
        assert k >= 1
    else:
        assert k == 0
    assert int(mine["v"].sum().item()) > 0


def test_landmark_methods_of_circuit_graph():
    dev = _cuda()
    n = 512
    a = _causal_attention(dev, n, seed=5)
    g = _C.CircuitGraph(1024, 16, 0.85, 1024, 100)
    assert g.get_landmark_positions().numel() == 0
    g.update_and_step_landmark_walker(a, n - 1)
    sc = g.get_landmark_scores()
    pos = g.get_landmark_positions()
    assert sc.shape == (n,) and float(sc[:4].abs().sum().item()) == 0.0 and float(sc.max().item()) > 0
    assert pos.numel() >= 1 and bool((pos[1:] > pos[:-1]).all()) and int(pos.min()) >= 24 and int(pos.max()) < n - 64
    g.update_and_step_landmark_absorbing_walker(a, n - 1, num_landmarks=8)
    raw = g.get_landmark_absorbing_raw_visits()
    assert raw.dtype == torch.int32 and raw.shape == (n,) and int(raw.sum().item()) > 0
    assert g.get_landmark_absorbing_scores().shape == (n,)
    with pytest.raises(RuntimeError):
        g.update_and_step_landmark_walker(a, n - 1, num_landmarks=33)
    with pytest.raises(RuntimeError):
        g.update_and_step_landmark_walker(a, n - 1, num_landmarks=32, walkers_per_source=600)
    with pytest.raises(RuntimeError):
        g.update_and_step_landmark_walker(a.half(), n - 1)
    # the monitor on top
    from submission_folder_b200.circuit_kv import LandmarkWalkerConfig, LandmarkWalkerMonitor
    mon = LandmarkWalkerMonitor(LandmarkWalkerConfig(max_seq_len=1024))
    mon.update(a, n - 1)
    s = mon.get_scores()
    assert s.shape == (n,) and float(s.max().item()) > 0
    m = mon.get_keep_mask(0.5, n)
    assert int(m.sum().item()) == n // 2
