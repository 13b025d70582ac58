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
    with pytest.raises(NotImplementedError):
        g.update_and_step_landmark_walker(torch.rand(8, 8, device=dev), 7, 4, 10, 2.0, 2, 0.6, False)
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
