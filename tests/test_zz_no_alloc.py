"""The workspace-free selection entry point, ckv_select_scores_noalloc.

It exists for callers that cannot give this library device memory -- a serving
engine that reserved nearly all HBM for its KV-cache pool at start-up, or a C /
FFI caller with no device allocator -- and keeps its scratch in a static device
array inside the library (n <= 32768).  This test calls it through the C ABI and
checks that two calls in a row return exactly what the workspace entry point
(ckv_select_scores) returns on the same inputs, that the calls leave the device's
memory untouched, and that the static scratch's status word reads back clean.  It
runs last in the suite (file name) and passes both alone in a fresh process and
after the other tests.
"""

import ctypes

import numpy as np
import pytest
import torch

from _golden import case, load
from submission_folder_b200 import _lib, ops
from submission_folder_b200.cluster import CircuitKVCluster, cli_cluster_kwargs

pytestmark = pytest.mark.gpu

SCORE_RTOL = 1e-3   # the score tolerance of the parity tests (results here are bit-identical)


def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _noalloc_twice(lib, p, n, a, b, c, ref_idx, ref_sc, dev):
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    outs = [(torch.full_like(ref_idx, -1), torch.full_like(ref_sc, -1.0)) for _ in range(3)]
    torch.cuda.synchronize()
    cptr = None if c is None else c.data_ptr()
    # the first call may load the library's module (and with it the static array)
    rc = lib.ckv_select_scores_noalloc(ctypes.byref(p), n, a.data_ptr(), b.data_ptr(), cptr,
                                       outs[0][0].data_ptr(), outs[0][1].data_ptr(), stream)
    assert rc == 0, lib.ckv_last_error_string()
    torch.cuda.synchronize()
    free0, alloc0 = torch.cuda.mem_get_info(dev)[0], torch.cuda.memory_allocated(dev)
    for idx, sc in outs[1:]:
        rc = lib.ckv_select_scores_noalloc(ctypes.byref(p), n, a.data_ptr(), b.data_ptr(), cptr,
                                           idx.data_ptr(), sc.data_ptr(), stream)
        assert rc == 0, lib.ckv_last_error_string()
        torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(dev)[0] == free0, "the calls changed the device's free memory"
    assert torch.cuda.memory_allocated(dev) == alloc0
    status = ctypes.c_int32(-1)
    assert lib.ckv_read_status(None, stream, ctypes.byref(status)) == 0
    assert status.value == 0
    for idx, sc in outs:
        assert torch.equal(idx, ref_idx)
        torch.testing.assert_close(sc, ref_sc, rtol=SCORE_RTOL, atol=0.0)


@pytest.mark.parametrize("name,keys", [("bf16_n2048_default", ("qi", "hi")),
                                       ("bf16_n8192_cfg2", ("qi", "hi")),
                                       ("bf16_union", ("union_qi", "union_hi"))])
def test_noalloc_matches_workspace_entry(name, keys):
    dev = _cuda()
    lib = _lib.load()
    c = case(name)
    g = load(name)
    p = CircuitKVCluster(**c["kwargs"]).params(c["n"])
    n = c["n"]
    a = torch.from_numpy(np.ascontiguousarray(g[keys[0]])).to(dev)
    b = torch.from_numpy(np.ascontiguousarray(g[keys[1]])).to(dev)
    ref_idx, ref_sc = ops.select_scores(p, a, b, want_scores=True)
    _noalloc_twice(lib, p, n, a, b, None, ref_idx, ref_sc, dev)


def test_noalloc_at_the_size_limit_with_bridge_vector():
    """n = 32768, the largest size the static array holds, with the third (bridge
    importance) vector, which fills every part of the selection area."""
    dev = _cuda()
    lib = _lib.load()
    n = 32768
    rng = np.random.default_rng(7)
    a, b, c = (torch.from_numpy(rng.random(n).astype(np.float32)).to(dev) for _ in range(3))
    p = CircuitKVCluster(**cli_cluster_kwargs(64, 2048, use_bridge_importance=True)).params(n)
    assert p.use_bridge_importance == 1
    ref_idx, ref_sc = ops.select_scores(p, a, b, c, want_scores=True)
    _noalloc_twice(lib, p, n, a, b, c, ref_idx, ref_sc, dev)


def test_noalloc_rejects_oversized_n_and_unsupported_modes():
    dev = _cuda()
    lib = _lib.load()
    p = _lib.default_params()
    n = 32769
    a = torch.zeros(n, dtype=torch.float32, device=dev)
    idx = torch.zeros(2048, dtype=torch.int32, device=dev)
    rc = lib.ckv_select_scores_noalloc(ctypes.byref(p), n, a.data_ptr(), a.data_ptr(), None,
                                       idx.data_ptr(), None, None)
    assert rc == _lib.CKV_OK - 1
    assert b"32768" in lib.ckv_last_error_string()
    p.combination_mode = 2   # weighted
    rc = lib.ckv_select_scores_noalloc(ctypes.byref(p), 4096, a.data_ptr(), a.data_ptr(), None,
                                       idx.data_ptr(), None, None)
    assert rc == -3
