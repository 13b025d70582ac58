"""The workspace-free selection entry point, ckv_select_scores_noalloc.

It exists for callers that cannot give this library device memory -- a serving
engine that reserved nearly all HBM for its KV-cache pool at start-up, or a C /
FFI caller with no device allocator -- and keeps its scratch in a static device
array inside the library (n <= 32768).  This test calls it through the C ABI and
checks that two calls in a row return exactly what the workspace entry point
(ckv_select_scores) returns on the same inputs.  It runs last in the suite (file
name) and passes both alone in a fresh process and after the other tests.
"""

import ctypes

import numpy as np
import pytest
import torch

from _golden import case, load
from submission_folder_b200 import _lib, ops
from submission_folder_b200.cluster import CircuitKVCluster

pytestmark = pytest.mark.gpu

SCORE_RTOL = 1e-3   # the score tolerance of the parity tests (results here are bit-identical)


def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


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
    torch.cuda.synchronize()
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    for _ in range(2):
        idx = torch.full_like(ref_idx, -1)
        sc = torch.full_like(ref_sc, -1.0)
        rc = lib.ckv_select_scores_noalloc(ctypes.byref(p), n, a.data_ptr(), b.data_ptr(), None,
                                           idx.data_ptr(), sc.data_ptr(), stream)
        assert rc == 0, lib.ckv_last_error_string()
        torch.cuda.synchronize()
        assert torch.equal(idx, ref_idx)
        torch.testing.assert_close(sc, ref_sc, rtol=SCORE_RTOL, atol=0.0)


def test_noalloc_rejects_oversized_n():
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
