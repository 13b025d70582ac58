"""The C ABI library: it loads, exports every declared entry point, and its host-side
logic (plans, sizes, argument checks) works without a GPU."""

import ctypes
import os
import re

import pytest

from submission_folder_b200 import _lib
from submission_folder_b200.cluster import CircuitKVCluster, cli_cluster_kwargs

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    src = open(os.path.join(ROOT, "include", "ckv.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ckv_[a-z_]+)\s*\(", src)))


def test_library_exports_every_declared_function():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 12
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(_lib.EXPORTED)


def test_version_and_defaults():
    assert _lib.version().startswith("circuitkv-b200")
    p = _lib.default_params()
    assert (p.window_size, p.max_capacity_prompt, p.sink_size, p.neumann_iterations) == (64, 2048, 4, 10)
    assert p.entropy_aware == 1 and p.top_k_heads == 10 and abs(p.hi_mass_threshold - 0.5) < 1e-7
    assert (p.qi_kernel_size, p.hi_kernel_size, p.use_gaussian) == (3, 5, 1)


def test_output_len_and_workspace():
    lib = _lib.load()
    p = _lib.default_params()
    out = ctypes.c_int32()
    assert lib.ckv_output_len(ctypes.byref(p), 32768, ctypes.byref(out)) == 0
    assert out.value == 2048
    # shorter than the budget: the reference returns everything
    assert lib.ckv_output_len(ctypes.byref(p), 1000, ctypes.byref(out)) == 0
    assert out.value == 1000
    sz = ctypes.c_size_t()
    assert lib.ckv_workspace_size(ctypes.byref(p), 32768, 32, 8, 128, ctypes.byref(sz)) == 0
    assert 8 << 20 < sz.value < 256 << 20
    big = ctypes.c_size_t()
    assert lib.ckv_workspace_size(ctypes.byref(p), 131072, 32, 8, 128, ctypes.byref(big)) == 0
    assert big.value > sz.value


@pytest.mark.parametrize("field,value", [("neumann_iterations", 0), ("neumann_iterations", 17),
                                         ("window_size", 0), ("window_size", 256)])
def test_bad_params_rejected(field, value):
    lib = _lib.load()
    p = _lib.default_params()
    setattr(p, field, value)
    sz = ctypes.c_size_t()
    rc = lib.ckv_workspace_size(ctypes.byref(p), 32768, 32, 8, 128, ctypes.byref(sz))
    assert rc < 0
    assert lib.ckv_last_error_string()


def test_bad_shapes_rejected():
    lib = _lib.load()
    p = _lib.default_params()
    sz = ctypes.c_size_t()
    assert lib.ckv_workspace_size(ctypes.byref(p), 32768, 32, 7, 128, ctypes.byref(sz)) == _lib.CKV_OK - 1
    assert lib.ckv_workspace_size(ctypes.byref(p), 32768, 32, 8, 64, ctypes.byref(sz)) < 0


def test_null_arguments_rejected_without_gpu():
    lib = _lib.load()
    p = _lib.default_params()
    assert lib.ckv_score_evict(ctypes.byref(p), None, None, 0, None, None) < 0
    assert lib.ckv_select_scores(ctypes.byref(p), 4096, None, None, None, None, 0, None, None, None) < 0
    assert b"null" in lib.ckv_last_error_string()


def test_cluster_params_follow_reference_kwargs():
    cl = CircuitKVCluster(**cli_cluster_kwargs(64, 2048))
    p = cl.params(32768)
    assert p.combination_mode == _lib.COMB_CODES["dis"] and p.entropy_aware == 1
    assert p.hi_pooling_mode == 0 and p.head_selection_mode == 0
    cl2 = CircuitKVCluster(combination_mode="geometric")
    assert cl2.params(4096).combination_mode == _lib.COMB_CODES["max"]
    cl3 = CircuitKVCluster(max_capacity_prompt=0.25)
    assert cl3.params(8192).max_capacity_prompt == 2048
    cl4 = CircuitKVCluster(qi_gamma=None, neumann_gamma=0.9)
    assert abs(cl4.qi_gamma - 0.9) < 1e-12


def test_init_circuitkv_defaults():
    from submission_folder_b200.cluster import init_circuitkv

    class Cfg:
        pass

    class Attn:
        config = Cfg()

    a = Attn()
    init_circuitkv(a)
    kv = a.kv_cluster
    assert kv.window_size == 64 and kv.max_capacity_prompt == 2048 and kv.max_steps == 50
    assert kv.combination_mode == "dis" and kv.entropy_aware is False and kv.top_k_heads == 8
