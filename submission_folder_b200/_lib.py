"""ctypes binding of ``libckv.so`` (the C ABI declared in ``include/ckv.h``).

The library is built in-tree (``submission_folder_b200/libckv.so``).  There is
no fallback: if the library or a CUDA device is missing, the calls raise.
"""

from __future__ import annotations

import ctypes
import os
from typing import Optional

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libckv.so")

CKV_OK = 0
DTYPE_CODES = {"bf16": 0, "fp16": 1, "fp32": 2}
COMB_CODES = {"dis": 0, "max": 1, "weighted": 2, "union": 3, "union_da": 4}

EXPORTED = (
    "ckv_default_params", "ckv_output_len", "ckv_workspace_size", "ckv_score_evict",
    "ckv_score_evict_batched", "ckv_read_status", "ckv_select_scores", "ckv_select_scores_noalloc",
    "ckv_neumann_rows",
    "ckv_window_pool", "ckv_choose_heads", "ckv_pool_rows_given", "ckv_graph_update", "ckv_circuit_walk",
    "ckv_pcg_seed", "ckv_spectral_scores", "ckv_combine_scores", "ckv_landmark_workspace_size",
    "ckv_landmark_walk", "ckv_influence_walk", "ckv_influence_walk_dense", "ckv_walk_workspace_size",
    "ckv_rng_fill", "ckv_gather", "ckv_device_accessible", "ckv_copy_rows", "ckv_set_stage_events", "ckv_last_error_string",
    "ckv_version",
)
RNG_PHILOX, RNG_PCG = 0, 1
LANDMARK_POSITIONAL, LANDMARK_REACHABILITY, LANDMARK_ABSORBING = 0, 1, 2


class Params(ctypes.Structure):
    """Mirror of ``struct ckv_params``."""

    _fields_ = [
        ("window_size", ctypes.c_int32),
        ("max_capacity_prompt", ctypes.c_int32),
        ("sink_size", ctypes.c_int32),
        ("neumann_iterations", ctypes.c_int32),
        ("neumann_temperature", ctypes.c_float),
        ("neumann_gamma", ctypes.c_float),
        ("qi_gamma", ctypes.c_float),
        ("hi_gamma", ctypes.c_float),
        ("combination_mode", ctypes.c_int32),
        ("h2o_weight", ctypes.c_float),
        ("qi_ratio", ctypes.c_float),
        ("ablate_qi", ctypes.c_int32),
        ("ablate_hi", ctypes.c_int32),
        ("per_head_eviction", ctypes.c_int32),
        ("true_hub_hi", ctypes.c_int32),
        ("entropy_adaptive", ctypes.c_int32),
        ("smoothing_kernel", ctypes.c_int32),
        ("smooth_hi_only", ctypes.c_int32),
        ("use_gaussian", ctypes.c_int32),
        ("qi_kernel_size", ctypes.c_int32),
        ("hi_kernel_size", ctypes.c_int32),
        ("gaussian_sigma", ctypes.c_float),
        ("entropy_aware", ctypes.c_int32),
        ("top_k_heads", ctypes.c_int32),
        ("head_selection_mode", ctypes.c_int32),
        ("hi_pooling_mode", ctypes.c_int32),
        ("hi_mass_threshold", ctypes.c_float),
        ("hi_top_k_heads", ctypes.c_int32),
        ("hi_mass_cdf", ctypes.c_float),
        ("use_bridge_importance", ctypes.c_int32),
        ("bi_kernel_size", ctypes.c_int32),
    ]


class Layer(ctypes.Structure):
    """Mirror of ``struct ckv_layer``."""

    _fields_ = [
        ("q", ctypes.c_void_p), ("q_head_stride", ctypes.c_int64), ("q_tok_stride", ctypes.c_int64),
        ("k", ctypes.c_void_p), ("k_head_stride", ctypes.c_int64), ("k_tok_stride", ctypes.c_int64),
        ("v", ctypes.c_void_p), ("v_head_stride", ctypes.c_int64), ("v_tok_stride", ctypes.c_int64),
        ("n", ctypes.c_int32), ("num_heads", ctypes.c_int32), ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32), ("dtype", ctypes.c_int32),
    ]


class Outputs(ctypes.Structure):
    """Mirror of ``struct ckv_outputs``."""

    _fields_ = [
        ("out_k", ctypes.c_void_p), ("out_v", ctypes.c_void_p),
        ("out_idx", ctypes.c_void_p), ("out_scores", ctypes.c_void_p),
        ("distinct_kv_heads", ctypes.c_int32),
    ]


_lib: Optional[ctypes.CDLL] = None


class CKVError(RuntimeError):
    """A ckv_* entry point returned a non-zero status."""


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load (once) and type the C ABI; raises if the built library is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(
            f"libckv.so not found at {path}; build it with "
            "`python -m submission_folder_b200.build` (nvcc, sm_100a)")
    lib = ctypes.CDLL(path)
    vp, sz, i32, f32, u64 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int32, ctypes.c_float, ctypes.c_uint64
    P, L, O = ctypes.POINTER(Params), ctypes.POINTER(Layer), ctypes.POINTER(Outputs)
    sig = {
        "ckv_default_params": (None, [P]),
        "ckv_output_len": (i32, [P, i32, ctypes.POINTER(i32)]),
        "ckv_workspace_size": (i32, [P, i32, i32, i32, i32, ctypes.POINTER(sz)]),
        "ckv_score_evict": (i32, [P, L, vp, sz, O, vp]),
        "ckv_score_evict_batched": (i32, [P, i32, L, i32, vp, sz, O, vp]),
        "ckv_read_status": (i32, [vp, vp, ctypes.POINTER(i32)]),
        "ckv_select_scores": (i32, [P, i32, vp, vp, vp, vp, sz, vp, vp, vp]),
        "ckv_select_scores_noalloc": (i32, [P, i32, vp, vp, vp, vp, vp, vp]),
        "ckv_neumann_rows": (i32, [P, i32, vp, vp, i32, vp, sz, vp, vp, vp, vp]),
        "ckv_window_pool": (i32, [P, L, vp, sz, vp, vp, vp, vp, vp, vp, vp]),
        "ckv_choose_heads": (i32, [P, i32, vp, vp, vp, vp, vp]),
        "ckv_graph_update": (i32, [vp, vp, i32, i32, i32, i32, i32, vp, vp, vp, vp]),
        "ckv_circuit_walk": (i32, [vp, vp, i32, i32, i32, i32, vp, vp, i32, vp]),
        "ckv_pcg_seed": (i32, [u64, i32, vp, vp]),
        "ckv_spectral_scores": (i32, [vp, vp, i32, i32, i32, vp, vp, vp]),
        "ckv_combine_scores": (i32, [vp, vp, vp, vp, i32, vp]),
        "ckv_landmark_workspace_size": (i32, [i32, ctypes.POINTER(sz)]),
        "ckv_landmark_walk": (i32, [vp, i32, i32, i32, i32, i32, f32, i32, f32, i32, vp, vp, vp, vp, vp, vp, sz,
                                    vp]),
        "ckv_pool_rows_given": (i32, [P, L, i32, vp, vp, vp, sz, vp, vp, vp]),
        "ckv_influence_walk": (i32, [vp, i32, i32, i32, i32, i32, i32, i32, f32, f32, f32, i32, u64,
                                     vp, i32, vp, sz, vp, vp, vp, vp]),
        "ckv_influence_walk_dense": (i32, [vp, i32, i32, i32, i32, i32, f32, f32, f32, i32, u64, vp, i32,
                                           vp, vp, vp]),
        "ckv_walk_workspace_size": (i32, [i32, i32, ctypes.POINTER(sz)]),
        "ckv_rng_fill": (i32, [i32, u64, u64, i32, vp, vp]),
        "ckv_gather": (i32, [L, i32, vp, i32, i32, vp, vp, vp]),
        "ckv_device_accessible": (i32, [vp, ctypes.POINTER(i32)]),
        "ckv_copy_rows": (i32, [vp, sz, vp, sz, sz, i32, vp]),
        "ckv_set_stage_events": (i32, [ctypes.POINTER(vp), i32]),
        "ckv_last_error_string": (ctypes.c_char_p, []),
        "ckv_version": (ctypes.c_char_p, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int, what: str) -> None:
    if status != CKV_OK:
        msg = load().ckv_last_error_string().decode(errors="replace")
        raise CKVError(f"{what} failed with status {status}: {msg}")


def default_params() -> Params:
    p = Params()
    load().ckv_default_params(ctypes.byref(p))
    return p


def version() -> str:
    return load().ckv_version().decode()
