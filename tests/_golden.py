"""Golden-fixture access and tie-aware comparisons shared by the tests."""

from __future__ import annotations

import json
import os

import numpy as np

import ckv_oracle as O
from submission_folder_b200.synth import make_layer

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def cases():
    with open(os.path.join(GOLDEN, "cases.json")) as f:
        return json.load(f)["cases"]


def case(name):
    for c in cases():
        if c["name"] == name:
            return c
    raise KeyError(name)


def load(name):
    return dict(np.load(os.path.join(GOLDEN, name + ".npz")))


def inputs(c, device="cpu"):
    """Regenerate the case's (q [H,n,D], k [Hkv,n,D], v [Hkv,n,D]) torch tensors."""
    return make_layer(c["n"], seed=c["seed"], window=c["window"], planted=c["planted"],
                      qk_scale=c["qk_scale"], dtype=c["dtype"], device=device)


def oracle_params(c) -> O.Params:
    kw = {k: v for k, v in c["kwargs"].items() if k in O.Params.__dataclass_fields__}
    return O.Params(**kw)


def kth_value(combined, lo, hi, kk):
    cand = np.asarray(combined[lo:hi], dtype=np.float64)
    return np.sort(cand)[::-1][kk - 1]


def compare_keep(ours, ref, combined, lo, hi, kk, margin=0.0):
    """Kept sets equal, or differing only at positions whose combined score is within
    `margin` of the k-th value (margin 0: exact ties).  Returns (n_diff, ok)."""
    a, b = set(np.asarray(ours).tolist()), set(np.asarray(ref).tolist())
    if a == b:
        return 0, True
    if len(a) != len(b):
        return len(a ^ b), False
    t = kth_value(combined, lo, hi, kk)
    diff = a ^ b
    ok = all(abs(float(combined[i]) - t) <= margin + 1e-12 for i in diff)
    return len(diff), ok
