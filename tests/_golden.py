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
                      qk_scale=c["qk_scale"], dtype=c["dtype"], device=device,
                      grid_step=c.get("grid_step", 0.0))


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


SCORE_RTOL = 1e-3   # ranked vectors vs the reference's: max abs difference / max |reference|


def ranked_vectors_of_reference(c, g, op):
    """The two vectors the reference ranks (or unions), as recorded in the fixture:
    smoothed QI / HI for "dis", the union inputs for union modes, influence for
    "max" / "weighted" (its H2O partner is not recorded: None)."""
    mode = op.combination_mode
    if mode in ("union", "union_da"):
        return g["union_qi"], g["union_hi"]
    if mode in ("max", "weighted"):
        return g["influence"], None
    qk = op.qi_kernel_size if op.qi_kernel_size != 0 else op.smoothing_kernel
    hk = op.hi_kernel_size if op.hi_kernel_size != 0 else op.smoothing_kernel
    if op.smooth_hi_only and qk > 1:
        qk = 0
    qs = O.smooth(g["qi"], qk, op.use_gaussian, op.gaussian_sigma * 0.5 if op.use_gaussian else 1.0) \
        if qk > 1 else g["qi"]
    hs = O.smooth(g["hi"], hk, op.use_gaussian, op.gaussian_sigma) if hk > 1 else g["hi"]
    return qs, hs


def check_kept(name, idx, sc, ref_keep, ref_combined, ref_a, ref_b, op, n, exact, report):
    """Parity of one layer's kept positions, in three parts.

    1. Index work is exact: ``idx`` equals the reference's selection rule
       (``O.select_from_vectors``: stable ranks, MAX / union, top-k with lowest-index
       ties) applied to the GPU's own ranked vectors ``sc`` [2, n].
    2. The ranked vectors agree with the reference's within SCORE_RTOL.
    3. The kept positions equal the reference's except at exact ties of the k-th combined
       score (the reference's CPU topk orders those in an implementation-defined way; for
       union modes, which record no combined score, they must be equal).  ``exact`` marks
       inputs whose logits are the same bits on every device (``grid_*`` fixtures); the
       figures go to ``report`` either way.
    """
    s, W = op.sink_size, op.window_size
    if not op.use_bridge_importance:
        sel = O.select_from_vectors(sc[0], sc[1], op, n)
        assert np.array_equal(sel, idx), f"{name}: selection differs from the rule on the same vectors"
    errs = []
    for got, ref in ((sc[0], ref_a), (sc[1], ref_b)):
        if ref is not None:
            errs.append(float(np.max(np.abs(got - ref)) / max(float(np.max(np.abs(ref))), 1e-30)))
    assert all(e < SCORE_RTOL for e in errs), (name, errs)
    kk = len(ref_keep) - s
    if ref_combined is not None:
        nd, ties_only = compare_keep(idx, ref_keep, ref_combined, s, n - W, kk)
    else:
        nd = len(set(np.asarray(idx).tolist()) ^ set(np.asarray(ref_keep).tolist()))
        ties_only = nd == 0
    if report is not None:
        report[name] = {"n": int(n), "kept": int(len(ref_keep)), "differ": int(nd),
                        "differ_only_at_exact_ties": bool(ties_only), "score_max_rel_err": errs,
                        "exact_arithmetic_inputs": bool(exact)}
    assert ties_only, f"{name}: {nd} kept positions differ beyond exact ties of the k-th combined score"
    return nd, ties_only


PH_VEC_RTOL = SCORE_RTOL   # per-head vectors vs the oracle's: max abs difference / max |oracle| per head


def check_per_head(idx, vec, ent, attn, op, n, report=None, key=None):
    """Decomposed parity of per-head eviction (PU:3296-3446) against the oracle:

    1. the selection is exact: the oracle's selection rule applied to the device's own ranked
       vectors and entropies gives exactly the device's kept set, head by head;
    2. the device's vectors and entropies equal the oracle's within ``PH_VEC_RTOL``;
    3. the kept sets equal the oracle's, except in a head whose oracle vectors hold a near tie
       at the kept boundary: two values closer than twice the head's measured vector
       difference (so that the device's rounding -- a 16-bit logit rounded after a different
       fp32 accumulation order, a different summation order -- can order them the other
       way), one of them at a position whose oracle score lies within two rank steps of the
       head's k-th score; every differing position must lie within those two rank steps.
    Returns the number of differing positions per head."""
    idx = np.asarray(idx)
    vec = np.asarray(vec, dtype=np.float32)
    ent = np.asarray(ent, dtype=np.float32)
    own = O.per_head_select_from(vec, ent, op, n)
    for h in range(idx.shape[0]):
        assert set(own[h].tolist()) == set(idx[h].tolist()), ("selection not exact", h)
    ovec, oent = O.per_head_vectors(attn, op, n)
    abs_err = np.zeros((ovec.shape[0], 2))
    for h in range(ovec.shape[0]):
        for v in range(2):
            scale = max(float(np.abs(ovec[h, v]).max()), 1e-30)
            abs_err[h, v] = float(np.abs(vec[h, v].astype(np.float64) - ovec[h, v]).max())
            assert abs_err[h, v] / scale <= PH_VEC_RTOL, ("vector", h, v, abs_err[h, v] / scale)
    np.testing.assert_allclose(ent, oent, rtol=PH_VEC_RTOL, atol=1e-6)
    oidx = O.per_head_select_from(ovec, oent, op, n)
    osc = O.per_head_scores_from(ovec, oent, op)
    nw = ovec.shape[2]
    s = op.sink_size
    step = 1.0 / max(nw - 1, 1)
    diffs = []
    for h in range(idx.shape[0]):
        d = set(idx[h].tolist()) ^ set(oidx[h].tolist())
        diffs.append(len(d))
        if not d:
            continue
        kept = [j for j in oidx[h].tolist() if j >= s]
        T = float(osc[h, kept].min())
        near = [j for j in d if abs(float(osc[h, j]) - T) <= 2 * step + 1e-7]
        assert len(near) == len(d), ("difference away from the kept boundary", h, sorted(d), T)
        boundary = np.where(np.abs(osc[h].astype(np.float64) - T) <= 2 * step + 1e-7)[0]
        tie = False
        for v in range(2):
            x = ovec[h, v].astype(np.float64)
            order = np.argsort(x, kind="stable")
            gaps = np.diff(x[order]) <= 2 * abs_err[h, v] + 1e-12
            pairs = set(order[:-1][gaps].tolist()) | set(order[1:][gaps].tolist())
            if pairs & set(boundary.tolist()):
                tie = True
        assert tie, ("difference without a near tie at the kept boundary", h, sorted(d))
    if report is not None and key is not None:
        report[key] = {"n": int(n), "kept_per_head": int(idx.shape[1]), "differ_per_head": diffs}
    return diffs
