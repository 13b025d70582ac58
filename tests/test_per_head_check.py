"""The per-head parity check itself, on the CPU: the oracle's own outputs pass it, and kept
sets with a planted difference away from the kept boundary, or a wrong vector, fail it."""

import numpy as np
import pytest

import ckv_oracle as O
from _golden import check_per_head
from submission_folder_b200.synth import make_layer


def _case(n=1500, W=32, dtype="bf16"):
    q, k, _ = make_layer(n, seed=7, window=W, dtype=dtype)
    op = O.Params(window_size=W, max_capacity_prompt=256, per_head_eviction=True, qi_kernel_size=3,
                  hi_kernel_size=5, use_gaussian=True)
    attn = O.window_attention(q.float().numpy(), k.float().numpy(), W, 4, dtype)
    vec, ent = O.per_head_vectors(attn, op, n)
    return attn, op, vec, ent, n


def test_refactored_selection_is_the_same():
    attn, op, vec, ent, n = _case()
    assert np.array_equal(O.per_head_select(attn, op, n), O.per_head_select_from(vec, ent, op, n))


def test_oracle_outputs_pass():
    attn, op, vec, ent, n = _case()
    idx = O.per_head_select_from(vec, ent, op, n)
    assert max(check_per_head(idx, vec, ent, attn, op, n)) == 0


def test_planted_selection_error_fails():
    attn, op, vec, ent, n = _case()
    idx = O.per_head_select_from(vec, ent, op, n).copy()
    kept = set(idx[0].tolist())
    idx[0, -1] = next(j for j in range(op.sink_size, n - op.window_size) if j not in kept)
    idx[0] = np.sort(idx[0])
    with pytest.raises(AssertionError):
        check_per_head(idx, vec, ent, attn, op, n)


def test_planted_vector_error_fails():
    attn, op, vec, ent, n = _case()
    bad = vec.copy()
    bad[3, 0, 100] += 0.01 * float(np.abs(vec[3, 0]).max())   # 1% of the vector's scale
    idx = O.per_head_select_from(bad, ent, op, n)
    with pytest.raises(AssertionError):
        check_per_head(idx, bad, ent, attn, op, n)
