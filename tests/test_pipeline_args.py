"""Argument checks of the pipelined host-cache call (no GPU needed: they run first)."""

import pytest
import torch

from submission_folder_b200._lib import Params
from submission_folder_b200.pipeline import score_evict_pipelined


def _layers(n=2):
    q = torch.zeros(32, 256, 128, dtype=torch.bfloat16)
    k = torch.zeros(8, 256, 128, dtype=torch.bfloat16)
    return [(q, k, k)] * n


def test_empty_is_empty():
    assert score_evict_pipelined(Params(), []) == []


def test_params_count_must_match():
    with pytest.raises(ValueError):
        score_evict_pipelined([Params()] * 3, _layers(2))


def test_out_count_must_match():
    with pytest.raises(ValueError):
        score_evict_pipelined(Params(), _layers(2), out=[(torch.zeros(1), torch.zeros(1))])
