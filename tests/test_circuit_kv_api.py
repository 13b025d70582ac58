"""The ``circuit_kv`` package keeps the reference's public names, config fields and
defaults (CircuitKV/circuit_kv/__init__.py:14-28, engine.py:20-81), and the
monitors' host logic (prefill charge, keep mask) behaves like the reference's."""

import dataclasses

import pytest
import torch

REFERENCE_ALL = ["CircuitKVMonitor", "CircuitKVConfig", "LandmarkWalkerMonitor", "LandmarkWalkerConfig",
                 "set_seed"]


def test_star_import_has_reference_names():
    ns = {}
    exec("from submission_folder_b200.circuit_kv import *", ns)
    for name in REFERENCE_ALL:
        assert name in ns, name
    import submission_folder_b200.circuit_kv as ck
    assert list(ck.__all__) == REFERENCE_ALL
    assert callable(ck.get_extension) and ck.get_extension() is ck._C


def test_config_fields_and_defaults():
    from submission_folder_b200.circuit_kv import CircuitKVConfig, LandmarkWalkerConfig
    c = CircuitKVConfig()
    assert [f.name for f in dataclasses.fields(c)] == [
        "max_seq_len", "top_k", "num_walkers", "alpha", "num_steps", "sink_size", "local_window", "decay",
        "device", "dtype"]
    assert (c.max_seq_len, c.top_k, c.num_walkers, c.alpha, c.num_steps) == (8192, 32, 1024, 0.85, 100)
    assert (c.sink_size, c.local_window, c.decay, c.device, c.dtype) == (4, 64, 0.95, "cuda", torch.float16)
    lw = LandmarkWalkerConfig()
    assert [f.name for f in dataclasses.fields(lw)] == [
        "max_seq_len", "top_k", "num_landmarks", "min_spacing", "walkers_per_source", "query_boost",
        "use_reachability", "position_alpha", "sink_size", "local_window", "device"]
    assert (lw.num_landmarks, lw.min_spacing, lw.walkers_per_source, lw.query_boost) == (32, 50, 100, 2.0)
    assert (lw.use_reachability, lw.position_alpha, lw.sink_size, lw.local_window) == (False, 0.6, 4, 64)


def test_keep_mask_forces_sinks_and_window():
    from submission_folder_b200.circuit_kv.engine import _keep_mask
    s = torch.arange(100, dtype=torch.float32).flip(0)   # earlier positions score higher
    m = _keep_mask(s, 0.25, 100, 4, 10)
    assert m.sum().item() == 25
    assert m[:4].all() and m[90:].all()
    assert m[4:15].all() and not m[15:90].any()


@pytest.mark.gpu
def test_monitor_prefill_charge_and_mask():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from submission_folder_b200.circuit_kv import CircuitKVConfig, CircuitKVMonitor
    mon = CircuitKVMonitor(CircuitKVConfig(max_seq_len=256))
    a = torch.rand(128, 128, device="cuda")
    mon.initialize_from_prefill(a)
    cs = a.sum(0)
    torch.testing.assert_close(mon.get_scores()[:128], cs / cs.max())
    m = mon.get_keep_mask(0.75, 128)
    assert m.sum().item() == 96 and m[:4].all() and m[64:].all()
    mon.reset()
    assert mon._accumulated_charge is None
