"""The influence-walker oracle pinned on the CPU: generators against published answers
(pcg32) and numpy's Philox4x64-10, the walker restatement against the exact expectation
of its visit counts, the positional normalisation, and the ``circuit_kv._C`` mirror's
argument checks (which run before any device work)."""

import numpy as np
import pytest

import ckv_walker_oracle as W


def test_pcg32_known_answer():
    # pcg32_srandom_r(42, 54): the first outputs printed by the PCG reference demo
    g = W.Pcg32(42, 54)
    assert [g.next() for _ in range(6)] == [0xa15c02b7, 0x7b47f409, 0xba1d3330, 0x83d2f293,
                                            0xbfa4784b, 0xcbed606e]


def _numpy_philox(seed, stream, count):
    # numpy advances the 256-bit counter before each block: start one below (0, stream)
    bg = np.random.Philox(key=seed, counter=((stream << 64) - 1) % (1 << 256))
    return [int(x) for x in bg.random_raw(4 * ((count + 3) // 4))][:count]


@pytest.mark.parametrize("seed,stream,count", [(0, 0, 9), (3042, 1, 16), (2**63 + 5, 7, 13), (1, 2**40, 4)])
def test_philox_matches_numpy(seed, stream, count):
    assert W.philox_stream(seed, stream, count) == _numpy_philox(seed, stream, count)


def test_pcg_uniform_is_24_bits():
    g = W.Pcg32(7, 3)
    h = W.Pcg32(7, 3)
    for _ in range(50):
        u = g.uniform()
        assert 0.0 <= u < 1.0 and u == np.float32((h.next() >> 8) / 16777216.0)


def _row_stochastic(n, seed, peaked=False):
    rng = np.random.default_rng(seed)
    a = rng.random((n, n)).astype(np.float32)
    if peaked:
        a = a ** 8
    a = np.tril(a)
    return (a / a.sum(axis=1, keepdims=True)).astype(np.float32)


@pytest.mark.parametrize("temps", [(2.0, 10.0, 0.3), (1.0, 1.0, 0.0), (0.5, 4.0, 1.0)])
def test_walker_oracle_matches_expectation(temps):
    n, walkers, steps, sink = 48, 3000, 6, 4
    A = _row_stochastic(n, 1, peaked=True)
    t, te, r = temps
    _, visits, _ = W.influence_walk_dense(A, n - 1, walkers, steps, sink, t, te, r)
    exp = W.expected_visits(A, n - 1, walkers, steps, sink, t, te, r)
    assert visits.sum() == walkers * steps      # every step lands on a non-sink position
    assert np.abs(visits - exp).sum() / exp.sum() < 0.05


def test_walker_states_carry_over():
    A = _row_stochastic(32, 2)
    _, v1, gens = W.influence_walk_dense(A, 31, 200, 5, 4)
    _, v2, _ = W.influence_walk_dense(A, 31, 200, 5, 4, gens=gens)
    _, v3, _ = W.influence_walk_dense(A, 31, 200, 5, 4)
    assert np.array_equal(v1, v3) and not np.array_equal(v1, v2)


def test_normalise():
    v = np.array([5, 5, 1, 2, 8, 0, 3], dtype=np.float32)
    s = W.normalise(v, 2)
    adj = v / np.sqrt(7 - np.arange(7) + 1.0)
    assert np.all(s[:2] == 1.0)
    np.testing.assert_allclose(s[2:], adj[2:] / adj[2:].max(), rtol=1e-6)
    assert np.all(W.normalise(np.zeros(5, np.float32), 1)[1:] == 0.0)


def test_normalise_max_covers_first_65536_positions():
    n = 70000
    v = np.zeros(n, dtype=np.float32)
    v[100] = 1.0
    v[69000] = 1000.0       # beyond the 256 x 256 positions the reference reduces over
    s = W.normalise(v, 4)
    assert s[100] == 1.0 and s[69000] > 1.0


def test_circuit_graph_argument_checks():
    from submission_folder_b200.circuit_kv import _C
    for args in [(0, 8, 0.85, 100, 10), (100, 0, 0.85, 100, 10), (100, 65, 0.85, 100, 10),
                 (100, 8, 0.85, 0, 10)]:
        with pytest.raises(RuntimeError):
            _C.CircuitGraph(*args)


def test_philox_walker_draws_follow_the_stream_layout():
    """A walker's counter-based draws are the top 24 bits of its Philox stream (call 0:
    the same counters as ckv_rng_fill's stream = walker)."""
    for w in (0, 5, 1234):
        g = W.PhiloxWalker(7, w)
        raw = W.philox_stream(7, w, 9)
        for d in range(9):
            assert g.uniform() == np.float32(raw[d] >> 40) * np.float32(1.0 / 16777216.0)
