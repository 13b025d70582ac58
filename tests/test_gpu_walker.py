"""The influence walker of the use_neumann=False path on the GPU (through the C ABI):

* generators: the raw Philox4x64-10 and pcg32 outputs equal the oracle's (bit-exact);
* the dense walker, PCG-seeded like the reference, gives the reference's own walker
  kernel's visit counts and PCG states bit for bit (that kernel compiled from its
  source into oracle/_ref), and scores within 2e-6 relative (the reference divides and
  takes square roots with fast-math approximations);
* without that library: the dense walker against the oracle walker (same PCG draws;
  the oracle's float32 power may differ from __powf by an ulp, so visit counts agree
  to 0.5% in L1);
* Philox walkers and the structured walker (prefix rows sampled by binary search)
  against the exact expectation of the visit counts (5% in L1 at 10^5 steps) and the
  structured walker against the dense walker on the materialised matrix (2% in L1);
* the ``circuit_kv._C.CircuitGraph`` mirror and the hook's use_neumann=False path.
"""

import ctypes
import os

import numpy as np
import pytest
import torch

import ckv_oracle as O
import ckv_walker_oracle as WO
from _golden import case, inputs
from submission_folder_b200 import _lib, ops
from submission_folder_b200.circuit_kv import _C
from submission_folder_b200.cluster import CircuitKVCluster

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_SO = os.path.join(ROOT, "oracle", "_ref", "libref_walker.so")


def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _u64(t: torch.Tensor):
    return [int(x) & ((1 << 64) - 1) for x in t.cpu().tolist()]


def _row_stochastic(n, seed, peaked=True):
    rng = np.random.default_rng(seed)
    a = rng.random((n, n)).astype(np.float32)
    if peaked:
        a = a ** 8
    a = np.tril(a)
    return (a / a.sum(axis=1, keepdims=True)).astype(np.float32)


def _pooled_rows(n, W, seed):
    """Causal, row-stochastic pooled window rows [W, n] (row r: position n - W + r)."""
    rng = np.random.default_rng(seed)
    logits = rng.standard_normal((W, n)).astype(np.float32) * 2.0
    logits[:, :4] += 4.0
    for r in range(W):
        logits[r, n - W + r + 1:] = -np.inf
    e = np.exp(logits - logits.max(axis=1, keepdims=True))
    return (e / e.sum(axis=1, keepdims=True)).astype(np.float32)


def _l1(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.abs(a - b).sum() / max(b.sum(), 1.0)


# ---- generators ---------------------------------------------------------------------
@pytest.mark.parametrize("seed,stream,count", [(0, 0, 9), (3042, 1, 64), (2**63 + 5, 7, 13)])
def test_rng_fill_philox(seed, stream, count):
    dev = _cuda()
    out = ops.rng_fill(_lib.RNG_PHILOX, seed, stream, count, dev)
    assert _u64(out) == WO.philox_stream(seed, stream, count)


@pytest.mark.parametrize("seed,stream,count", [(42, 54, 6), (3042, 9999, 40)])
def test_rng_fill_pcg(seed, stream, count):
    dev = _cuda()
    out = ops.rng_fill(_lib.RNG_PCG, seed, stream, count, dev)
    assert _u64(out) == WO.pcg_stream(seed, stream, count)


# ---- dense walker against the reference's own kernel ----------------------------------
def _ref_lib():
    if not os.path.exists(REF_SO):
        pytest.skip("oracle/_ref/libref_walker.so not built (needs the reference source)")
    lib = ctypes.CDLL(REF_SO)
    f = lib.ref_influence_walk
    i32, f32, vp = ctypes.c_int32, ctypes.c_float, ctypes.c_void_p
    f.argtypes = [vp, i32, i32, i32, i32, i32, f32, f32, f32, vp, vp, vp, vp, vp]
    f.restype = ctypes.c_int
    return f


def _ref_walk(f, A, cur, walkers, steps, sink, t, te, r, states):
    n = A.shape[0]
    dev = A.device
    visits = torch.empty(n, dtype=torch.float32, device=dev)
    norm = torch.empty(n, dtype=torch.float32, device=dev)
    pmax = torch.empty(256, dtype=torch.float32, device=dev)
    rc = f(A.data_ptr(), n, cur, walkers, steps, sink, t, te, r, states.data_ptr(), visits.data_ptr(),
           norm.data_ptr(), pmax.data_ptr(), ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    assert rc == 0
    return norm, visits


@pytest.mark.parametrize("n,cur,walkers,steps,sink,temps", [
    (512, 511, 10000, 10, 4, (2.0, 10.0, 0.3)),
    (700, 650, 4096, 50, 4, (2.0, 10.0, 0.3)),
    (4096, 4095, 10000, 10, 4, (1.0, 5.0, 0.5)),
    (300, 3, 1000, 10, 4, (2.0, 10.0, 0.3)),          # query inside the sinks: no walk
    (256, 200, 999, 7, 0, (0.1, 100.0, 1.0)),
])
def test_dense_walker_matches_reference_kernel(n, cur, walkers, steps, sink, temps):
    dev = _cuda()
    f = _ref_lib()
    t, te, r = temps
    A = torch.from_numpy(_row_stochastic(n, n + walkers)).to(dev)
    st0 = torch.from_numpy(WO.states_array(WO.seed_states(3042, walkers))).to(dev)
    st_ref, st_ours = st0.clone(), st0.clone()
    for call in range(2):        # the second call continues the states of the first
        s_ref, v_ref = _ref_walk(f, A, cur, walkers, steps, sink, t, te, r, st_ref)
        s_ours, v_ours = ops.influence_walk_dense(A, cur, walkers, steps, sink, t, te, r, rng_mode=_lib.RNG_PCG,
                                                  seed=3042, rng_state=st_ours, init_state=False)
        torch.cuda.synchronize()
        assert torch.equal(v_ours, v_ref), f"call {call}: visit counts differ"
        assert torch.equal(st_ours, st_ref), f"call {call}: PCG states differ"
        torch.testing.assert_close(s_ours, s_ref, rtol=2e-6, atol=0)


def test_dense_walker_seeding_matches_reference_init():
    """init_state=1 seeds walker w with pcg_init(seed, w) like init_rng_kernel."""
    dev = _cuda()
    f = _ref_lib()
    n, walkers = 256, 3000
    A = torch.from_numpy(_row_stochastic(n, 3)).to(dev)
    st_ref = torch.from_numpy(WO.states_array(WO.seed_states(3042, walkers))).to(dev)
    st_ours = torch.zeros(2 * walkers, dtype=torch.int64, device=dev)
    _, v_ref = _ref_walk(f, A, n - 1, walkers, 10, 4, 2.0, 10.0, 0.3, st_ref)
    _, v_ours = ops.influence_walk_dense(A, n - 1, walkers, 10, 4, seed=3042, rng_state=st_ours, init_state=True)
    torch.cuda.synchronize()
    assert torch.equal(v_ours, v_ref) and torch.equal(st_ours, st_ref)


# ---- dense walker against the oracle walker -----------------------------------------
@pytest.mark.parametrize("temps", [(2.0, 10.0, 0.3), (0.5, 3.0, 0.6)])
def test_dense_walker_matches_oracle(temps):
    dev = _cuda()
    n, walkers, steps, sink = 64, 1500, 6, 4
    t, te, r = temps
    A = _row_stochastic(n, 11)
    gens = WO.seed_states(3042, walkers)
    _, v_or, gens = WO.influence_walk_dense(A, n - 1, walkers, steps, sink, t, te, r, gens=gens)
    st = torch.zeros(2 * walkers, dtype=torch.int64, device=dev)
    s_g, v_g = ops.influence_walk_dense(torch.from_numpy(A).to(dev), n - 1, walkers, steps, sink, t, te, r,
                                        seed=3042, rng_state=st, init_state=True)
    torch.cuda.synchronize()
    assert v_g.sum().item() == walkers * steps
    assert _l1(v_g.cpu().numpy(), v_or) < 5e-3
    np.testing.assert_allclose(s_g.cpu().numpy(), WO.normalise(v_g.cpu().numpy(), sink), rtol=1e-6)
    # every walker drew the same number of uniforms, so the states agree exactly
    assert np.array_equal(st.cpu().numpy(), WO.states_array(gens))


# ---- Philox walkers -------------------------------------------------------------------
def test_philox_walker_statistics_and_counter():
    dev = _cuda()
    n, walkers, steps, sink = 96, 10000, 10, 4
    A = _row_stochastic(n, 5)
    At = torch.from_numpy(A).to(dev)
    st = torch.zeros(1, dtype=torch.int64, device=dev)
    _, v1 = ops.influence_walk_dense(At, n - 1, walkers, steps, sink, rng_mode=_lib.RNG_PHILOX, seed=7,
                                     rng_state=st, init_state=True)
    v1 = v1.clone()
    assert st.item() == 1
    _, v2 = ops.influence_walk_dense(At, n - 1, walkers, steps, sink, rng_mode=_lib.RNG_PHILOX, seed=7,
                                     rng_state=st, init_state=False)
    v2 = v2.clone()
    assert st.item() == 2 and not torch.equal(v1, v2)
    _, v3 = ops.influence_walk_dense(At, n - 1, walkers, steps, sink, rng_mode=_lib.RNG_PHILOX, seed=7,
                                     rng_state=None)
    torch.cuda.synchronize()
    assert torch.equal(v1, v3)           # a fresh counter repeats the first call
    exp = WO.expected_visits(A, n - 1, walkers, steps, sink)
    assert _l1(v1.cpu().numpy(), exp) < 0.05
    assert _l1(v2.cpu().numpy(), exp) < 0.05


@pytest.mark.parametrize("n,steps", [(96, 10), (700, 20)])
def test_philox_warp_walker_matches_oracle_draws(n, steps):
    """The dense walker in Philox mode (one warp per walker, coalesced row reads, warp
    scans) against the oracle walker fed the same counter-based draws: the walks are the
    same except where a running sum crosses the target within fp32 rounding."""
    dev = _cuda()
    walkers, sink = 4000, 4
    A = _row_stochastic(n, 17)
    _, v_or, _ = WO.influence_walk_dense(A, n - 1, walkers, steps, sink, gens=WO.philox_walkers(7, walkers))
    _, v_g = ops.influence_walk_dense(torch.from_numpy(A).to(dev), n - 1, walkers, steps, sink,
                                      rng_mode=_lib.RNG_PHILOX, seed=7, rng_state=None)
    torch.cuda.synchronize()
    v_g = v_g.cpu().numpy()
    assert v_g.sum() == v_or.sum()
    assert _l1(v_g, v_or) < 2e-3


# ---- structured walker ----------------------------------------------------------------
@pytest.mark.parametrize("n,W,cur_off,mode", [(300, 64, 1, _lib.RNG_PCG), (300, 64, 1, _lib.RNG_PHILOX),
                                              (200, 32, 60, _lib.RNG_PCG), (130, 64, 1, _lib.RNG_PCG)])
def test_structured_walker_matches_dense(n, W, cur_off, mode):
    dev = _cuda()
    walkers, steps, sink = 10000, 10, 4
    cur = n - cur_off
    rows = _pooled_rows(n, W, n + W)
    A = O.build_full_attn(rows)
    st_a = torch.zeros(2 * walkers, dtype=torch.int64, device=dev)
    st_b = torch.zeros(2 * walkers, dtype=torch.int64, device=dev)
    s_s, v_s, h2o = ops.influence_walk(torch.from_numpy(rows).to(dev), cur, walkers, steps, sink, rng_mode=mode,
                                       rng_state=st_a, init_state=True)
    s_d, v_d = ops.influence_walk_dense(torch.from_numpy(A).to(dev), cur, walkers, steps, sink, rng_mode=mode,
                                        rng_state=st_b, init_state=True)
    torch.cuda.synchronize()
    v_s, v_d = v_s.cpu().numpy(), v_d.cpu().numpy()
    assert v_s.sum() == v_d.sum()
    assert _l1(v_s, v_d) < 0.02
    exp = WO.expected_visits(A, cur, walkers, steps, sink)
    assert _l1(v_s, exp) < 0.05
    np.testing.assert_allclose(s_s.cpu().numpy(), WO.normalise(v_s, sink), rtol=1e-6)
    np.testing.assert_allclose(h2o.cpu().numpy(), O.full_attn_colsum(rows), rtol=1e-4, atol=1e-6)


def test_structured_walker_long_sequence():
    """n = 70000 > 65536: the normalisation's maximum covers the first 65536 positions
    only (as the reference's 256 x 256 reduction), and the structured walker agrees with
    the dense one at n = 4096."""
    dev = _cuda()
    n, W = 70000, 64
    rows = torch.from_numpy(_pooled_rows(n, W, 1)).to(dev)
    s, v, h2o = ops.influence_walk(rows, n - 1, 10000, 10, 4)
    torch.cuda.synchronize()
    v = v.cpu().numpy()
    assert v.sum() == 10000 * 10
    np.testing.assert_allclose(s.cpu().numpy(), WO.normalise(v, 4), rtol=1e-6)
    assert torch.isfinite(h2o).all()
    n = 4096
    rows = _pooled_rows(n, W, 2)
    s1, v1, _ = ops.influence_walk(torch.from_numpy(rows).to(dev), n - 1, 10000, 10, 4)
    s2, v2 = ops.influence_walk_dense(torch.from_numpy(O.build_full_attn(rows)).to(dev), n - 1, 10000, 10, 4)
    torch.cuda.synchronize()
    assert _l1(v1.cpu().numpy(), v2.cpu().numpy()) < 0.02


# ---- circuit_kv._C mirror ---------------------------------------------------------------
def test_circuit_graph_influence_walker():
    dev = _cuda()
    torch.cuda.set_device(dev)
    n = 400
    A = torch.from_numpy(_row_stochastic(n, 21)).to(dev)
    g = _C.CircuitGraph(8192, 32, 0.85, 10000, 100)
    g.update_and_step_influence_walker(A, n - 1, 10000, 10, 4)
    v1 = g.get_influence_raw_visits()
    s1 = g.get_influence_scores()
    assert v1.shape == (n,) and s1.shape == (n,)
    st = torch.from_numpy(WO.states_array(WO.seed_states(42 + 3000, 10000))).to(dev)
    if os.path.exists(REF_SO):
        f = _ref_lib()
        s_r, v_r = _ref_walk(f, A, n - 1, 10000, 10, 4, 2.0, 10.0, 0.3, st)
        assert torch.equal(v1, v_r)
        torch.testing.assert_close(s1, s_r, rtol=2e-6, atol=0)
    g.update_and_step_influence_walker(A, n - 1, 10000, 10, 4)      # states carried over
    v2 = g.get_influence_raw_visits()
    assert not torch.equal(v1, v2) and v2.sum().item() == 10000 * 10
    if os.path.exists(REF_SO):
        _, v_r2 = _ref_walk(f, A, n - 1, 10000, 10, 4, 2.0, 10.0, 0.3, st)
        assert torch.equal(v2, v_r2)
    g.reset()
    bad = [(A.t(), n - 1), (A.half(), n - 1), (A[0], 0), (A[:, :10].contiguous(), 0), (A, n), (A.cpu(), 0)]
    for m, cur in bad:
        with pytest.raises(RuntimeError):
            g.update_and_step_influence_walker(m, cur)
    with pytest.raises(RuntimeError):
        g.update_and_step_influence_walker(A, n - 1, num_walkers=10001)
    small = _C.CircuitGraph(100, 32, 0.85, 100, 10)
    with pytest.raises(RuntimeError):
        small.update_and_step_influence_walker(A, n - 1)
    # after reset: no landmark walk has run, so no landmark positions
    assert g.get_landmark_positions().numel() == 0


# ---- the hook with use_neumann=False --------------------------------------------------
def test_hook_walker_path_end_to_end():
    dev = _cuda()
    c = case("bf16_n2048_default")
    q, k, v = inputs(c)
    kwargs = dict(c["kwargs"], use_neumann=False, combination_mode="max")
    cl = CircuitKVCluster(**kwargs)
    n, W, B = c["n"], c["window"], kwargs["max_capacity_prompt"]
    from submission_folder_b200.synth import repeat_kv
    K, V = repeat_kv(k, 4).to(dev), repeat_kv(v, 4).to(dev)
    ko, vo = cl.update_kv(K, q[None].to(dev), V, None, 4)
    torch.cuda.synchronize()
    idx = cl.last_keep_indices.cpu().numpy()
    assert ko.shape[2] == B and len(idx) == B - W
    # the same rows and a freshly seeded walker reproduce the hook's scores
    p = cl.params(n)
    _, _, _, rows, _ = ops.window_pool(p, q.to(dev), k.to(dev))
    st = torch.zeros(2 * 10000, dtype=torch.int64, device=dev)
    infl, _, h2o = ops.influence_walk(rows, n - 1, int(cl.num_walkers), int(cl.max_steps), int(cl.sink_size),
                                      rng_state=st, init_state=True)
    torch.cuda.synchronize()
    np.testing.assert_allclose(h2o.cpu().numpy(), O.full_attn_colsum(rows.cpu().numpy()), rtol=1e-4, atol=1e-6)
    comb = np.maximum(O.rank_normalize(h2o.cpu().numpy()), O.rank_normalize(infl.cpu().numpy()))
    mask = O.keep_mask(comb, B, n, int(cl.sink_size), W)
    mask[n - W:] = False
    assert np.array_equal(np.nonzero(mask)[0], idx)
    Kh = K[0].cpu()
    assert torch.equal(ko[0, :, :B - W].cpu(), Kh[:, torch.from_numpy(idx).long()])
    assert torch.equal(ko[0, :, B - W:].cpu(), Kh[:, n - W:])
    # a second layer continues the walker states, like the reference's CircuitGraph
    cl.update_kv(K, q[None].to(dev), V, None, 4)
    torch.cuda.synchronize()
    assert len(cl.last_keep_indices) == B - W
