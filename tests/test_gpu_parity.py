"""Parity of the sm_100a kernels (through the C ABI) with the reference's golden
outputs and with the CPU oracle, stage by stage and end to end.

Tolerances: the ranked score vectors agree
within 1e-3 relative; the index work is exact -- the kept positions are exactly
the reference's selection rule applied to the ranked vectors (stable ranks,
lowest-index-first ties of the k-th value, as torch's CUDA argsort / topk do,
pinned by ``test_selection_ties_follow_torch_cuda``); and the kept positions equal
the reference's except at exact ties of the k-th combined score (the reference's
CPU topk breaks those in an implementation-defined order).  The ``grid_*`` fixtures
use exact-arithmetic inputs, whose logits are the same bits on every device.
"""

import numpy as np
import pytest
import torch

import ckv_oracle as O
from _golden import (case, cases, check_kept, check_per_head, compare_keep, inputs, load, oracle_params,
                     ranked_vectors_of_reference)
from submission_folder_b200 import ops
from submission_folder_b200.cluster import CircuitKVCluster
from submission_folder_b200.synth import repeat_kv

pytestmark = pytest.mark.gpu

SCORE_RTOL = 1e-3


def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _cluster(c):
    return CircuitKVCluster(**c["kwargs"])


SHARED = [c["name"] for c in cases() if "perhead" not in c["name"]]


@pytest.mark.parametrize("name", ["bf16_n2048_default", "cfg1_fp32_n4096", "fp16_n2048_w32",
                                  "bf16_w128", "bf16_hi_max", "bf16_hi_cdf", "bf16_mass_sel",
                                  "bf16_no_entropy", "bf16_literal_scale"])
def test_window_pool_matches_oracle(name):
    dev = _cuda()
    c = case(name)
    q, k, _ = inputs(c)
    cl = _cluster(c)
    p = cl.params(c["n"])
    ent, mass, sets, rq, rh = ops.window_pool(p, q.to(dev), k.to(dev))
    torch.cuda.synchronize()
    op = oracle_params(c)
    attn = O.window_attention(q.float().numpy(), k.float().numpy(), c["window"], 4, c["dtype"])
    ch = O.choose_heads(attn, op)
    np.testing.assert_allclose(ent.cpu().numpy(), ch.entropy, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(mass.cpu().numpy(), ch.mass, rtol=1e-4, atol=1e-5)
    qset = int(sets[0].item()) & ((1 << 64) - 1)
    assert qset == sum(1 << int(h) for h in ch.qi_heads)
    oq, oh = O.pool_rows(attn, ch)
    gq = rq.cpu().numpy()
    # elementwise: nearly all within 1e-4 relative; a 16-bit logit that rounds
    # differently (MMA vs BLAS accumulation order) moves one entry by < 2%
    rel = np.abs(gq - oq) / np.maximum(np.abs(oq), 1e-30)
    assert np.mean(rel > 1e-4) < 2e-3, np.mean(rel > 1e-4)
    assert rel.max() < 0.05
    if oh is not None:
        gh = rh.cpu().numpy()
        relh = np.abs(gh - oh) / np.maximum(np.abs(oh), 1e-30)
        assert np.mean(relh > 1e-4) < 2e-3
        assert relh.max() < 0.05


@pytest.mark.parametrize("name", ["bf16_n2048_default", "bf16_temp07", "bf16_gamma09", "bf16_iters3",
                                  "bf16_sink8", "bf16_w128", "bf16_no_entropy", "bf16_max",
                                  "cfg1_fp32_n4096", "bf16_n8192_cfg2"])
def test_neumann_rows_matches_oracle(name):
    dev = _cuda()
    c = case(name)
    q, k, _ = inputs(c)
    op = oracle_params(c)
    attn = O.window_attention(q.float().numpy(), k.float().numpy(), c["window"], 4, c["dtype"])
    ch = O.choose_heads(attn, op)
    rq, rh = O.pool_rows(attn, ch)
    single = op.combination_mode not in ("dis", "union", "union_da")
    chains = [O.Chain(rq, "query")] if single else [O.Chain(rq, "query"),
                                                     O.Chain(rh if rh is not None else rq, "uniform")]
    sc, steps, _ = O.neumann_structured(chains, c["n"] - 1, op.sink_size, op.neumann_iterations,
                                        op.neumann_temperature, op.neumann_gamma)
    p = _cluster(c).params(c["n"])
    gq, gh, gsteps = ops.neumann_rows(p, torch.from_numpy(rq).to(dev),
                                      None if (single or rh is None) else torch.from_numpy(rh).to(dev),
                                      single_chain=single)
    torch.cuda.synchronize()
    assert int(gsteps.item()) == steps
    np.testing.assert_allclose(gq.cpu().numpy(), sc[0], rtol=SCORE_RTOL, atol=1e-7)
    if not single:
        np.testing.assert_allclose(gh.cpu().numpy(), sc[1], rtol=SCORE_RTOL, atol=1e-7)


@pytest.mark.parametrize("name", ["bf16_n2048_default", "cfg1_fp32_n4096", "fp16_n2048_w32",
                                  "bf16_ablate_qi", "bf16_ablate_hi", "bf16_boxcar5", "bf16_sink8",
                                  "bf16_w128", "bf16_n8192_cfg2", "bf16_union", "bf16_union_da",
                                  "bf16_max", "bf16_bridge", "bf16_weighted"])
def test_select_from_reference_scores(name):
    """Selection stage fed with the reference's own score vectors."""
    dev = _cuda()
    c = case(name)
    g = load(name)
    p = _cluster(c).params(c["n"])
    n, W, s = c["n"], c["window"], p.sink_size
    op = oracle_params(c)
    mode = op.combination_mode
    if mode in ("union", "union_da"):
        a, b = g["union_qi"], g["union_hi"]
        cvec = None
    elif mode in ("max", "weighted"):
        q, k, _ = inputs(c)
        at = O.window_attention(q.float().numpy(), k.float().numpy(), W, 4, c["dtype"])
        rq, _ = O.pool_rows(at, O.choose_heads(at, op))
        a, b = g["influence"], O.full_attn_colsum(rq)
        cvec = None
    else:
        a, b = g["qi"], g["hi"]
        cvec = None
        if op.use_bridge_importance:
            q, k, _ = inputs(c)
            at = O.window_attention(q.float().numpy(), k.float().numpy(), W, 4, c["dtype"])
            chh = O.choose_heads(at, op)
            rq, rh = O.pool_rows(at, chh)
            cvec = O.bridge_importance(rh if rh is not None else rq)
    idx, sc = ops.select_scores(p, torch.from_numpy(np.ascontiguousarray(a)).to(dev),
                                torch.from_numpy(np.ascontiguousarray(b)).to(dev),
                                None if cvec is None else torch.from_numpy(cvec).to(dev),
                                want_scores=True)
    torch.cuda.synchronize()
    ours = idx.cpu().numpy()
    ref = g["keep"]
    assert len(ours) == len(ref)
    assert np.all(np.diff(ours) > 0)
    kk = len(ref) - s
    if "combined" in g:
        nd, ok = compare_keep(ours, ref, g["combined"], s, n - W, kk)
        assert ok, f"{name}: {nd} positions differ beyond ties"
    else:
        nd = len(set(ours.tolist()) ^ set(ref.tolist()))
        assert nd <= 2, nd
    # and exactly the oracle's selection (same tie rules) from the same vectors
    if mode == "dis":
        qk = op.qi_kernel_size if op.qi_kernel_size != 0 else op.smoothing_kernel
        hk = op.hi_kernel_size if op.hi_kernel_size != 0 else op.smoothing_kernel
        if op.smooth_hi_only and qk > 1:
            qk = 0
        qs = O.smooth(a, qk, op.use_gaussian, op.gaussian_sigma * 0.5 if op.use_gaussian else 1.0) if qk > 1 else a
        hs = O.smooth(b, hk, op.use_gaussian, op.gaussian_sigma) if hk > 1 else b
        got = sc.cpu().numpy()
        np.testing.assert_allclose(got[0], qs, rtol=1e-5, atol=1e-8)
        np.testing.assert_allclose(got[1], hs, rtol=1e-5, atol=1e-8)


@pytest.mark.parametrize("name", SHARED)
def test_update_kv_matches_reference(name, parity_report):
    """The drop-in hook end to end on the GPU vs the reference's kept positions.

    The kept set must be exactly the reference's selection rule applied to the GPU's own
    ranked vectors, those vectors must agree with the reference's within 1e-3, and the kept
    set must equal the reference's except at exact ties of the k-th combined score.  The
    number of positions that differ (all at such ties) is recorded per case
    (``parity_report``)."""
    dev = _cuda()
    c = case(name)
    g = load(name)
    q, k, v = inputs(c, device="cpu")
    cl = _cluster(c)
    K, V = repeat_kv(k, 4).to(dev), repeat_kv(v, 4).to(dev)
    ko, vo = cl.update_kv(K, q[None].to(dev), V, None, 4)
    torch.cuda.synchronize()
    idx = cl.last_keep_indices.cpu().numpy()
    n, W = c["n"], c["window"]
    s = cl.sink_size
    ref = g["keep"]
    assert ko.shape == (1, 32, len(ref) + W, 128)
    assert np.all(np.diff(idx) > 0) and np.all(idx[:s] == np.arange(s))
    # K/V rows are exactly the rows at the kept positions, then the window
    kk_ = K[0, :, torch.from_numpy(idx).long().to(dev)]
    assert torch.equal(ko[0, :, :len(idx)], kk_)
    assert torch.equal(ko[0, :, len(idx):], K[0, :, n - W:])
    assert torch.equal(vo[0, :, :len(idx)], V[0, :, torch.from_numpy(idx).long().to(dev)])
    assert ops.read_status(dev) == 0
    # the same layer through the C ABI, with the ranked vectors
    p = cl.params(n)
    _, _, idx2, sc = ops.score_evict(p, q.to(dev), k.to(dev), v.to(dev), want_scores=True)
    torch.cuda.synchronize()
    assert np.array_equal(idx2.cpu().numpy(), idx)
    op = oracle_params(c)
    sc = sc.cpu().numpy()
    ra, rb = ranked_vectors_of_reference(c, g, op)
    if op.combination_mode in ("max", "weighted"):
        at = O.window_attention(q.float().numpy(), k.float().numpy(), W, 4, c["dtype"])
        rq, _ = O.pool_rows(at, O.choose_heads(at, op))
        rb = O.full_attn_colsum(rq)
    check_kept(name, idx, sc, ref, g.get("combined"), ra, rb, op, n, c.get("grid_step", 0) > 0,
               parity_report)


def test_scores_within_tolerance_end_to_end():
    """QI / HI scores of the full GPU path vs the reference's (1e-3 relative)."""
    dev = _cuda()
    for name in ("bf16_n2048_default", "cfg1_fp32_n4096", "bf16_n8192_cfg2"):
        c = case(name)
        g = load(name)
        q, k, v = inputs(c)
        cl = _cluster(c)
        p = cl.params(c["n"])
        _, _, _, sc = ops.score_evict(p, q.to(dev), k.to(dev), v.to(dev), want_scores=True)
        torch.cuda.synchronize()
        op = oracle_params(c)
        qs = O.smooth(g["qi"], op.qi_kernel_size, True, op.gaussian_sigma * 0.5)
        hs = O.smooth(g["hi"], op.hi_kernel_size, True, op.gaussian_sigma)
        got = sc.cpu().numpy()
        err_q = np.abs(got[0] - qs) / np.abs(qs).max()
        err_h = np.abs(got[1] - hs) / np.abs(hs).max()
        assert err_q.max() < SCORE_RTOL and err_h.max() < SCORE_RTOL, (name, err_q.max(), err_h.max())


def test_deterministic_and_batched():
    dev = _cuda()
    c = case("bf16_n2048_default")
    q, k, v = (x.to(dev) for x in inputs(c))
    p = _cluster(c).params(c["n"])
    a = ops.score_evict(p, q, k, v, want_scores=True)
    b = ops.score_evict(p, q, k, v, want_scores=True)
    torch.cuda.synchronize()
    for x, y in zip(a, b):
        assert torch.equal(x, y)


def test_batched_matches_single_calls():
    """ckv_score_evict_batched (concurrent lanes, per-layer params, ragged n, mixed
    dtypes, more layers than lanes) gives bit-identical results to one call per layer."""
    dev = _cuda()
    names = ["bf16_n2048_default", "fp16_n2048_w32", "cfg1_fp32_n4096", "bf16_w128", "bf16_hi_max",
             "bf16_n2048_default"]
    layers, params = [], []
    for nm in names:
        c = case(nm)
        layers.append(tuple(x.to(dev) for x in inputs(c)))
        params.append(_cluster(c).params(c["n"]))
    single = [ops.score_evict(p, *lay, want_scores=True) for p, lay in zip(params, layers)]
    batched = ops.score_evict_batched(params, layers, want_scores=True)
    torch.cuda.synchronize()
    for nm, a, b in zip(names, single, batched):
        for x, y in zip(a, b):
            assert torch.equal(x, y), nm
    # one shared params struct for identical layers
    c = case("bf16_n2048_default")
    p = _cluster(c).params(c["n"])
    shared = ops.score_evict_batched(p, [layers[0], layers[5]])
    torch.cuda.synchronize()
    for out in shared:
        for x, y in zip(out[:3], single[0][:3]):
            assert torch.equal(x, y)


@pytest.mark.parametrize("n,budget,w", [(5000, 700, 0.5), (2048, 256, 0.3), (33000, 2048, 0.7)])
def test_weighted_selection_exact(n, budget, w):
    """Weighted combination (PU:3237-3240) from given influence / H2O vectors: full stable
    ranks on the GPU (cluster radix sort), combined score, top-k with lowest-index ties --
    the same kept set as the oracle, exactly.  Values repeat to exercise rank ties."""
    dev = _cuda()
    rng = np.random.default_rng(n)
    infl = rng.integers(0, n // 4, n).astype(np.float32) / np.float32(n)   # many exact ties
    h2o = rng.random(n).astype(np.float32)
    h2o[rng.integers(0, n, n // 10)] = np.float32(0.25)
    cl = CircuitKVCluster(window_size=64, max_capacity_prompt=budget, combination_mode="weighted",
                          h2o_weight=w)
    p = cl.params(n)
    idx, sc = ops.select_scores(p, torch.from_numpy(infl).to(dev), torch.from_numpy(h2o).to(dev),
                                want_scores=True)
    torch.cuda.synchronize()
    ir, hr = O.rank_normalize(infl), O.rank_normalize(h2o)
    comb = (np.float32(w) * hr + np.float32(1 - w) * ir).astype(np.float32)
    mask = O.keep_mask(comb, budget, n, 4, 64)
    mask[n - 64:] = False
    ref = np.nonzero(mask)[0]
    got = idx.cpu().numpy()
    np.testing.assert_array_equal(got, ref)


def _per_head_run(c, kwargs, dev):
    q, k, v = inputs(c)
    cl = CircuitKVCluster(**kwargs)
    K, V = repeat_kv(k, 4).to(dev), repeat_kv(v, 4).to(dev)
    ko, vo = cl.update_kv(K, q[None].to(dev), V, None, 4)
    torch.cuda.synchronize()
    idx = cl.last_keep_indices.cpu().numpy()
    nk = idx.shape[1]
    hk = torch.from_numpy(idx).long().to(dev)
    for h in range(idx.shape[0]):
        assert np.all(np.diff(idx[h]) > 0)
        assert torch.equal(ko[0, h, :nk], K[0, h, hk[h]])
        assert torch.equal(vo[0, h, :nk], V[0, h, hk[h]])
        assert torch.equal(ko[0, h, nk:], K[0, h, c["n"] - c["window"]:])
    # the same call through ops, with the ranked vectors: deterministic kept sets
    _, _, idx2, (vec, ent) = ops.score_evict(cl.params(c["n"]), q.to(dev), k.to(dev), v.to(dev), want_scores=True)
    assert np.array_equal(idx2.cpu().numpy(), idx)
    return q, k, idx, vec.cpu().numpy(), ent.cpu().numpy()


@pytest.mark.parametrize("name", ["bf16_perhead", "bf16_perhead_hub", "grid_bf16_perhead", "bf16_perhead_n8192"])
def test_per_head_matches_reference(name, parity_report):
    """Per-head eviction (PU:2208-2382, 3296-3464) end to end vs the reference's kept sets
    (per-head differences recorded in ``parity_report``)."""
    dev = _cuda()
    c = case(name)
    g = load(name)
    _, _, idx, _, _ = _per_head_run(c, c["kwargs"], dev)
    ref = g["keep_per_head"]
    assert idx.shape == ref.shape
    d = [len(set(idx[h].tolist()) ^ set(ref[h].tolist())) for h in range(ref.shape[0])]
    parity_report["per_head_" + name] = {"n": c["n"], "kept_per_head": int(ref.shape[1]), "differ_per_head": d}
    assert max(d) == 0, d   # every head keeps exactly the reference's positions
    assert ops.read_status(dev) == 0


@pytest.mark.parametrize("extra", [dict(ablate_qi=True), dict(ablate_hi=True),
                                   dict(ablate_qi=True, ablate_hi=True), dict(entropy_adaptive=False),
                                   dict(smoothing_kernel=3), dict(true_hub_hi=True, entropy_adaptive=False)])
def test_per_head_variants_match_oracle(extra, parity_report):
    """Ablations and variants: decomposed parity against the oracle (``check_per_head``)."""
    dev = _cuda()
    c = case("bf16_perhead")
    kwargs = dict(c["kwargs"], **extra)
    q, k, idx, vec, ent = _per_head_run(c, kwargs, dev)
    op = oracle_params(dict(c, kwargs=kwargs))
    attn = O.window_attention(q.float().numpy(), k.float().numpy(), c["window"], 4, c["dtype"])
    check_per_head(idx, vec, ent, attn, op, c["n"], parity_report, "per_head_variant_" + "_".join(sorted(extra)))


def test_per_head_fp32_ragged(parity_report):
    """fp32 inputs, W = 32, n not a multiple of the column tile."""
    dev = _cuda()
    torch.manual_seed(3)
    from submission_folder_b200.synth import make_layer
    n, W = 3001, 32
    q, k, v = make_layer(n, seed=5, window=W, dtype="fp32")
    kwargs = dict(window_size=W, max_capacity_prompt=300, per_head_eviction=True, qi_kernel_size=3,
                  hi_kernel_size=5, use_gaussian=True)
    cl = CircuitKVCluster(**kwargs)
    K, V = repeat_kv(k, 4).to(dev), repeat_kv(v, 4).to(dev)
    ko, vo = cl.update_kv(K, q[None].to(dev), V, None, 4)
    torch.cuda.synchronize()
    idx = cl.last_keep_indices.cpu().numpy()
    _, _, _, (vec, ent) = ops.score_evict(cl.params(n), q.to(dev), k.to(dev), v.to(dev), want_scores=True)
    op = O.Params(**kwargs)
    attn = O.window_attention(q.numpy(), k.numpy(), W, 4, "fp32")
    check_per_head(idx, vec.cpu().numpy(), ent.cpu().numpy(), attn, op, n, parity_report, "per_head_fp32_ragged")
    assert ops.read_status(dev) == 0


@pytest.mark.parametrize("n,W,dtype", [(3001, 32, "bf16"), (5000, 128, "bf16"), (4222, 64, "fp16"),
                                       (1100, 128, "bf16"), (640, 64, "bf16"), (1153, 32, "fp16")])
def test_per_head_tensor_core_windows(n, W, dtype, parity_report):
    """The tcgen05 per-head pass for windows of 32, 64 and 128 rows (ragged n, the last key
    tile partly past n): decomposed parity against the oracle (``check_per_head``)."""
    dev = _cuda()
    from submission_folder_b200.synth import make_layer
    q, k, v = make_layer(n, seed=n, window=W, dtype=dtype)
    kwargs = dict(window_size=W, max_capacity_prompt=512, per_head_eviction=True, qi_kernel_size=3,
                  hi_kernel_size=5, use_gaussian=True)
    cl = CircuitKVCluster(**kwargs)
    K, V = repeat_kv(k, 4).to(dev), repeat_kv(v, 4).to(dev)
    cl.update_kv(K, q[None].to(dev), V, None, 4)
    torch.cuda.synchronize()
    idx = cl.last_keep_indices.cpu().numpy()
    _, _, _, (vec, ent) = ops.score_evict(cl.params(n), q.to(dev), k.to(dev), v.to(dev), want_scores=True)
    op = O.Params(**kwargs)
    attn = O.window_attention(q.float().numpy(), k.float().numpy(), W, 4, dtype)
    check_per_head(idx, vec.cpu().numpy(), ent.cpu().numpy(), attn, op, n, parity_report,
                   f"per_head_tc_{dtype}_w{W}_n{n}")
    assert ops.read_status(dev) == 0


@pytest.mark.parametrize("n,W", [(4460, 64), (11554, 64), (4466, 32)])
def test_moments_chunk_of_one_masked_tile(n, W, parity_report):
    """Lengths where a moments-pass CTA gets only the last, partly masked key tile:
    finite scores, and the kept set checked against the oracle (``check_kept``)."""
    from submission_folder_b200.cluster import cli_cluster_kwargs
    from submission_folder_b200.synth import make_layer
    dev = _cuda()
    B = n // 8
    q, k, v = make_layer(n, seed=n, window=W, planted=16, dtype="bf16", device="cpu")
    p = CircuitKVCluster(**cli_cluster_kwargs(W, B)).params(n)
    ent, mass, _, rq, rh = ops.window_pool(p, q.to(dev), k.to(dev))
    ko, vo, idx, sc = ops.score_evict(p, q.to(dev), k.to(dev), v.to(dev), want_scores=True)
    torch.cuda.synchronize()
    for t in (ent, mass, rq, rh, sc):
        assert torch.isfinite(t).all()
    r = O.update_kv(q.float().numpy(), k.float().numpy(), v.float().numpy(), 4,
                    O.Params(window_size=W, max_capacity_prompt=B), dtype="bf16")
    np.testing.assert_allclose(mass.cpu().numpy(), r.choice.mass, rtol=1e-4, atol=1e-5)
    check_kept(f"masked_tile_n{n}_w{W}", idx.cpu().numpy(), sc.cpu().numpy(), r.keep_idx, r.combined, r.qi,
               r.hi, O.Params(window_size=W, max_capacity_prompt=B), n, False, parity_report)


@pytest.mark.parametrize("H,Hkv,W,n", [(28, 4, 64, 3000), (32, 4, 64, 2600), (32, 2, 32, 2500)])
def test_other_head_groupings(H, Hkv, W, n, parity_report):
    """Query heads per KV head other than 4 (Qwen2-style 28 / 4, 8 and 16 per KV head): the
    kept set checked against the oracle (``check_kept``) and the gathered rows against the
    inputs."""
    from submission_folder_b200.cluster import cli_cluster_kwargs
    from submission_folder_b200.synth import make_layer
    dev = _cuda()
    B = n // 8
    q, k, v = make_layer(n, seed=n + H, heads=H, kv_heads=Hkv, window=W, planted=16, dtype="bf16")
    p = CircuitKVCluster(**cli_cluster_kwargs(W, B)).params(n)
    ko, vo, idx, sc = ops.score_evict(p, q.to(dev), k.to(dev), v.to(dev), want_scores=True)
    torch.cuda.synchronize()
    assert ops.read_status(dev) == 0 and torch.isfinite(sc).all()
    r = O.update_kv(q.float().numpy(), k.float().numpy(), v.float().numpy(), H // Hkv,
                    O.Params(window_size=W, max_capacity_prompt=B), dtype="bf16")
    check_kept(f"groups_{H}_{Hkv}_w{W}", idx.cpu().numpy(), sc.cpu().numpy(), r.keep_idx, r.combined, r.qi,
               r.hi, O.Params(window_size=W, max_capacity_prompt=B), n, False, parity_report)
    kk = torch.from_numpy(np.asarray(idx.cpu().numpy(), dtype=np.int64))
    rows = torch.cat([kk, torch.arange(n - W, n)])
    for h in (0, H // Hkv, H - 1):
        assert torch.equal(ko[h].cpu(), k[h // (H // Hkv), rows]) and torch.equal(vo[h].cpu(), v[h // (H // Hkv), rows])


def test_both_pooling_branches_are_exercised(parity_report):
    """The pooling pass skips the exact entropy / mass recomputation when the moments
    pass settles the head sets (header word need_exact = 0) and redoes it otherwise;
    the golden cases that reach the tensor-core pooling pass must cover both, so the
    parity tests above check both branches against the reference."""
    dev = _cuda()
    seen = {}
    for c in cases():
        if c["dtype"] != "bf16" or c["window"] != 64 or "perhead" in c["name"]:
            continue
        q, k, v = (x.to(dev) for x in inputs(c))
        p = _cluster(c).params(c["n"])
        ops.score_evict(p, q, k, v)
        torch.cuda.synchronize()
        ws = ops._workspaces[(dev.type, dev.index)]
        seen[c["name"]] = int(ws[56:60].cpu().view(torch.int32).item())   # Header.need_exact
    assert 0 in seen.values(), seen
    # the four query heads of each KV group identical: their entropies tie, so the 10-head
    # selection boundary falls inside a tied group and the exact branch must run
    c = case("bf16_n2048_default")
    q, k, v = inputs(c)
    q = q.reshape(8, 4, *q.shape[1:])[:, :1].expand(8, 4, *q.shape[1:]).reshape(q.shape).contiguous()
    p = _cluster(c).params(c["n"])
    ko, vo, idx, sc = ops.score_evict(p, q.to(dev), k.to(dev), v.to(dev), want_scores=True)
    torch.cuda.synchronize()
    ws = ops._workspaces[(dev.type, dev.index)]
    assert int(ws[56:60].cpu().view(torch.int32).item()) == 1
    r = O.update_kv(q.float().numpy(), k.float().numpy(), v.float().numpy(), 4, oracle_params(c),
                    dtype=c["dtype"])
    check_kept("tied_heads_exact_branch", idx.cpu().numpy(), sc.cpu().numpy(), r.keep_idx, r.combined, r.qi,
               r.hi, oracle_params(c), c["n"], False, parity_report)


def test_short_sequence_returns_inputs():
    dev = _cuda()
    c = case("bf16_n2048_default")
    q, k, v = inputs(c)
    cl = CircuitKVCluster(**dict(c["kwargs"], max_capacity_prompt=4096))
    K, V = repeat_kv(k, 4).to(dev), repeat_kv(v, 4).to(dev)
    ko, vo = cl.update_kv(K, q[None].to(dev), V, None, 4)
    assert ko is K and vo is V


def test_host_tensors_round_trip():
    """Host tensors in, host tensors out (the kernels run on the GPU in between)."""
    _cuda()
    c = case("bf16_n2048_default")
    g = load("bf16_n2048_default")
    q, k, v = inputs(c)
    cl = _cluster(c)
    ko, vo = cl.update_kv(repeat_kv(k, 4), q[None], repeat_kv(v, 4), None, 4)
    assert not ko.is_cuda
    idx = cl.last_keep_indices.cpu().numpy()
    assert len(idx) == len(g["keep"])
    # pinned host tensors: K is copied, V's kept rows are read in place by the gather; the
    # outputs equal those of device-resident inputs exactly
    dev = torch.device("cuda", 0)
    K, Q, V = repeat_kv(k, 4), q[None], repeat_kv(v, 4)
    kp, qp, vp = K.pin_memory(), Q.pin_memory(), V.pin_memory()
    assert ops.device_readable(vp[0]) and not ops.device_readable(V[0])
    cd = _cluster(c)
    kd, vd = cd.update_kv(K.to(dev), Q.to(dev), V.to(dev), None, 4)
    assert np.array_equal(cd.last_keep_indices.cpu().numpy(), idx)
    kh, vh = _cluster(c).update_kv(kp, qp, vp, None, 4)
    assert kh.is_pinned() and vh.is_pinned()
    assert torch.equal(kh, kd.cpu()) and torch.equal(vh, vd.cpu())
    assert torch.equal(ko, kd.cpu()) and torch.equal(vo, vd.cpu())


def test_copy_rows_strided_heads():
    """ckv_copy_rows: strided row blocks (the window rows of every head; every 4th head) in
    one DMA, host to device and back, pinned and pageable; layouts it cannot take decline."""
    dev = _cuda()
    x = torch.randn(32, 300, 128).to(torch.bfloat16)
    for src in (x, x.pin_memory()):
        d = torch.zeros(32, 300, 128, dtype=torch.bfloat16, device=dev)
        assert ops.copy_rows_async(d[:, 236:], src[:, 236:])
        torch.cuda.synchronize()
        assert torch.equal(d[:, 236:].cpu(), x[:, 236:]) and int(d[:, :236].abs().sum().item()) == 0
        e = torch.empty(8, 300, 128, dtype=torch.bfloat16, device=dev)
        assert ops.copy_rows_async(e, src[::4])
        back = torch.empty(8, 300, 128, dtype=torch.bfloat16).pin_memory()
        assert ops.copy_rows_async(back, e)
        torch.cuda.synchronize()
        assert torch.equal(back, x[::4])
    assert not ops.copy_rows_async(torch.empty(4, 8, device=dev), torch.randn(8, 4).t())


def _flip_case(n=4096, W=64, H=32, Hkv=8, D=128, seed=11):
    """Window queries whose speculated QI head set is wrong.

    The moments pass ranks heads by their unclamped entropy; the reference clamps
    probabilities at 1e-8 inside the entropy (PU:1452-1477), which can only raise it.
    Head 1 puts its mass on 20 keys and leaves every other key ~30 logits lower (below
    the clamp), so clamping raises its entropy by ~7.5e-4; head 12 has Gaussian logits
    whose scale is searched so that its unclamped entropy lies just above head 1's and
    its clamped entropy just below.  Nine heads are far more peaked, the rest far
    flatter, so heads 1 and 12 share the 10th place of the 10-head QI set: the pass-1
    choice takes head 1, the exact one head 12, and the pooling pass must re-run.
    """
    G = H // Hkv
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((H, n, D)).astype(np.float32)
    k = rng.standard_normal((Hkv, n, D)).astype(np.float32)
    v = rng.standard_normal((Hkv, n, D)).astype(np.float32)
    bf = lambda x: torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(torch.bfloat16).float().numpy()
    X, Y = 1, 12
    P = rng.choice(np.arange(100, n - W - 100), size=20, replace=False)
    k[X // G, :, 0] = 0.0
    k[X // G, P, 0] = 10.0
    q[X, n - W:, :] = 0.0
    q[X, n - W:, 0] = 34.0
    q[20:29, n - W:] *= 8.0
    q, k, v = bf(q), bf(k), bf(v)

    def entropy(qh, kg):
        att = O.window_attention(qh[None], kg[None], W, 1, "bf16")[0].astype(np.float64)
        with np.errstate(divide="ignore", invalid="ignore"):
            un = float(np.where(att > 0, -att * np.log(att), 0.0).sum(-1).mean())
        return un, float(O.head_entropy(att[None].astype(np.float32))[0])

    unX, clX = entropy(q[X], k[X // G])
    base = q[Y, n - W:].copy()

    def scaled(s):
        qq = q[Y].copy()
        qq[n - W:] = bf(base * s)
        return qq

    lo, hi = 1.0, 8.0   # the entropy falls as the scale grows: bisect to the window's middle
    for _ in range(16):
        mid = 0.5 * (lo + hi)
        if entropy(scaled(mid), k[Y // G])[0] > 0.5 * (unX + clX):
            lo = mid
        else:
            hi = mid
    # the logits' 16-bit rounding makes the entropy a staircase of ~1e-3 steps there:
    # scan nearby scales for one that lands inside the window with margins
    for d in sorted(np.arange(-0.02, 0.02, 5e-5), key=abs):
        qq = scaled(lo + d)
        un, cl = entropy(qq, k[Y // G])
        if unX + 1.5e-4 < un and cl < clX - 1.5e-4:
            q[Y] = qq
            return q, k, v
    pytest.skip("no scale of head 12 lands between head 1's entropies")


def test_speculated_head_set_wrong_reruns_pooling(parity_report):
    """The re-run path: pass 1's head set differs from the exact one (header words
    need_exact = 1 and fixup = 1 after the call), and the pooling pass re-runs with the
    exact sets, so the kept positions follow the reference's (clamped) head choice."""
    from submission_folder_b200.cluster import cli_cluster_kwargs
    dev = _cuda()
    n, W, B = 4096, 64, 512
    q, k, v = _flip_case(n=n, W=W)
    kw = cli_cluster_kwargs(W, B)
    p = CircuitKVCluster(**kw).params(n)
    to = lambda x: torch.from_numpy(x).to(torch.bfloat16).to(dev)
    ko, vo, idx, sc = ops.score_evict(p, to(q), to(k), to(v), want_scores=True)
    torch.cuda.synchronize()
    ws = ops._workspaces[(dev.type, dev.index)]
    assert int(ws[56:60].cpu().view(torch.int32).item()) == 1   # Header.need_exact
    assert int(ws[12:16].cpu().view(torch.int32).item()) == 1   # Header.fixup
    r = O.update_kv(q, k, v, 4, O.Params(**{a: b for a, b in kw.items() if a in O.Params.__dataclass_fields__}),
                    dtype="bf16")
    assert 12 in r.choice.qi_heads and 1 not in r.choice.qi_heads
    check_kept("speculated_set_wrong", idx.cpu().numpy(), sc.cpu().numpy(), r.keep_idx, r.combined, r.qi,
               r.hi, O.Params(**{a: b for a, b in kw.items() if a in O.Params.__dataclass_fields__}), n, False,
               parity_report)


@pytest.mark.parametrize("n,budget,mode", [(8192, 1024, "dis"), (32768, 2048, "dis"), (32768, 2048, "weighted"),
                                           (4096, 512, "max")])
def test_selection_ties_follow_torch_cuda(n, budget, mode):
    """The reference ranks with ``argsort(argsort(s))`` and selects with ``topk``
    (PU:1878, PU:2640).  Those torch ops, run on the B200 on vectors full of exact
    ties, pick exactly the kept set of the GPU selection: the tie order the product
    follows is the one the reference has on CUDA tensors, observed rather than assumed."""
    dev = _cuda()
    rng = np.random.default_rng(n + len(mode))
    a = rng.integers(0, n // 16, n).astype(np.float32) / np.float32(n)
    b = rng.integers(0, n // 16, n).astype(np.float32) / np.float32(n)
    kw = dict(window_size=64, max_capacity_prompt=budget, combination_mode=mode, qi_kernel_size=1,
              hi_kernel_size=1, smoothing_kernel=0, h2o_weight=0.5)
    p = CircuitKVCluster(**kw).params(n)
    ta, tb = torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev)
    idx, _ = ops.select_scores(p, ta, tb)

    def rank(x):
        return torch.argsort(torch.argsort(x)).float() / (len(x) - 1)

    if mode == "dis":
        comb = torch.maximum(rank(ta), rank(tb))
    elif mode == "max":
        comb = torch.maximum(rank(tb), rank(ta))          # H2O rank, influence rank
    else:
        comb = 0.5 * rank(tb) + (1 - 0.5) * rank(ta)
    W, s = 64, 4
    mask = torch.zeros(n, dtype=torch.bool, device=dev)
    mask[:s] = True
    mask[max(s, n - W):] = True
    remaining = budget - int(mask.sum().item())
    masked = comb.clone()
    masked[mask] = float("-inf")
    _, top = torch.topk(masked, remaining)
    mask[top] = True
    mask[n - W:] = False
    ref = torch.nonzero(mask).flatten().to(torch.int32)
    torch.cuda.synchronize()
    # the vectors really tie at the boundary: many positions share the k-th combined value
    kth = torch.sort(masked, descending=True).values[remaining - 1]
    assert int((masked == kth).sum().item()) > 1
    assert torch.equal(idx, ref)


@pytest.mark.parametrize("W,B", [(32, 512), (128, 1024)])
def test_exact_branch_other_windows(W, B, parity_report):
    """Windows of 32 and 128 rows when the moments pass cannot settle the head sets
    (header word need_exact = 1): the clamped entropy and transient mass are recomputed on
    the tensor cores (the moments kernel in its exact form) beside the keys-on-lanes
    pooling.  Query heads identical within each KV group tie their entropies, so the
    10-head selection boundary falls inside a tied group; the kept set is checked against
    the oracle."""
    from submission_folder_b200.cluster import cli_cluster_kwargs
    from submission_folder_b200.synth import make_layer
    dev = _cuda()
    n = 4096
    q, k, v = make_layer(n, seed=W + 7, window=W, planted=32, dtype="bf16", device="cpu")
    q = q.reshape(8, 4, *q.shape[1:])[:, :1].expand(8, 4, *q.shape[1:]).reshape(q.shape).contiguous()
    p = CircuitKVCluster(**cli_cluster_kwargs(W, B)).params(n)
    ko, vo, idx, sc = ops.score_evict(p, q.to(dev), k.to(dev), v.to(dev), want_scores=True)
    torch.cuda.synchronize()
    ws = ops._workspaces[(dev.type, dev.index)]
    assert int(ws[56:60].cpu().view(torch.int32).item()) == 1   # Header.need_exact
    assert ops.read_status(dev) == 0
    op = O.Params(window_size=W, max_capacity_prompt=B)
    r = O.update_kv(q.float().numpy(), k.float().numpy(), v.float().numpy(), 4, op, dtype="bf16")
    check_kept(f"exact_w{W}", idx.cpu().numpy(), sc.cpu().numpy(), r.keep_idx, r.combined, r.qi, r.hi,
               op, n, False, parity_report)


@pytest.mark.parametrize("W", [32, 128])
def test_speculated_head_set_wrong_other_windows(W, parity_report):
    """The re-run path for windows of 32 and 128 rows: the moments pass's QI set differs
    from the exact one (need_exact = 1 and fixup = 1 after the call) and the keys-on-lanes
    pooling re-runs with the exact sets."""
    from submission_folder_b200.cluster import cli_cluster_kwargs
    dev = _cuda()
    n, B = 4096, 512
    q, k, v = _flip_case(n=n, W=W)
    kw = cli_cluster_kwargs(W, B)
    p = CircuitKVCluster(**kw).params(n)
    to = lambda x: torch.from_numpy(x).to(torch.bfloat16).to(dev)
    ko, vo, idx, sc = ops.score_evict(p, to(q), to(k), to(v), want_scores=True)
    torch.cuda.synchronize()
    ws = ops._workspaces[(dev.type, dev.index)]
    assert int(ws[56:60].cpu().view(torch.int32).item()) == 1   # Header.need_exact
    assert int(ws[12:16].cpu().view(torch.int32).item()) == 1   # Header.fixup
    assert ops.read_status(dev) == 0
    op = O.Params(**{a: b for a, b in kw.items() if a in O.Params.__dataclass_fields__})
    r = O.update_kv(q, k, v, 4, op, dtype="bf16")
    assert 12 in r.choice.qi_heads and 1 not in r.choice.qi_heads
    check_kept(f"speculated_set_wrong_w{W}", idx.cpu().numpy(), sc.cpu().numpy(), r.keep_idx, r.combined, r.qi,
               r.hi, op, n, False, parity_report)


@pytest.mark.parametrize("n,W,B,dtype", [(8192, 32, 819, "bf16"), (6000, 128, 1024, "bf16"), (4096, 32, 512, "fp16"),
                                         (20000, 128, 2048, "fp16")])
def test_keys_on_lanes_pooling_other_windows(n, W, B, dtype, parity_report):
    """Windows of 32 and 128 rows: when the moments pass settles the head sets (header
    word need_exact = 0) the pooling pass runs the tcgen05 keys-on-lanes form (W = 128 in
    two 64-row halves); the kept set is checked against the oracle (``check_kept``)."""
    from submission_folder_b200.cluster import cli_cluster_kwargs
    from submission_folder_b200.synth import make_layer
    dev = _cuda()
    q, k, v = make_layer(n, seed=n + W, window=W, planted=32, dtype=dtype, device="cpu")
    p = CircuitKVCluster(**cli_cluster_kwargs(W, B)).params(n)
    ko, vo, idx, sc = ops.score_evict(p, q.to(dev), k.to(dev), v.to(dev), want_scores=True)
    torch.cuda.synchronize()
    ws = ops._workspaces[(dev.type, dev.index)]
    assert int(ws[56:60].cpu().view(torch.int32).item()) == 0   # Header.need_exact: the lanes form ran
    assert ops.read_status(dev) == 0
    op = O.Params(window_size=W, max_capacity_prompt=B)
    r = O.update_kv(q.float().numpy(), k.float().numpy(), v.float().numpy(), 4, op, dtype=dtype)
    check_kept(f"lanes_w{W}_n{n}_{dtype}", idx.cpu().numpy(), sc.cpu().numpy(), r.keep_idx, r.combined, r.qi, r.hi,
               op, n, False, parity_report)
