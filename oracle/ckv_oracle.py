"""CPU oracle for the CircuitKV prefill scoring + eviction path.

THIS IS TEST INFRASTRUCTURE.  Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline / reference arm may import it, and only as the
checker or as the timed CPU baseline -- never as the product path.  The product
path (``submission_folder_b200``) runs the sm_100a CUDA kernels and fails
loudly when they are missing.

What it restates (all citations are to
``KVCache-Factory/pyramidkv/pyramidkv_utils.py`` of the reference, "PU"):

* window logits, causal mask and fp32 softmax ............ PU:2874-2892
* per-head entropy / transient mass ...................... PU:1452-1508
* entropy-aware head selection and QI / HI pooling ....... PU:2905-2999
* prefix transition rows and ``full_attn`` assembly ...... PU:3003-3034
* dual Neumann absorption (QI, HI) with early stop ....... PU:2060-2206
* single-chain Neumann influence + H2O MAX / weighted .... PU:1939-2058, 3205-3242
* Gaussian / boxcar smoothing ............................ PU:1884-1937, 3131-3160
* bridge importance colsum(A @ A) ........................ PU:1510-1546, 3164-3173
* rank normalisation and MAX ............................. PU:1865-1882, 3177-3196
* static keep mask (sinks + local window + top-k) ........ PU:2591-2644
* union / union_da keep mask ............................. PU:2489-2589, 3044-3113
* per-head Markov importance + per-head eviction ......... PU:2208-2382, 3296-3464
* shared gather / compaction ............................. PU:3496-3517

Two restatements of the absorption solve are given:

* ``neumann_dense`` builds the n x n matrices exactly as the reference does and
  iterates ``v <- gamma * Q^T v``.  It is O(n^2) and only for small n.
* ``neumann_structured`` uses the rank structure of the prefix rows:
  ``P[i, j] = g[j] / G[i-1]`` for ``j < i < n - W`` (``g`` the clamped
  column sums of the pooled window rows, ``G`` their cumulative sum; the
  reference's ``+1e-8`` terms cancel between the entry and its row sum), so
  ``Q^T v`` on the prefix is ``g * SuffixSum(c * v) + (window rows)^T v_w``
  with ``c[i] = 1 / G[i-1]``.  Each of the reference's iterations becomes one
  reverse cumulative sum: O(W * n) per iteration instead of O(n^2).

Tie semantics follow the reference as it runs on CUDA tensors (its production
device): ``argsort`` of a 1-D CUDA tensor is a stable radix sort, so equal
scores rank by index; ``topk`` on CUDA takes, among values equal to the k-th,
the lowest indices first.  The CPU reference's own tie order is
implementation-defined; the parity tests treat those ties explicitly.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional

import numpy as np

F32 = np.float32
EPS_ENTROPY = F32(1e-8)          # PU:1452 eps clamp in _compute_head_entropy
PREFIX_CLAMP = F32(1e-6)         # PU:3016 h2o_prefix.clamp(min=1e-6)
ROWSUM_CLAMP = F32(1e-8)         # PU:2132 row_sums.clamp(min=1e-8)
EARLY_STOP = 1e-8                # PU:2183 early-stop threshold
SINK_FRACTION = F32(0.01)        # PU:2191 sinks get 1% of the total


# --------------------------------------------------------------------------
# dtype helpers
# --------------------------------------------------------------------------

def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), returned as float32."""
    x = np.ascontiguousarray(x, dtype=F32)
    b = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    rounded = ((b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = rounded.view(F32).copy()
    out[nan] = np.nan
    return out


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return round_bf16(x)
    if dtype == "fp16":
        return x.astype(np.float16).astype(F32)
    return x.astype(F32)


# --------------------------------------------------------------------------
# parameters (the kwargs of CircuitKVCluster.__init__, PU:1244-1331, with the
# values KVCache-Factory's run_longbench.py CLI passes by default)
# --------------------------------------------------------------------------

@dataclass
class Params:
    window_size: int = 64
    max_capacity_prompt: int = 2048
    sink_size: int = 4
    neumann_iterations: int = 10
    neumann_temperature: float = 1.0
    neumann_gamma: float = 1.0
    qi_gamma: Optional[float] = None
    hi_gamma: Optional[float] = None
    combination_mode: str = "dis"
    h2o_weight: float = 0.5
    qi_ratio: float = 0.5
    ablate_qi: bool = False
    ablate_hi: bool = False
    per_head_eviction: bool = False
    true_hub_hi: bool = False
    entropy_adaptive: bool = True
    smoothing_kernel: int = 0
    smooth_hi_only: bool = False
    use_gaussian: bool = True
    qi_kernel_size: int = 3
    hi_kernel_size: int = 5
    gaussian_sigma: float = 1.0
    entropy_aware: bool = True
    top_k_heads: int = 10
    head_selection_mode: str = "entropy"
    hi_pooling_mode: str = "mean"
    hi_mass_threshold: float = 0.5
    hi_top_k_heads: int = 0
    hi_mass_cdf: float = 0.0
    use_bridge_importance: bool = False
    bi_kernel_size: int = 5

    def resolved_qi_gamma(self) -> float:
        return self.neumann_gamma if self.qi_gamma is None else self.qi_gamma

    def resolved_hi_gamma(self) -> float:
        return self.neumann_gamma if self.hi_gamma is None else self.hi_gamma


# --------------------------------------------------------------------------
# a2: window logits, causal mask, fp32 softmax  (PU:2874-2892)
# --------------------------------------------------------------------------

def window_logits(q: np.ndarray, k: np.ndarray, window: int, groups: int, dtype: str) -> np.ndarray:
    """Window-query logits ``[H, W, n]`` in the input dtype's rounding, mask applied as -inf.

    ``q``: ``[H, n, D]`` (only the last ``window`` rows are read), ``k``: ``[Hkv, n, D]``
    distinct KV heads; q-head ``h`` reads KV head ``h // groups`` (the reference's
    ``repeat_kv`` layout has identical heads ``g*groups .. g*groups+groups-1``).
    The reference computes ``bf16(bf16(Q_w K^T) / sqrt(D))`` for 16-bit inputs
    (PU:2874-2877); the fp32 product is rounded to the dtype, divided in fp32 and
    rounded again.
    """
    H, n, D = q.shape
    qw = q[:, n - window:, :].astype(F32)
    out = np.empty((H, window, n), dtype=F32)
    scale = F32(math.sqrt(D))
    for h in range(H):
        kk = k[h // groups].astype(F32)
        acc = qw[h] @ kk.T
        acc = round_to(acc, dtype)
        out[h] = round_to(acc / scale, dtype)
    # causal mask on the last W columns: window row r may see key n-W+c only if c <= r
    r = np.arange(window)[:, None]
    c = np.arange(window)[None, :]
    masked = c > r
    tail = out[:, :, n - window:]
    tail[:, masked] = -np.inf
    return out


def softmax_f32(logits: np.ndarray) -> np.ndarray:
    m = logits.max(axis=-1, keepdims=True)
    e = np.exp(logits - m, dtype=F32)
    return (e / e.sum(axis=-1, keepdims=True, dtype=F32)).astype(F32)


def window_attention(q, k, window, groups, dtype) -> np.ndarray:
    """``attn_weights`` of PU:2892: ``[H, W, n]`` fp32 probabilities."""
    return softmax_f32(window_logits(q, k, window, groups, dtype))


# --------------------------------------------------------------------------
# a3-a6: head statistics, selection and pooling  (PU:1452-1508, 2905-2999)
# --------------------------------------------------------------------------

def head_entropy(attn: np.ndarray) -> np.ndarray:
    """PU:1452-1477: mean over window rows of -sum(p log p), p clamped at 1e-8."""
    c = np.maximum(attn, EPS_ENTROPY)
    ent_rows = -(c * np.log(c)).sum(axis=-1, dtype=np.float64)
    return ent_rows.mean(axis=-1).astype(F32)


def head_transient_mass(attn: np.ndarray, sink: int) -> np.ndarray:
    """PU:1479-1508: mean over window rows of the attention mass on keys >= sink."""
    return attn[..., sink:].sum(axis=-1, dtype=np.float64).mean(axis=-1).astype(F32)


def smallest_k(values: np.ndarray, k: int) -> np.ndarray:
    order = np.lexsort((np.arange(len(values)), values))
    return np.sort(order[:k])


def largest_k(values: np.ndarray, k: int) -> np.ndarray:
    order = np.lexsort((np.arange(len(values)), -values.astype(np.float64)))
    return np.sort(order[:k])


@dataclass
class HeadChoice:
    qi_heads: np.ndarray          # heads max-pooled into the QI rows
    hi_heads: Optional[np.ndarray]  # heads pooled into the HI rows (None: HI uses the QI matrix)
    hi_mode: str                  # "mean" or "max"
    entropy: np.ndarray
    mass: np.ndarray


def choose_heads(attn: np.ndarray, p: Params) -> HeadChoice:
    """Head sets of PU:2905-2999 (entropy-aware) or all heads (PU:2996-2999)."""
    return choose_heads_from(head_entropy(attn), head_transient_mass(attn, p.sink_size), p)


def choose_heads_from(ent: np.ndarray, mass: np.ndarray, p: Params) -> HeadChoice:
    """The same head sets from per-head entropy / transient mass ``[H]``."""
    H = len(ent)
    ent = np.asarray(ent, dtype=F32)
    mass = np.asarray(mass, dtype=F32)
    if not p.entropy_aware:
        return HeadChoice(np.arange(H), None, "max", ent, mass)
    k = min(p.top_k_heads, H)
    if p.head_selection_mode == "mass":
        qi = largest_k(mass, k)
    else:
        qi = smallest_k(ent, k)
    if p.hi_pooling_mode != "mean":
        return HeadChoice(qi, np.arange(H), "max", ent, mass)
    if p.hi_mass_cdf > 0:
        total = mass.astype(np.float64).sum()
        if total > 0:
            order = np.lexsort((np.arange(H), -mass.astype(np.float64)))
            cdf = np.cumsum(mass[order].astype(np.float64)) / total
            need = min(int((cdf < p.hi_mass_cdf).sum()) + 1, H)
            return HeadChoice(qi, order[:need], "mean", ent, mass)
        return HeadChoice(qi, np.arange(H), "mean", ent, mass)
    if p.hi_top_k_heads > 0:
        return HeadChoice(qi, largest_k(mass, min(p.hi_top_k_heads, H)), "mean", ent, mass)
    if p.hi_mass_threshold > 0:
        alive = np.nonzero(mass >= F32(p.hi_mass_threshold))[0]
        if len(alive) == 0:
            alive = np.arange(H)
        return HeadChoice(qi, alive, "mean", ent, mass)
    return HeadChoice(qi, np.arange(H), "mean", ent, mass)


def pool_rows(attn: np.ndarray, choice: HeadChoice):
    """Pooled window rows ``[W, n]``: QI = max over its heads; HI = mean/max over its heads."""
    qi_rows = attn[choice.qi_heads].max(axis=0)
    if choice.hi_heads is None:
        return qi_rows, None
    sel = attn[choice.hi_heads]
    if choice.hi_mode == "mean":
        acc = np.zeros(sel.shape[1:], dtype=F32)
        for h in range(sel.shape[0]):
            acc += sel[h]
        hi_rows = (acc / F32(sel.shape[0])).astype(F32)
    else:
        hi_rows = sel.max(axis=0)
    return qi_rows, hi_rows


# --------------------------------------------------------------------------
# a7-a8: absorption solve
# --------------------------------------------------------------------------

def build_full_attn(rows: np.ndarray) -> np.ndarray:
    """Dense ``full_attn`` of PU:3003-3027 for pooled window rows ``[W, n]`` (small n only)."""
    W, n = rows.shape
    A = np.zeros((n, n), dtype=F32)
    A[n - W:, :] = rows
    n_p = n - W
    if n_p > 1:
        h = np.maximum(rows.sum(axis=0, dtype=F32)[:n_p], PREFIX_CLAMP)
        C = np.cumsum(h, dtype=F32)
        denom = np.zeros(n_p, dtype=F32)
        denom[1:] = C[:-1]
        denom[0] = 1.0
        trans = h[None, :] / (denom[:, None] + F32(1e-8))
        A[:n_p, :n_p] = np.tril(trans, k=-1)
    return A


def _finish_scores(result: np.ndarray, n: int, sink: int) -> np.ndarray:
    """PU:2189-2204: scatter transient results, sinks = 1% of the total, divide by max."""
    s = np.zeros(n, dtype=F32)
    s[sink:] = result
    s[:sink] = F32(result.sum(dtype=F32)) * SINK_FRACTION
    mx = s.max()
    if mx > 0:
        s = (s / mx).astype(F32)
    return s


def neumann_dense(A_list, query_idx: int, sink: int, iters: int, temperature: float, gamma: float,
                  starts=("query", "uniform")):
    """Dense restatement of ``_compute_dual_importance_scores`` (PU:2060-2206) and of
    ``_compute_influence_neumann`` (PU:1939-2058, one chain).

    ``A_list`` holds one matrix per chain; ``starts`` gives each chain's start vector
    ("query": one-hot at the query, "uniform": 1/n_transient).  All chains stop
    together once every chain's new term has max < 1e-8 (the term is included).
    """
    n = A_list[0].shape[0]
    if n <= sink or query_idx - sink < 0:
        u = np.full(n, F32(1.0 / n), dtype=F32)
        return [u.copy() for _ in A_list], 0
    Qs = []
    for A in A_list:
        a = A ** F32(1.0 / temperature) if (temperature != 1.0 and temperature > 0) else A
        rs = np.maximum(a.sum(axis=1, keepdims=True, dtype=F32), ROWSUM_CLAMP)
        P = (a / rs).astype(F32)
        Qs.append(np.ascontiguousarray(P[sink:, sink:]))
    nt = n - sink
    vs, res = [], []
    for st in starts:
        v = np.zeros(nt, dtype=F32)
        if st == "query":
            v[query_idx - sink] = 1.0
        else:
            v[:] = F32(1.0) / F32(nt)
        vs.append(v)
        res.append(v.copy())
    steps = 0
    for _ in range(iters):
        vs = [(F32(gamma) * (Q.T @ v)).astype(F32) for Q, v in zip(Qs, vs)]
        res = [r + v for r, v in zip(res, vs)]
        steps += 1
        if all(np.abs(v).max() < EARLY_STOP for v in vs):
            break
    return [_finish_scores(r, n, sink) for r in res], steps


@dataclass
class Chain:
    """One absorbing chain in structured form (pooled window rows + start vector)."""
    rows: np.ndarray          # [W, n] pooled window rows (un-tempered)
    start: str                # "query" or "uniform"


def _chain_parts(rows: np.ndarray, sink: int, temperature: float):
    W, n = rows.shape
    n_p = n - W
    t = temperature != 1.0 and temperature > 0
    colsum = rows.sum(axis=0, dtype=F32)
    rw = rows ** F32(1.0 / temperature) if t else rows
    rs = np.maximum(rw.sum(axis=1, dtype=F32), ROWSUM_CLAMP)
    Pw = (rw / rs[:, None]).astype(F32)               # window rows of P, [W, n]
    if n_p > 1:
        hpre = np.maximum(colsum[:n_p], PREFIX_CLAMP)
        g = hpre ** F32(1.0 / temperature) if t else hpre
        G = np.cumsum(g, dtype=F32)
        c = np.zeros(n_p, dtype=F32)
        c[1:] = F32(1.0) / G[:-1]                      # P[i, j] = g[j] * c[i], j < i < n_p
    else:
        g = np.zeros(max(n_p, 0), dtype=F32)
        c = np.zeros(max(n_p, 0), dtype=F32)
    return Pw, g, c, n_p


def neumann_structured(chains, query_idx: int, sink: int, iters: int, temperature: float,
                       gamma: float):
    """Structured restatement of the same iteration as ``neumann_dense`` in O(W n) per step.

    For transient prefix positions ``s <= j < n_p``:
        (Q^T v)[j] = g[j] * sum_{i > j, i < n_p} c[i] v[i] + sum_r Pw[r, j] v[n_p + r]
    and for window positions ``n_p + c``:
        (Q^T v)[n_p + c] = sum_r Pw[r, n_p + c] v[n_p + r]
    since prefix rows have no entries in window columns.
    Returns (scores per chain, number of iterations taken, raw results per chain).
    """
    W, n = chains[0].rows.shape
    n_p = n - W
    if n <= sink or query_idx - sink < 0 or n_p < sink:
        dense = [build_full_attn(ch.rows) for ch in chains]
        sc, steps = neumann_dense(dense, query_idx, sink, iters, temperature, gamma,
                                  starts=tuple(ch.start for ch in chains))
        return sc, steps, None
    parts = [_chain_parts(ch.rows, sink, temperature) for ch in chains]
    nt = n - sink
    gam = F32(gamma)
    xs, ys, res_x, res_y = [], [], [], []
    for ch in chains:
        x = np.zeros(n_p - sink, dtype=F32)
        y = np.zeros(W, dtype=F32)
        if ch.start == "query":
            y[query_idx - n_p] = 1.0
        else:
            x[:] = F32(1.0) / F32(nt)
            y[:] = F32(1.0) / F32(nt)
        xs.append(x)
        ys.append(y)
        res_x.append(x.copy())
        res_y.append(y.copy())
    steps = 0
    for _ in range(iters):
        nxs, nys = [], []
        for (Pw, g, c, _), x, y in zip(parts, xs, ys):
            cx = c[sink:] * x
            suffix = np.zeros_like(cx)
            if len(cx) > 1:
                suffix[:-1] = np.cumsum(cx[::-1], dtype=F32)[::-1][1:]
            bw = Pw[:, sink:n_p].T @ y
            nx = (gam * (g[sink:] * suffix + bw)).astype(F32)
            ny = (gam * (Pw[:, n_p:].T @ y)).astype(F32)
            nxs.append(nx)
            nys.append(ny)
        xs, ys = nxs, nys
        res_x = [r + v for r, v in zip(res_x, xs)]
        res_y = [r + v for r, v in zip(res_y, ys)]
        steps += 1
        if all(max(np.abs(x).max(initial=0.0), np.abs(y).max(initial=0.0)) < EARLY_STOP
               for x, y in zip(xs, ys)):
            break
    raw = [np.concatenate([rx, ry]).astype(F32) for rx, ry in zip(res_x, res_y)]
    return [_finish_scores(r, n, sink) for r in raw], steps, raw


# --------------------------------------------------------------------------
# H2O column sums and bridge importance on the un-normalised full_attn
# --------------------------------------------------------------------------

def full_attn_colsum(rows: np.ndarray) -> np.ndarray:
    """``full_attn.sum(dim=0)`` (PU:3216) in O(W n): prefix part h[j] * sum_{i>j} 1/(C[i-1]+1e-8)."""
    W, n = rows.shape
    n_p = n - W
    colw = rows.sum(axis=0, dtype=F32)
    out = colw.copy()
    if n_p > 1:
        h = np.maximum(colw[:n_p], PREFIX_CLAMP)
        C = np.cumsum(h, dtype=F32)
        inv = np.zeros(n_p, dtype=F32)
        inv[1:] = F32(1.0) / (C[:-1] + F32(1e-8))
        suf = np.zeros(n_p, dtype=F32)
        suf[:-1] = np.cumsum(inv[::-1], dtype=F32)[::-1][1:]
        out[:n_p] = out[:n_p] + h * suf
    return out


def bridge_importance(rows: np.ndarray) -> np.ndarray:
    """``(A @ A).sum(dim=0)`` (PU:1510-1546) = A^T (A^T 1) in O(W n), A = un-normalised full_attn."""
    W, n = rows.shape
    n_p = n - W
    u = full_attn_colsum(rows)                       # A^T 1
    out = (rows.T @ u[n_p:]).astype(F32)             # window rows' contribution
    if n_p > 1:
        h = np.maximum(rows.sum(axis=0, dtype=F32)[:n_p], PREFIX_CLAMP)
        C = np.cumsum(h, dtype=F32)
        inv = np.zeros(n_p, dtype=F32)
        inv[1:] = F32(1.0) / (C[:-1] + F32(1e-8))
        w = u[:n_p] * inv
        suf = np.zeros(n_p, dtype=F32)
        suf[:-1] = np.cumsum(w[::-1], dtype=F32)[::-1][1:]
        out[:n_p] = out[:n_p] + h * suf
    return out


# --------------------------------------------------------------------------
# a10, a12, a13: smoothing, ranks, keep mask
# --------------------------------------------------------------------------

def gaussian_weights(k: int, sigma: float) -> np.ndarray:
    x = np.arange(k, dtype=F32) - F32((k - 1) / 2)
    w = np.exp(-(x ** 2) / F32(2 * sigma ** 2), dtype=F32)
    return (w / w.sum(dtype=F32)).astype(F32)


def smooth(scores: np.ndarray, k: int, gaussian: bool, sigma: float) -> np.ndarray:
    """PU:1884-1937: zero-padded conv1d with padding k//2, truncated to n."""
    n = len(scores)
    if k <= 1 or n <= k:
        return scores
    w = gaussian_weights(k, sigma) if gaussian else np.full(k, F32(1.0) / F32(k), dtype=F32)
    pad = k // 2
    padded = np.zeros(n + 2 * pad, dtype=F32)
    padded[pad:pad + n] = scores
    out_len = n + 2 * pad - k + 1
    out = np.zeros(out_len, dtype=F32)
    for t in range(k):
        out += w[t] * padded[t:t + out_len]
    return out[:n].astype(F32)


def stable_rank(scores: np.ndarray) -> np.ndarray:
    """``argsort(argsort(s))`` with a stable sort: equal values rank by index."""
    order = np.argsort(scores, kind="stable")
    ranks = np.empty(len(scores), dtype=np.int64)
    ranks[order] = np.arange(len(scores))
    return ranks


def rank_normalize(scores: np.ndarray) -> np.ndarray:
    """PU:1865-1882."""
    n = len(scores)
    if n <= 1:
        return np.ones(n, dtype=F32)
    return (stable_rank(scores).astype(F32) / F32(n - 1)).astype(F32)


def topk_lowest_index_ties(values: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest values; among values equal to the k-th, lowest index first."""
    if k <= 0:
        return np.zeros(0, dtype=np.int64)
    order = np.lexsort((np.arange(len(values)), -values.astype(np.float64)))
    return order[:k]


def keep_mask(scores: np.ndarray, budget: int, n: int, sink: int, window: int) -> np.ndarray:
    """PU:2591-2644 (static budget)."""
    target = max(int(budget), sink + window)
    mask = np.zeros(n, dtype=bool)
    mask[:sink] = True
    mask[max(sink, n - window):] = True
    remaining = max(0, target - int(mask.sum()))
    if remaining > 0:
        masked = scores[:n].astype(np.float64).copy()
        masked[mask] = -np.inf
        k = min(remaining, int((~mask).sum()))
        if k > 0:
            mask[topk_lowest_index_ties(masked, k)] = True
    return mask


def union_keep_mask(qi: np.ndarray, hi: np.ndarray, budget: int, n: int, sink: int, window: int,
                    qi_ratio: float) -> np.ndarray:
    """PU:2489-2589."""
    target = max(int(budget), sink + window)
    mask = np.zeros(n, dtype=bool)
    mask[:sink] = True
    mask[max(sink, n - window):] = True
    remaining = max(0, target - int(mask.sum()))
    if remaining <= 0:
        return mask
    qi_budget = int(remaining * qi_ratio)
    hi_budget = remaining - qi_budget
    cand = np.nonzero(~mask)[0]
    if len(cand) == 0:
        return mask
    qk = min(qi_budget, len(cand))
    hk = min(hi_budget, len(cand))
    sel = set(cand[topk_lowest_index_ties(qi[cand], qk)].tolist())
    sel |= set(cand[topk_lowest_index_ties(hi[cand], hk)].tolist())
    if len(sel) < remaining:
        shortfall = remaining - len(sel)
        ext_k = min(len(cand), hi_budget + shortfall + qi_budget)
        for idx in cand[topk_lowest_index_ties(hi[cand], ext_k)].tolist():
            if idx not in sel:
                sel.add(idx)
                if len(sel) >= remaining:
                    break
    mask[list(sel)] = True
    return mask


def select_from_vectors(a: np.ndarray, b: np.ndarray, p: Params, n: int) -> np.ndarray:
    """The shared-eviction selection from the two vectors it ranks, ascending kept
    prefix positions (local window excluded).

    ``a`` / ``b`` are the vectors after finishing and smoothing, exactly as ranked:
    QI / HI for "dis" (PU:3177-3196, ablations at 3186-3191, no bridge vector),
    influence / H2O for "max" / "weighted" (PU:3205-3242), the (DA-weighted) QI / HI
    for "union" / "union_da" (PU:2489-2589).  Keep mask: PU:2591-2644.
    """
    W, s, mode = p.window_size, p.sink_size, p.combination_mode
    if mode in ("union", "union_da"):
        mask = union_keep_mask(a, b, p.max_capacity_prompt, n, s, W, p.qi_ratio)
    else:
        ra, rb = rank_normalize(a), rank_normalize(b)
        if mode == "dis":
            if p.ablate_qi:
                ra = np.zeros_like(ra)
            if p.ablate_hi:
                rb = np.zeros_like(rb)
            comb = np.maximum(ra, rb)
        elif mode == "weighted":
            comb = (F32(p.h2o_weight) * rb + F32(1 - p.h2o_weight) * ra).astype(F32)
        else:
            comb = np.maximum(rb, ra)
        mask = keep_mask(comb, p.max_capacity_prompt, n, s, W)
    mask = mask.copy()
    mask[n - W:] = False
    return np.nonzero(mask)[0]


# --------------------------------------------------------------------------
# a16-a17: per-head mode
# --------------------------------------------------------------------------

def per_head_importance(attn: np.ndarray, p: Params):
    """PU:2208-2382 for batch 1: per-head QI (1-hop + 2-hop through the window) and HI."""
    H, W, n = attn.shape
    s = p.sink_size
    nt = n - s
    query = attn[:, -1, :]
    q2w = query[:, n - W:]
    two_hop = np.einsum("hr,hrj->hj", q2w, attn).astype(F32)
    eq = F32(p.resolved_qi_gamma() ** (p.neumann_iterations / 2))
    eh = F32(p.resolved_hi_gamma() ** (p.neumann_iterations / 2))
    res_qi = (query + eq * two_hop)[:, s:]
    if p.true_hub_hi:
        res_hi = attn[:, :, s:].sum(axis=1, dtype=F32)
    else:
        qt = query[:, s:]
        pos = np.arange(nt, dtype=F32)
        hw = ((F32(nt) - pos) / F32(nt))[None, :]
        res_hi = qt * hw * eh + qt
    out = []
    for res in (res_qi, res_hi):
        full = np.zeros((H, n), dtype=F32)
        full[:, s:] = res
        full[:, :s] = res.sum(axis=-1, keepdims=True, dtype=F32) * SINK_FRACTION
        mx = np.maximum(full.max(axis=-1, keepdims=True), F32(1e-8))
        out.append((full / mx).astype(F32))
    return out[0], out[1]


def per_head_vectors(attn: np.ndarray, p: Params, n: int):
    """PU:3296-3400: the per-head vectors the selection ranks, ``[H, 2, n - W]`` (QI and HI
    truncated to n - W and smoothed; with both ablations the second is the raw column sum
    over the window rows, H2O), and the query rows' entropies ``[H]``."""
    H, W, _ = attn.shape
    qi, hi = per_head_importance(attn, p)
    nw = n - W
    qi, hi = qi[:, :nw], hi[:, :nw]
    ksz = p.smoothing_kernel if p.smoothing_kernel > 0 else max(p.qi_kernel_size, p.hi_kernel_size)
    if ksz > 1:
        qi = np.stack([smooth(qi[h], ksz, True, p.gaussian_sigma) for h in range(H)])
        hi = np.stack([smooth(hi[h], ksz, True, p.gaussian_sigma) for h in range(H)])
    if p.ablate_hi and p.ablate_qi:
        hi = attn[:, :, :nw].sum(axis=1, dtype=F32)
    qa = attn[:, -1, :]
    ent = -(qa * np.log(qa + F32(1e-10))).sum(axis=-1, dtype=F32)
    return np.stack([qi, hi], axis=1).astype(F32), ent.astype(F32)


def per_head_scores_from(vec: np.ndarray, ent: np.ndarray, p: Params) -> np.ndarray:
    """PU:3400-3446: the per-head combined scores ``[H, nw]`` from the ranked vectors
    ``vec [H, 2, nw]`` and the query-row entropies ``ent [H]``."""
    H = vec.shape[0]
    qi, hi = vec[:, 0], vec[:, 1]
    qr = np.stack([rank_normalize(qi[h]) for h in range(H)])
    hr = np.stack([rank_normalize(hi[h]) for h in range(H)])
    if p.ablate_hi and not p.ablate_qi:
        return qr
    if p.ablate_qi and not p.ablate_hi:
        ghi = rank_normalize(hi.mean(axis=0, dtype=F32).astype(F32))
        return np.broadcast_to(ghi, qr.shape)
    if p.ablate_hi and p.ablate_qi:
        return hr
    if p.entropy_adaptive:
        lo, hi_e = ent.min(), ent.max()
        if hi_e > lo:
            w = (F32(1.0) - (ent - lo) / (hi_e - lo)).astype(F32)
        else:
            w = np.full(H, F32(0.5), dtype=F32)
        return (w[:, None] * qr + (F32(1.0) - w[:, None]) * hr).astype(F32)
    ghi = rank_normalize(hi.mean(axis=0, dtype=F32).astype(F32))
    return np.maximum(qr, ghi[None, :])


def per_head_select_from(vec: np.ndarray, ent: np.ndarray, p: Params, n: int):
    """PU:3400-3446: per-head index sets (sorted ascending) from the ranked vectors."""
    H, _, nw = vec.shape
    s = p.sink_size
    W = n - nw
    sc = per_head_scores_from(vec, ent, p)
    budget = p.max_capacity_prompt - W - s
    middle = nw - s
    sinks = np.arange(s)
    if middle > 0 and budget > 0:
        m = min(budget, middle)
        idx = [np.sort(np.concatenate([sinks, s + topk_lowest_index_ties(sc[h, s:], m)]))
               for h in range(H)]
        return np.stack(idx)
    return np.stack([sinks for _ in range(H)])


def per_head_select(attn: np.ndarray, p: Params, n: int):
    """PU:3296-3446: per-head index sets (sorted ascending), excluding the local window."""
    vec, ent = per_head_vectors(attn, p, n)
    return per_head_select_from(vec, ent, p, n)


# --------------------------------------------------------------------------
# a1: the whole update_kv (batch 1)
# --------------------------------------------------------------------------

@dataclass
class Result:
    keep_idx: np.ndarray                  # [B-W] ascending (shared) or [H, B-W] (per head)
    k_out: np.ndarray
    v_out: np.ndarray
    qi: Optional[np.ndarray] = None       # final QI scores fed to ranking (after smoothing)
    hi: Optional[np.ndarray] = None
    combined: Optional[np.ndarray] = None
    steps: int = 0
    choice: Optional[HeadChoice] = None
    extra: dict = field(default_factory=dict)


def update_kv(q: np.ndarray, k: np.ndarray, v: np.ndarray, groups: int, p: Params,
              dtype: str = "bf16", solver: str = "structured") -> Result:
    """Whole-path restatement of ``CircuitKVCluster.update_kv`` (PU:2775-3519), batch 1.

    ``q``: ``[H, n, D]``; ``k``/``v``: ``[Hkv, n, D]`` distinct KV heads.  Returns the
    kept indices and the compacted ``[H, B, D]`` K/V (in float32 holding the input
    dtype's values).
    """
    H, n, D = q.shape
    W = p.window_size
    s = p.sink_size
    if n < p.max_capacity_prompt:
        kk = np.repeat(k, groups, axis=0)
        vv = np.repeat(v, groups, axis=0)
        return Result(np.arange(n), kk, vv)
    attn = window_attention(q, k, W, groups, dtype)
    res = Result(np.zeros(0), None, None)
    if p.per_head_eviction:
        idx = per_head_select(attn, p, n)
        kk = np.repeat(k, groups, axis=0)
        vv = np.repeat(v, groups, axis=0)
        hs = np.arange(H)[:, None]
        k_out = np.concatenate([kk[hs, idx], kk[:, n - W:]], axis=1)
        v_out = np.concatenate([vv[hs, idx], vv[:, n - W:]], axis=1)
        return Result(idx, k_out, v_out)
    choice = choose_heads(attn, p)
    qi_rows, hi_rows = pool_rows(attn, choice)
    res.choice = choice
    qidx = n - 1
    mode = p.combination_mode
    solve = neumann_structured if solver == "structured" else None

    def run(chains):
        if solver == "structured":
            sc, st, _ = neumann_structured(chains, qidx, s, p.neumann_iterations,
                                           p.neumann_temperature, p.neumann_gamma)
        else:
            mats = [build_full_attn(ch.rows) for ch in chains]
            sc, st = neumann_dense(mats, qidx, s, p.neumann_iterations, p.neumann_temperature,
                                   p.neumann_gamma, starts=tuple(ch.start for ch in chains))
        return sc, st

    hi_src = hi_rows if hi_rows is not None else qi_rows
    if mode in ("dis", "union", "union_da"):
        (qi, hi), steps = run([Chain(qi_rows, "query"), Chain(hi_src, "uniform")])
        res.steps = steps
        if mode == "dis":
            qk = p.qi_kernel_size if p.qi_kernel_size != 0 else p.smoothing_kernel
            hk = p.hi_kernel_size if p.hi_kernel_size != 0 else p.smoothing_kernel
            if p.smooth_hi_only and qk > 1:
                qk = 0
            if qk > 1:
                qsig = p.gaussian_sigma * 0.5 if p.use_gaussian else 1.0
                qi = smooth(qi, qk, p.use_gaussian, qsig)
            if hk > 1:
                hi = smooth(hi, hk, p.use_gaussian, p.gaussian_sigma)
            qr = rank_normalize(qi)
            hr = rank_normalize(hi)
            br = None
            if p.use_bridge_importance:
                bi = bridge_importance(hi_src)
                if p.bi_kernel_size > 1:
                    bi = smooth(bi, p.bi_kernel_size, p.use_gaussian, p.gaussian_sigma)
                br = rank_normalize(bi)
            if p.ablate_qi:
                qr = np.zeros_like(qr)
            if p.ablate_hi:
                hr = np.zeros_like(hr)
            comb = np.maximum(qr, hr)
            if br is not None:
                comb = np.maximum(comb, br)
            mask = keep_mask(comb, p.max_capacity_prompt, n, s, W)
            res.qi, res.hi, res.combined = qi, hi, comb
        else:
            if mode == "union_da":
                da = np.maximum(qi_rows.sum(axis=0, dtype=F32), F32(1e-8))
                qi = (qi * da).astype(F32)
                hi = (hi * da).astype(F32)
            mask = union_keep_mask(qi, hi, p.max_capacity_prompt, n, s, W, p.qi_ratio)
            res.qi, res.hi = qi, hi
    else:
        (infl,), steps = run([Chain(qi_rows, "query")])
        res.steps = steps
        h2o = full_attn_colsum(qi_rows)
        hr = rank_normalize(h2o)
        ir = rank_normalize(infl)
        if mode == "weighted":
            comb = (F32(p.h2o_weight) * hr + F32(1 - p.h2o_weight) * ir).astype(F32)
        else:
            comb = np.maximum(hr, ir)
        mask = keep_mask(comb, p.max_capacity_prompt, n, s, W)
        res.qi, res.hi, res.combined = infl, h2o, comb
    nl = mask.copy()
    nl[n - W:] = False
    keep = np.nonzero(nl)[0]
    res.keep_idx = keep
    kk = np.repeat(k, groups, axis=0)
    vv = np.repeat(v, groups, axis=0)
    res.k_out = np.concatenate([kk[:, keep], kk[:, n - W:]], axis=1)
    res.v_out = np.concatenate([vv[:, keep], vv[:, n - W:]], axis=1)
    return res
