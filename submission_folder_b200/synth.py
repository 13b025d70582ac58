"""Seeded synthetic prefill caches with planted structure.

Stands in for the LongBench / RULER prompts the reference evaluates on (their
data is not shipped).  Shapes follow a Llama-3-8B / Mistral-7B layer: 32 query
heads, 8 KV heads, head_dim 128.

Distribution (per layer, per KV group ``g`` of ``groups`` query heads):

* ``Q``, ``K`` i.i.d. ``N(0, qk_scale^2)`` per component, ``V`` i.i.d. ``N(0, 1)``.
  With the default ``qk_scale = 1`` the scaled logits ``q.k / sqrt(D)`` are
  ``N(0, 1)``; ``qk_scale = 1/sqrt(D)`` gives the literal ``N(0,1)/sqrt(128)``
  components, whose logits have standard deviation ~0.008 (near-uniform attention).
* ``u_g`` = unit mean of the window queries of the group's query heads.
* sinks: keys ``0..3`` get ``+c u_g`` with ``c`` chosen so the mean window query's
  logit rises by ``sink_boost`` (3).
* locality: the last ``locality`` keys get ``+c u_g`` for a logit rise of 1.
* planted tokens: ``planted`` random positions per KV group get keys
  ``||k|| (0.8 u_g + 0.6 w)`` with ``w`` a random unit vector orthogonal to
  ``u_g`` (cosine 0.8 with the mean window query).
* values are generated in float32 and cast to the requested dtype last.
* ``grid_step > 0`` (exact-arithmetic inputs): ``Q`` and ``K`` are finally rounded to
  multiples of ``grid_step`` with at most 15 steps either side of zero.  With the
  default 0.25 every product ``q_d k_d`` is a multiple of 1/16 and every partial sum of
  a 128-term dot product is exactly representable in fp32, so the logits are the same
  bits in any summation order (CPU BLAS, cuBLAS, tensor-core MMA).
"""

from __future__ import annotations

import math

import torch

DTYPES = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}


def make_layer(n: int, *, seed: int = 0, layer: int = 0, heads: int = 32, kv_heads: int = 8,
               head_dim: int = 128, window: int = 64, planted: int = 16, locality: int = 256,
               sink: int = 4, sink_boost: float = 3.0, locality_boost: float = 1.0,
               qk_scale: float = 1.0, dtype: str = "bf16", device: str = "cpu", grid_step: float = 0.0):
    """Return ``(q [H,n,D], k [Hkv,n,D], v [Hkv,n,D])`` for one layer.

    Generation happens on ``device`` with a generator seeded from ``(seed, layer)``;
    CPU generation is reproducible across machines for the same torch build.
    """
    groups = heads // kv_heads
    gen = torch.Generator(device=device)
    gen.manual_seed(int(seed) * 1_000_003 + int(layer))
    f32 = torch.float32
    q = torch.randn(heads, n, head_dim, generator=gen, device=device, dtype=f32) * qk_scale
    k = torch.randn(kv_heads, n, head_dim, generator=gen, device=device, dtype=f32) * qk_scale
    v = torch.randn(kv_heads, n, head_dim, generator=gen, device=device, dtype=f32)
    w0 = max(0, n - window)
    sq = math.sqrt(head_dim)
    for g in range(kv_heads):
        qm = q[g * groups:(g + 1) * groups, w0:, :].reshape(-1, head_dim).mean(dim=0)
        norm = qm.norm().clamp_min(1e-12)
        u = qm / norm
        unit_c = sq / norm            # adding unit_c*u raises the mean query's logit by 1
        s = min(sink, n)
        k[g, :s] += sink_boost * unit_c * u
        lo = max(0, n - locality)
        k[g, lo:] += locality_boost * unit_c * u
        if planted > 0 and n > sink + 1:
            cnt = min(planted, n - sink)
            pos = torch.randperm(n - sink, generator=gen, device=device)[:cnt] + sink
            r = torch.randn(cnt, head_dim, generator=gen, device=device, dtype=f32)
            r = r - (r @ u)[:, None] * u[None, :]
            r = r / r.norm(dim=1, keepdim=True).clamp_min(1e-12)
            kn = k[g, pos].norm(dim=1, keepdim=True)
            k[g, pos] = kn * (0.8 * u[None, :] + 0.6 * r)
    if grid_step > 0:
        q = torch.clamp(torch.round(q / grid_step), -15, 15) * grid_step
        k = torch.clamp(torch.round(k / grid_step), -15, 15) * grid_step
    dt = DTYPES[dtype]
    return q.to(dt), k.to(dt), v.to(dt)


def repeat_kv(x: torch.Tensor, groups: int) -> torch.Tensor:
    """``[Hkv, n, D]`` -> ``[1, Hkv*groups, n, D]`` materialised like HF ``repeat_kv``."""
    hkv, n, d = x.shape
    return x[:, None].expand(hkv, groups, n, d).reshape(1, hkv * groups, n, d)


def ragged_lengths(batch: int, lo: int, hi: int, seed: int = 0):
    """Seeded sequence lengths uniform in ``[lo, hi]`` (the batched serving sweep)."""
    gen = torch.Generator().manual_seed(int(seed))
    return [int(x) for x in torch.randint(lo, hi + 1, (batch,), generator=gen)]
