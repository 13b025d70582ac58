"""CPU restatement of the influence walker and its generators (test infrastructure only).

Follows CircuitKV/csrc/kernels/influence_walker.cu:66-456 (walker, positional
normalisation) common.cuh:48-93 (PCG) and circuit_walker.cu:157-171
(the PCG initialiser CircuitGraph uses).  The generators restate published
algorithms:

* pcg32 (PCG-XSH-RR, 64-bit state): M. E. O'Neill, "PCG: A Family of Simple Fast
  Space-Efficient Statistically Good Algorithms for Random Number Generation" (2014),
  seeding as in its reference implementation (state 0, inc = 2 * seq + 1, step, add
  the seed, step);
* Philox4x64-10: J. K. Salmon, M. A. Moraes, R. O. Dror, D. E. Shaw, "Parallel random
  numbers: as easy as 1, 2, 3" (SC'11); pinned against ``numpy.random.Philox``.

The walker's float32 arithmetic uses numpy's float32 power where the GPU (like the
reference, built with fast math) uses the __powf intrinsic, so individual draws that
fall within a few ulps of a cumulative-sum boundary can branch differently: compare
visit counts statistically.
"""

from __future__ import annotations

import numpy as np

MASK64 = (1 << 64) - 1
PCG_MULT = 6364136223846793005


class Pcg32:
    def __init__(self, initstate: int, initseq: int):
        self.state = 0
        self.inc = ((initseq << 1) | 1) & MASK64
        self.next()
        self.state = (self.state + initstate) & MASK64
        self.next()

    def next(self) -> int:
        old = self.state
        self.state = (old * PCG_MULT + self.inc) & MASK64
        xs = (((old >> 18) ^ old) >> 27) & 0xFFFFFFFF
        rot = old >> 59
        return ((xs >> rot) | (xs << ((-rot) & 31))) & 0xFFFFFFFF

    def uniform(self) -> np.float32:
        return np.float32(self.next() >> 8) * np.float32(1.0 / 16777216.0)


PHILOX_M = (0xD2E7470EE14C6C93, 0xCA5A826395121157)
PHILOX_W = (0x9E3779B97F4A7C15, 0xBB67AE8584CAA73B)


def philox4x64_10(ctr, key):
    c = list(ctr)
    k0, k1 = key
    for rnd in range(10):
        if rnd > 0:
            k0, k1 = (k0 + PHILOX_W[0]) & MASK64, (k1 + PHILOX_W[1]) & MASK64
        p0, p1 = PHILOX_M[0] * c[0], PHILOX_M[1] * c[2]
        hi0, lo0 = p0 >> 64, p0 & MASK64
        hi1, lo1 = p1 >> 64, p1 & MASK64
        c = [hi1 ^ c[1] ^ k0, lo1, hi0 ^ c[3] ^ k1, lo0]
    return c


class PhiloxWalker:
    """A walker's counter-based uniforms (the library's Philox mode): draw d of walker w
    in call c is word d % 4 of Philox4x64-10(counter (d // 4, w, c, 0), key (seed, 0)),
    its top 24 bits times 2^-24."""

    def __init__(self, seed: int, walker: int, call: int = 0):
        self.key = (seed & MASK64, 0)
        self.walker, self.call, self.draw = walker, call, 0
        self.blk = None

    def uniform(self) -> np.float32:
        if self.draw % 4 == 0:
            self.blk = philox4x64_10((self.draw // 4, self.walker, self.call, 0), self.key)
        bits = self.blk[self.draw % 4] >> 40
        self.draw += 1
        return np.float32(bits) * np.float32(1.0 / 16777216.0)


def philox_walkers(seed: int, num_walkers: int, call: int = 0):
    return [PhiloxWalker(seed, w, call) for w in range(num_walkers)]


def philox_stream(seed: int, stream_id: int, count: int):
    """The library's ckv_rng_fill(PHILOX) layout: block b = counter (b, stream, 0, 0)."""
    out = []
    for b in range((count + 3) // 4):
        out.extend(philox4x64_10((b, stream_id, 0, 0), (seed & MASK64, 0)))
    return out[:count]


def pcg_stream(seed: int, stream_id: int, count: int):
    g = Pcg32(seed & MASK64, stream_id)
    return [g.next() for _ in range(count)]


def seed_states(seed: int, num_walkers: int):
    """init_rng_kernel (circuit_walker.cu:157-171): walker w gets pcg_init(seed, w)."""
    return [Pcg32(seed, w) for w in range(num_walkers)]


def states_array(gens) -> np.ndarray:
    """The device layout of the states: [num_walkers][2] (state, inc) as int64 bits."""
    a = np.array([[g.state, g.inc] for g in gens], dtype=np.uint64)
    return a.view(np.int64).reshape(-1)


def influence_walk_dense(attn: np.ndarray, current_idx: int, num_walkers: int, max_steps: int, sink: int,
                         temperature: float = 2.0, explore_temp: float = 10.0, explore_ratio: float = 0.3,
                         seed: int = 3042, gens=None):
    """influence_walker.cu:66-171 with PCG walkers; ``gens`` carries the states from an
    earlier call (None: seeded (seed, w) as init_rng_kernel).  Returns (normalised scores,
    raw visits, gens) like get_influence_scores / get_influence_raw_visits."""
    n = attn.shape[0]
    A = attn.astype(np.float32)
    if gens is None:
        gens = seed_states(seed, num_walkers)
    visits = np.zeros(n, dtype=np.float32)
    it_base = np.float32(1.0) / np.float32(max(temperature, 0.1))
    it_expl = np.float32(1.0) / np.float32(max(explore_temp, 0.1))
    explore_start = int(np.float32(np.float32(1.0) - np.float32(explore_ratio)) * np.float32(num_walkers))
    for w in range(num_walkers):
        g = gens[w]
        it = it_expl if w >= explore_start else it_base
        if w < num_walkers // 2:
            pos = current_idx
        else:
            nvs = current_idx - sink + 1
            if nvs <= 0:
                pos = current_idx
            else:
                off = int(np.float32(g.uniform() * np.float32(nvs)))
                off = min(off, nvs - 1)
                pos = sink + off
        for _ in range(max_steps):
            if pos < sink:
                break
            wts = np.power(np.maximum(A[pos, sink:pos + 1], np.float32(1e-10)), it, dtype=np.float32)
            cs = np.cumsum(wts, dtype=np.float32)          # sequential float32 sums
            total = cs[-1]
            if total < np.float32(1e-10):
                break
            r = np.float32(g.uniform() * total)
            hit = np.nonzero(r < cs)[0]
            nxt = sink + (int(hit[0]) if len(hit) else len(cs) - 1)
            visits[nxt] += 1.0
            pos = nxt
    return normalise(visits, sink), visits, gens


def expected_visits(attn: np.ndarray, current_idx: int, num_walkers: int, max_steps: int, sink: int,
                    temperature: float = 2.0, explore_temp: float = 10.0, explore_ratio: float = 0.3):
    """Exact expectation of the visit counts (float64 Markov-chain propagation of the
    walkers' start distributions through the temperature-scaled transition rows)."""
    n = attn.shape[0]
    A = np.maximum(attn.astype(np.float64), 1e-10)
    explore_start = int(np.float32(np.float32(1.0) - np.float32(explore_ratio)) * np.float32(num_walkers))

    def trans(inv_t):
        P = np.zeros((n, n))
        for i in range(sink, n):
            w = A[i, sink:i + 1] ** inv_t
            P[i, sink:i + 1] = w / w.sum()
        return P

    out = np.zeros(n)
    half = num_walkers // 2
    nvs = current_idx - sink + 1
    for inv_t, lo, hi in ((1.0 / max(temperature, 0.1), 0, explore_start),
                          (1.0 / max(explore_temp, 0.1), explore_start, num_walkers)):
        if hi <= lo:
            continue
        P = trans(inv_t)
        n_query = max(0, min(hi, half) - lo)
        n_rand = (hi - lo) - n_query
        d = np.zeros(n)
        d[current_idx] += n_query
        if nvs > 0:
            d[sink:current_idx + 1] += n_rand / nvs
        else:
            d[current_idx] += n_rand
        for _ in range(max_steps):
            d = d @ P
            out += d
    return out


def normalise(visits: np.ndarray, sink: int) -> np.ndarray:
    """influence_walker.cu:296-456: visits / sqrt(n - p + 1), / max over the first
    min(n, 65536) non-sink positions, sinks = 1."""
    n = len(visits)
    p = np.arange(n)
    adj = np.where(p < sink, np.float32(0.0),
                   visits / np.sqrt((n - p + 1).astype(np.float32))).astype(np.float32)
    lim = min(n, min(256, (n + 255) // 256) * 256)
    m = adj[sink:lim].max() if lim > sink else np.float32(0.0)
    out = np.where(p < sink, np.float32(1.0), adj / m if m > 1e-10 else np.float32(0.0)).astype(np.float32)
    return out
