"""Independent eviction units over the ranks of one node.

Each ``update_kv`` call (one layer of one sequence) is independent of every other, and
scoring needs all heads of a layer (entropy ranking and pooling run across heads), so
the units that shard are layers and sequences, never heads.  A rank scores its own
units with no collective on the data path; afterwards one all-gather shares the kept
positions of every unit (the metadata a cache manager needs to lay out the compacted
caches of all ranks).  Works on any ``torch.distributed`` backend: NCCL with CUDA
tensors on GPUs, gloo with CPU tensors in the CPU tests.
"""

from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence, Tuple

import torch


def layers_for_rank(num_layers: int, rank: int, world: int) -> List[int]:
    """Round-robin: layer l belongs to rank l % world."""
    if world < 1 or not (0 <= rank < world):
        raise ValueError("need 0 <= rank < world")
    return [l for l in range(num_layers) if l % world == rank]


def sequences_for_rank(lengths: Sequence[int], rank: int, world: int) -> List[int]:
    """Greedy longest-first balance of ragged sequences (cost grows with n): each
    sequence, longest first (ties: lower index first), goes to the least-loaded rank
    (ties: lower rank).  Deterministic, so every rank computes the same assignment."""
    if world < 1 or not (0 <= rank < world):
        raise ValueError("need 0 <= rank < world")
    load = [0] * world
    owner = [0] * len(lengths)
    for i in sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i)):
        r = min(range(world), key=lambda r: (load[r], r))
        owner[i] = r
        load[r] += int(lengths[i])
    return [i for i in range(len(lengths)) if owner[i] == rank]


def _pack(local: Dict[int, torch.Tensor]) -> torch.Tensor:
    """[count, (unit, ndim, rows, cols) * count, data...] as one int32 vector."""
    head = [len(local)]
    body = []
    for unit in sorted(local):
        t = local[unit].to(torch.int32)
        if t.dim() == 2:
            t2 = t
        elif t.dim() <= 1:
            t2 = t.reshape(1, t.numel())
        else:
            raise ValueError("kept indices are [kept] or [heads, kept]")
        head += [int(unit), 2 if t.dim() == 2 else 1, int(t2.shape[0]), int(t2.shape[1])]
        body.append(t2.reshape(-1).cpu())
    return torch.cat([torch.tensor(head, dtype=torch.int32)] + body)


def _unpack(buf: torch.Tensor, out: Dict[int, torch.Tensor]) -> None:
    count = int(buf[0])
    pos = 1 + 4 * count
    for c in range(count):
        unit, ndim, rows, cols = (int(x) for x in buf[1 + 4 * c: 5 + 4 * c])
        t = buf[pos: pos + rows * cols].reshape(rows, cols)
        out[unit] = t.clone() if ndim == 2 else t.reshape(-1).clone()
        pos += rows * cols


def gather_kept(local: Dict[int, torch.Tensor], group=None,
                device: Optional[torch.device] = None) -> Dict[int, torch.Tensor]:
    """All-gather of every rank's kept positions: ``local`` maps unit id -> kept index
    tensor (``[kept]`` shared or ``[heads, kept]`` per head); returns the map of all
    units on every rank (CPU int32 tensors).  Two collectives: the sizes, then the
    padded payloads.  ``device``: where the collective's buffers live (CUDA for NCCL)."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    dev = device if device is not None else torch.device("cpu")
    mine = _pack(local)
    size = torch.tensor([mine.numel()], dtype=torch.int64, device=dev)
    sizes = [torch.zeros_like(size) for _ in range(world)]
    dist.all_gather(sizes, size, group=group)
    cap = int(max(int(s.item()) for s in sizes))
    padded = torch.zeros(cap, dtype=torch.int32, device=dev)
    padded[: mine.numel()] = mine.to(dev)
    bufs = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(bufs, padded, group=group)
    out: Dict[int, torch.Tensor] = {}
    for b, s in zip(bufs, sizes):
        _unpack(b[: int(s.item())].cpu(), out)
    return out


def max_over_ranks(x: float, group=None, device: Optional[torch.device] = None) -> float:
    """The step time of a multi-rank run: the slowest rank's."""
    import torch.distributed as dist

    t = torch.tensor([float(x)], dtype=torch.float64, device=device or torch.device("cpu"))
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


class KeptExchange:
    """The kept positions of every unit, shared by ONE all-gather with no host round trip.

    Each unit's owner and kept-index shape are known to every rank in advance (they follow
    from the sequence lengths, budgets and the assignment above), so each rank lays its
    units out in one int32 buffer of a common capacity, lets the scoring call write each
    unit's kept positions straight into its slice (``out(unit)``), and ``exchange()`` runs
    a single ``all_gather_into_tensor`` into ``[world * cap]``; ``result(unit)`` is a view of
    any unit's positions there.  The collective can be enqueued right after the scoring
    work on the same stream (NCCL) without synchronising the host.
    """

    def __init__(self, shapes: Dict[int, Tuple[int, ...]], owner: Dict[int, int], rank: int, world: int,
                 device: Optional[torch.device] = None):
        if set(shapes) != set(owner):
            raise ValueError("every unit needs a shape and an owner")
        self.rank, self.world = rank, world
        used = [0] * world
        self.slots = {}
        for u in sorted(shapes):
            r = int(owner[u])
            if not 0 <= r < world:
                raise ValueError("owner out of range")
            size = int(math.prod(shapes[u]))
            self.slots[u] = (r, used[r], tuple(int(x) for x in shapes[u]))
            used[r] += size
        self.cap = max(1, max(used))
        dev = device if device is not None else torch.device("cpu")
        self.local = torch.zeros(self.cap, dtype=torch.int32, device=dev)
        self.all = torch.zeros(world * self.cap, dtype=torch.int32, device=dev)

    def units_of(self, rank: int) -> List[int]:
        return [u for u, (r, _, _) in sorted(self.slots.items()) if r == rank]

    def out(self, unit: int) -> torch.Tensor:
        r, off, shape = self.slots[unit]
        if r != self.rank:
            raise ValueError("unit owned by another rank")
        return self.local[off: off + math.prod(shape)].view(shape)

    def exchange(self, group=None) -> None:
        import torch.distributed as dist
        dist.all_gather_into_tensor(self.all, self.local, group=group)

    def result(self, unit: int) -> torch.Tensor:
        r, off, shape = self.slots[unit]
        base = r * self.cap + off
        return self.all[base: base + math.prod(shape)].view(shape)
