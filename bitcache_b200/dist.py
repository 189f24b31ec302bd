"""Multi-GPU decode: head sharding and sequence split over one process per GPU.

Head sharding (no data-path collective): rank r owns KV slots
[slot_range(r)) and the query heads that read them; every rank writes the
outputs of its own heads.

Sequence split (one exchange step): every rank holds a contiguous slice of
each slot's positions, runs the split-K decode kernel on it with
``partial`` output (per head m, l, o[d]), the triples are all-gathered over
NCCL (NVLink) and merged with the log-sum-exp rule on every rank.

The collective and the merge are passed in, so the host logic here runs
unchanged over NCCL on GPUs and over gloo on CPU in the tests.
"""
from __future__ import annotations

from typing import Callable

import torch


def seq_range(seq_len: int, world: int, rank: int, align: int = 8) -> tuple[int, int]:
    """Contiguous positions [start, end) of rank `rank`; boundaries are multiples of `align`
    so every shard's plane rows stay 16-byte aligned."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    chunk = -(-seq_len // world)
    chunk = -(-chunk // align) * align
    start = min(seq_len, rank * chunk)
    end = min(seq_len, start + chunk)
    return start, end


def slot_range(n_slots: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous KV slots [start, end) of rank `rank` (balanced, sizes differ by at most one)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    base, extra = divmod(n_slots, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def merge_partials_torch(parts: torch.Tensor) -> torch.Tensor:
    """Reference log-sum-exp merge in torch float64 for host-side checks:
    parts [n_parts, n_heads, d+2] (m, l, o) -> float32 [n_heads, d]."""
    p = parts.double()
    m, l, o = p[..., 0], p[..., 1], p[..., 2:]
    m = torch.where(l > 0, m, torch.full_like(m, float("-inf")))
    M = m.max(dim=0).values
    M = torch.where(torch.isfinite(M), M, torch.zeros_like(M))
    f = torch.exp(m - M)
    f = torch.where(l > 0, f, torch.zeros_like(f))
    L = (f * l).sum(0)
    O = (f[..., None] * o).sum(0)
    out = torch.where(L[:, None] > 0, O / L.clamp_min(1e-300)[:, None], torch.zeros_like(O))
    return out.float()


class SeqSplitStep:
    """One decode step of the sequence-split path on one rank.

    local_partial(q) -> float32 [n_heads, d+2]: this rank's triples (the
    decode kernel with partial output on GPU).
    all_gather(t) -> [world, ...]: the collective (NCCL all_gather_into_tensor
    on GPU, gloo in tests).
    merge(parts) -> [n_heads, d]: the log-sum-exp merge (bc_lse_merge on GPU).
    """

    def __init__(self, local_partial: Callable, all_gather: Callable, merge: Callable) -> None:
        self.local_partial = local_partial
        self.all_gather = all_gather
        self.merge = merge

    def __call__(self, q: torch.Tensor) -> torch.Tensor:
        part = self.local_partial(q)
        parts = self.all_gather(part)
        return self.merge(parts)


def nccl_all_gather(group=None) -> Callable[[torch.Tensor], torch.Tensor]:
    import torch.distributed as dist

    def fn(t: torch.Tensor) -> torch.Tensor:
        world = dist.get_world_size(group)
        out = torch.empty((world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(out, t.contiguous(), group=group)
        return out

    return fn
