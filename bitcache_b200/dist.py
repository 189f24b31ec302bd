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

PeerExchange is the fused alternative for the sequence split: the decode
kernel itself stores each head's triple into every rank's buffer over
NVLink as 64-bit (value, epoch) words and merges once every word it needs
carries the call's epoch (bc_decode_attention_xchg), so a step is one launch
per rank with no separate collective or merge.
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


class PeerExchange:
    """Exchange buffers for bc_decode_attention_xchg (one process per GPU).

    Construction is collective over `group` (torch.distributed): every rank
    allocates its buffer (bc_xchg_alloc), the 64-byte CUDA IPC handles are
    all-gathered, and the peers' buffers are mapped (bc_ipc_open).  With
    world size 1 (no process group) the buffer is only this rank's own.
    """

    def __init__(self, n_heads: int, head_dim: int, group=None, spin_limit: int = 0) -> None:
        import ctypes

        from . import _lib

        dist = torch.distributed
        self._lib = _lib
        lib = _lib.load()
        on = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if on else 1
        self.rank = dist.get_rank(group) if on else 0
        if self.world > 8:
            raise RuntimeError("PeerExchange supports up to 8 ranks")
        self.n_heads, self.head_dim = n_heads, head_dim
        nbytes = lib.bc_xchg_bytes(n_heads, head_dim, self.world)
        own = ctypes.c_void_p()
        _lib.check(lib.bc_xchg_alloc(nbytes, ctypes.byref(own)), "xchg_alloc")
        self._own = own.value
        self._opened: list[int] = []
        bufs = [0] * self.world
        bufs[self.rank] = self._own
        if self.world > 1:
            handle = (ctypes.c_char * 64)()
            _lib.check(lib.bc_ipc_handle(self._own, handle), "ipc_handle")
            handles: list = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
            for j in range(self.world):
                if j == self.rank:
                    continue
                p = ctypes.c_void_p()
                hb = (ctypes.c_char * 64).from_buffer_copy(handles[j])
                _lib.check(lib.bc_ipc_open(hb, ctypes.byref(p)), "ipc_open")
                bufs[j] = p.value
                self._opened.append(p.value)
        self._x = _lib.Xchg()
        for j, b in enumerate(bufs):
            self._x.bufs[j] = b
        self._x.world, self._x.rank, self._x.epoch = self.world, self.rank, 0
        # polls of one exchange word before the kernel gives up (0: about a second)
        self._x.spin_limit = spin_limit
        self._x.buf_bytes = nbytes

    def decode(self, q: torch.Tensor, K, V, seq_len: int, mode: int, out: torch.Tensor | None = None) -> torch.Tensor:
        """One sequence-split decode step: this rank's slice [K, V] of every slot,
        the merged output of all heads on every rank.  q and out may be pinned
        host tensors: q is staged to the device first (planes.device_query), and
        the kernel writes out over the host link itself."""
        from . import planes
        lib = self._lib.load()
        d = q.shape[-1]
        n_heads = q.numel() // d
        n_slots = K.n_slots
        group = n_heads // n_slots
        # the exchange buffers were sized for (n_heads, head_dim) of __init__;
        # every rank stores into every other rank's buffer, so a larger call
        # would write past the end of a peer's buffer
        if n_heads != self.n_heads or d != self.head_dim:
            raise RuntimeError(f"PeerExchange built for {self.n_heads} heads of dim {self.head_dim}, "
                               f"called with {n_heads} heads of dim {d}")
        if group * n_slots != n_heads:
            raise RuntimeError("number of query heads must be a multiple of the number of KV slots")
        if out is not None:
            planes._check_half_dev_or_pinned(out, "out")
            if out.numel() < n_heads * d:
                raise RuntimeError(f"out holds {out.numel()} elements, the call writes {n_heads * d}")
        q = planes.device_query(q, K.sign.device)
        if out is None:
            out = torch.empty((n_heads, d), dtype=torch.float16, device=q.device)
        st = self._lib.stream_of(q.device)
        wsb = lib.bc_decode_workspace_bytes(n_slots, group, seq_len, d)
        ws = self._lib.workspace(q.device, st, wsb, ("decode", n_slots, group))
        self._x.epoch += 1
        self._lib.check(lib.bc_decode_attention_xchg(q.data_ptr(), K.c(), V.c(), out.data_ptr(), n_slots, group,
                                                     seq_len, K.kv_stride, d, mode, self._x, self._lib.ptr(ws),
                                                     ws.numel() if ws is not None else 0, st), "decode_attention_xchg")
        return out

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (after all ranks are done with it)."""
        lib = self._lib.load()
        torch.cuda.synchronize()
        if self.world > 1 and torch.distributed.is_initialized():
            torch.distributed.barrier()
        for p in self._opened:
            lib.bc_ipc_close(p)
        self._opened = []
        if self._own:
            lib.bc_xchg_free(self._own)
            self._own = None
