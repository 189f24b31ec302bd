"""Native plane-layout cache and the B200 decode-path operators on it.

Layout (per K or V cache; include/bitcache_b200.h):
    sign   uint32 [slots, kv_stride, head_dim/32]
    nib    uint8  [slots, kv_stride, head_dim/2] bytes, interleaved in blocks of 8
           positions (16-byte chunk c of position p at (p/8)*4d + 128c + 16(p%8));
           nib_rows() gives the per-position view    (compensated caches only)
    bscale fp16   [slots, kv_stride]
    rscale fp16   [slots, kv_stride]                (compensated caches only)
kv_stride is the position capacity rounded up to a multiple of 8 so every
per-slot row of the scale planes starts on a 16-byte boundary (the TMA bulk
copies in the decode kernel need 16-byte aligned sources and sizes).
"""
from __future__ import annotations

import functools
from dataclasses import dataclass

import torch

from . import _lib

RES_NONE, RES_FP16_SCALE, RES_FP32_SCALE = _lib.BC_RES_NONE, _lib.BC_RES_FP16_SCALE, _lib.BC_RES_FP32_SCALE
MODE_BINARY, MODE_COMPENSATED = _lib.BC_MODE_BINARY, _lib.BC_MODE_COMPENSATED


def round_stride(max_seq: int) -> int:
    return (max_seq + 7) // 8 * 8


def vector_bytes(head_dim: int, compensated: bool = True) -> int:
    """Stored bytes per K or V vector: 5d/8 + 4 (d/8 + 2 binary only)."""
    return head_dim // 8 + 2 + ((head_dim // 2 + 2) if compensated else 0)


@dataclass
class Planes:
    """One K or V plane cache."""

    sign: torch.Tensor
    bscale: torch.Tensor
    nib: torch.Tensor | None
    rscale: torch.Tensor | None
    head_dim: int

    @staticmethod
    def empty(n_slots: int, kv_stride: int, head_dim: int, compensated: bool, device, zero: bool = True) -> "Planes":
        assert kv_stride % 8 == 0, "kv_stride must be a multiple of 8"
        mk = torch.zeros if zero else torch.empty
        sign = mk((n_slots, kv_stride, head_dim // 32), dtype=torch.int32, device=device)
        bscale = mk((n_slots, kv_stride), dtype=torch.float16, device=device)
        nib = rscale = None
        if compensated:
            # zero codes are 0x88 bytes in the offset-binary nibble plane
            nib = (torch.full if zero else torch.empty)(
                (n_slots, kv_stride, head_dim // 2), *((0x88,) if zero else ()), dtype=torch.uint8, device=device)
            rscale = mk((n_slots, kv_stride), dtype=torch.float16, device=device)
        return Planes(sign, bscale, nib, rscale, head_dim)

    @property
    def n_slots(self) -> int:
        return self.sign.shape[0]

    @property
    def kv_stride(self) -> int:
        return self.sign.shape[1]

    @property
    def compensated(self) -> bool:
        return self.nib is not None

    def c(self) -> _lib.KVPlanes:
        return _lib.KVPlanes(_lib.ptr(self.sign), _lib.ptr(self.nib), _lib.ptr(self.bscale), _lib.ptr(self.rscale))

    def nib_rows(self) -> torch.Tensor:
        """The INT4 codes per position, uint8 [slots, kv_stride, head_dim/2] (a copy)."""
        return nib_rows(self.nib, self.head_dim)

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.sign, self.bscale, self.nib, self.rscale)
                   if t is not None)

    def zero_(self) -> None:
        """Reset to all-zero fields (nibble bytes 0x88 = codes 0)."""
        for t in (self.sign, self.bscale, self.rscale):
            if t is not None:
                t.zero_()
        if self.nib is not None:
            self.nib.fill_(0x88)


def _by_bit(head_dim: int) -> bool:
    """Nibble order of the planes.  At head dims 64, 128 and 256 every plane byte holds
    bits t and t + 4 (t < 4) of one sign byte b, i.e. dims 8b + t (low nibble) and
    8b + t + 4 (high), placed so that one 16-byte chunk lines up with one 16-byte window
    of the sign row (`_nib_dims` gives the placement).  Other head dims keep the
    reference's order: byte j of chunk c holds dims 32c + 2j and 32c + 2j + 1."""
    return head_dim in (64, 128, 256)


@functools.lru_cache(maxsize=None)
def _nib_dims(head_dim: int) -> tuple[torch.Tensor, torch.Tensor]:
    """(low, high): the dim held by each nibble of a plane row in chunk order, byte
    p = 16c + j (the same rule as the kernels' nib_dim)."""
    c = torch.arange(head_dim // 2) // 16
    j = torch.arange(head_dim // 2) % 16
    if head_dim == 128:
        lo = 8 * j + c
    elif head_dim == 256:
        lo = 128 * (c // 4) + 8 * j + c % 4
    elif head_dim == 64:
        lo = 8 * (j % 8) + 2 * c + j // 8
    else:
        return 32 * c + 2 * j, 32 * c + 2 * j + 1
    return lo, lo + 4


def _chunk_rows(nib: torch.Tensor, head_dim: int) -> torch.Tensor:
    slots, stride = nib.shape[0], nib.shape[1]
    return (nib.reshape(slots, stride // 8, head_dim // 32, 8, 16).permute(0, 1, 3, 2, 4)
            .reshape(slots, stride, head_dim // 2))


def nib_rows(nib: torch.Tensor, head_dim: int) -> torch.Tensor:
    """De-interleave a nibble plane [slots, kv_stride, head_dim/2] into per-position rows of
    the reference's byte format (two's-complement codes, element 2i in the low nibble)."""
    rows = torch.bitwise_xor(_chunk_rows(nib, head_dim), 0x88)
    if _by_bit(head_dim):  # chunk-order bytes -> codes in dim order -> reference bytes
        lo, hi = _nib_dims(head_dim)
        order = torch.argsort(torch.cat([lo, hi])).to(rows.device)
        codes = torch.cat([rows & 0xF, rows >> 4], -1).index_select(-1, order)
        rows = codes[..., 0::2] | (codes[..., 1::2] << 4)
    return rows.contiguous()


def nib_interleave(rows: torch.Tensor, head_dim: int) -> torch.Tensor:
    """Inverse of nib_rows: reference-format rows [slots, kv_stride, head_dim/2] -> plane bytes."""
    slots, stride = rows.shape[0], rows.shape[1]
    x = rows
    if _by_bit(head_dim):  # reference bytes -> codes in dim order -> chunk-order bytes
        lo, hi = _nib_dims(head_dim)
        codes = torch.stack([x & 0xF, x >> 4], -1).reshape(slots, stride, head_dim)
        x = codes.index_select(-1, lo.to(x.device)) | (codes.index_select(-1, hi.to(x.device)) << 4)
    x = torch.bitwise_xor(x, 0x88)
    return (x.reshape(slots, stride // 8, 8, head_dim // 32, 16).permute(0, 1, 3, 2, 4)
            .reshape(slots, stride, head_dim // 2).contiguous())


def _stream(t: torch.Tensor) -> int:
    return _lib.stream_of(t.device)


def _check_half(x: torch.Tensor, name: str) -> None:
    if not x.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if not x.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")
    if x.dtype != torch.float16:
        raise RuntimeError(f"{name} must be float16")


def _check_half_dev_or_pinned(x: torch.Tensor, name: str) -> None:
    """fp16, contiguous, and either on the GPU or in pinned (page-locked) host memory,
    which kernels read and write directly through unified addressing."""
    if not (x.is_cuda or x.is_pinned()):
        raise RuntimeError(f"{name} must be a CUDA tensor or a pinned host tensor")
    if not x.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")
    if x.dtype != torch.float16:
        raise RuntimeError(f"{name} must be float16")


# Device buffers that pinned host queries are staged into, per (device, stream, elements).
_qstage: dict[tuple, torch.Tensor] = {}


def device_query(q: torch.Tensor, device: torch.device) -> torch.Tensor:
    """q itself when it is on the GPU; a pinned host q is copied to a device buffer
    (one per device, stream and size, reused by later calls) by one bc_stage_rows launch on
    the current stream.  That kernel reads the host before it waits for the previous
    kernel in the stream, so the host must not rewrite q while earlier steps that
    read it are still queued."""
    if q.is_cuda:
        _check_half(q, "Q")
        return q
    _check_half_dev_or_pinned(q, "Q")
    if q.data_ptr() % 16 or (2 * q.numel()) % 16:
        raise RuntimeError("a pinned host Q must be 16-byte aligned and a multiple of 16 bytes")
    key = (device, _lib.stream_of(device), q.numel())  # per stream: calls on one stream are ordered
    buf = _qstage.get(key)
    if buf is None:
        buf = _qstage[key] = torch.empty(q.numel(), dtype=torch.float16, device=device)
    stage_rows([(q.reshape(-1), buf)])
    return buf.view(q.shape)


def encode_planes(src: torch.Tensor, out: Planes, residual_mode: int = RES_FP16_SCALE) -> None:
    """Prefill: encode src fp16 [n_slots, seq_len, head_dim] into rows [slot, 0:seq_len] of out."""
    _check_half(src, "src")
    n_slots, seq_len, d = src.shape
    lib = _lib.load()
    _lib.check(lib.bc_encode_planes(src.data_ptr(), out.c(), n_slots, seq_len, out.kv_stride, d, residual_mode,
                                    _stream(src)), "encode_planes")


def append_kv(k: torch.Tensor, v: torch.Tensor, K: Planes, V: Planes, pos: int,
              residual_mode: int = RES_FP32_SCALE) -> None:
    """Decode-step append of one K and one V token per slot ([n_slots, head_dim]) at position pos."""
    _check_half(k, "K")
    _check_half(v, "V")
    d = k.shape[-1]
    n_slots = k.numel() // d
    lib = _lib.load()
    _lib.check(lib.bc_append_kv(k.data_ptr(), v.data_ptr(), K.c(), V.c(), n_slots, d, K.kv_stride, pos,
                                residual_mode, _stream(k)), "append_kv")


def decode_attention(q: torch.Tensor, K: Planes, V: Planes, seq_len: int, mode: int = MODE_COMPENSATED,
                     out: torch.Tensor | None = None, partial: torch.Tensor | None = None,
                     want_out: bool = True) -> torch.Tensor | None:
    """Fused split-K decode attention.

    q fp16 [n_slots * group, head_dim] (query head h reads KV slot h // group).
    Returns out fp16 [n_heads, head_dim] (or None when want_out is False and a
    partial buffer float32 [n_heads, head_dim + 2] is given)."""
    _check_half(q, "Q")
    d = q.shape[-1]
    n_heads = q.numel() // d
    n_slots = K.n_slots
    group = n_heads // n_slots
    if group * n_slots != n_heads:
        raise RuntimeError("number of query heads must be a multiple of the number of KV slots")
    if want_out and out is None:
        out = torch.empty((n_heads, d), dtype=torch.float16, device=q.device)
    lib = _lib.load()
    st = _stream(q)
    wsb = lib.bc_decode_workspace_bytes(n_slots, group, seq_len, d)
    ws = _lib.workspace(q.device, st, wsb, ("decode", n_slots, group))
    _lib.check(lib.bc_decode_attention(q.data_ptr(), K.c(), V.c(), _lib.ptr(out) if want_out else None,
                                       _lib.ptr(partial), n_slots, group, seq_len, K.kv_stride, d, mode,
                                       _lib.ptr(ws), ws.numel() if ws is not None else 0, st),
               "decode_attention")
    return out


def decode_step(q: torch.Tensor, k: torch.Tensor | None, v: torch.Tensor | None, K: Planes, V: Planes,
                seq_len: int, append_pos: int, mode: int = MODE_COMPENSATED, residual_mode: int = RES_FP32_SCALE,
                out: torch.Tensor | None = None, partial: torch.Tensor | None = None,
                want_out: bool = True) -> torch.Tensor | None:
    """Fused decode step: append k, v ([n_slots, head_dim]) at append_pos with residual_mode
    arithmetic, then attend q over keys [0, seq_len), in one launch (bc_decode_step).
    append_pos = -1 (k, v None) attends only.  Results equal append_kv + decode_attention.
    q, k, v and out may be pinned host tensors: the kernel then reads the step's inputs
    and writes its output over the host link itself, with no separate copies."""
    _check_half_dev_or_pinned(q, "Q")
    if append_pos >= 0:
        _check_half_dev_or_pinned(k, "K")
        _check_half_dev_or_pinned(v, "V")
    d = q.shape[-1]
    n_heads = q.numel() // d
    n_slots = K.n_slots
    group = n_heads // n_slots
    if group * n_slots != n_heads:
        raise RuntimeError("number of query heads must be a multiple of the number of KV slots")
    if append_pos >= 0 and (k.numel() != n_slots * d or v.numel() != n_slots * d):
        raise RuntimeError("k and v must hold one head_dim row per KV slot")
    if want_out and out is None:
        out = (torch.empty((n_heads, d), dtype=torch.float16, device=q.device) if q.is_cuda
               else torch.empty((n_heads, d), dtype=torch.float16).pin_memory())
    if want_out:
        _check_half_dev_or_pinned(out, "out")
    dev = K.sign.device
    lib = _lib.load()
    st = _lib.stream_of(dev)
    wsb = lib.bc_decode_workspace_bytes(n_slots, group, seq_len, d)
    ws = _lib.workspace(dev, st, wsb, ("decode", n_slots, group))
    _lib.check(lib.bc_decode_step(q.data_ptr(), _lib.ptr(k) if append_pos >= 0 else None,
                                  _lib.ptr(v) if append_pos >= 0 else None, K.c(), V.c(),
                                  _lib.ptr(out) if want_out else None, _lib.ptr(partial), n_slots, group, seq_len,
                                  K.kv_stride, d, mode, append_pos, residual_mode, _lib.ptr(ws),
                                  ws.numel() if ws is not None else 0, st),
               "decode_step")
    return out


@dataclass
class PageTable:
    """Block table of a paged cache (bc_page_table).

    The K and V pools are ``Planes`` with ``n_slots = n_pages`` and
    ``kv_stride = page_size``; logical position ``pos`` of slot ``s`` lives in
    pool row ``pages[s, pos // page_size] * page_size + pos % page_size``.
    ``page_size`` is a multiple of 128 (the decode tile)."""

    pages: torch.Tensor  # int32 [n_slots, max_pages], device
    page_size: int
    n_pages: int

    def c(self) -> _lib.PageTable:
        return _lib.PageTable(self.pages.data_ptr(), self.pages.shape[1], self.page_size, self.n_pages)

    @property
    def n_slots(self) -> int:
        return self.pages.shape[0]


def paginate(P: Planes, pt: PageTable, seq_len: int, pool: Planes | None = None) -> Planes:
    """Copy positions [0, seq_len) of a contiguous cache into a page pool laid out by pt
    (page-sized row blocks; the nibble interleave is per 8 rows, so blocks copy as bytes)."""
    ps = pt.page_size
    if pool is None:
        pool = Planes.empty(pt.n_pages, ps, P.head_dim, P.compensated, P.sign.device)
    table = pt.pages.cpu()
    for s in range(pt.n_slots):
        for j in range((seq_len + ps - 1) // ps):
            pg = int(table[s, j])
            for name in ("sign", "bscale", "nib", "rscale"):
                src, dst = getattr(P, name), getattr(pool, name)
                if src is not None:
                    dst[pg].copy_(src[s, j * ps:(j + 1) * ps])
    return pool


def decode_step_paged(q: torch.Tensor, k: torch.Tensor | None, v: torch.Tensor | None, K: Planes, V: Planes,
                      pt: PageTable, seq_len: int, append_pos: int = -1, mode: int = MODE_COMPENSATED,
                      residual_mode: int = RES_FP32_SCALE, out: torch.Tensor | None = None,
                      partial: torch.Tensor | None = None, want_out: bool = True) -> torch.Tensor | None:
    """bc_decode_step_paged: optional append at logical append_pos, then attention over
    logical keys [0, seq_len) of the paged cache (pools K, V and block table pt)."""
    _check_half(q, "Q")
    if append_pos >= 0:
        _check_half(k, "K")
        _check_half(v, "V")
    d = q.shape[-1]
    n_heads = q.numel() // d
    n_slots = pt.n_slots
    group = n_heads // n_slots
    if group * n_slots != n_heads:
        raise RuntimeError("number of query heads must be a multiple of the number of KV slots")
    if want_out and out is None:
        out = torch.empty((n_heads, d), dtype=torch.float16, device=q.device)
    lib = _lib.load()
    st = _stream(q)
    wsb = lib.bc_decode_workspace_bytes(n_slots, group, seq_len, d)
    ws = _lib.workspace(q.device, st, wsb, ("decode", n_slots, group))
    _lib.check(lib.bc_decode_step_paged(q.data_ptr(), _lib.ptr(k) if append_pos >= 0 else None,
                                        _lib.ptr(v) if append_pos >= 0 else None, K.c(), V.c(),
                                        _lib.ptr(out) if want_out else None, _lib.ptr(partial), pt.c(), n_slots,
                                        group, seq_len, d, mode, append_pos, residual_mode, _lib.ptr(ws),
                                        ws.numel() if ws is not None else 0, st),
               "decode_step_paged")
    return out


def append_kv_paged(k: torch.Tensor, v: torch.Tensor, K: Planes, V: Planes, pt: PageTable, pos: int,
                    residual_mode: int = RES_FP32_SCALE) -> None:
    """bc_append_kv_paged: one K and V token per slot at logical position pos."""
    _check_half(k, "K")
    _check_half(v, "V")
    d = k.shape[-1]
    lib = _lib.load()
    _lib.check(lib.bc_append_kv_paged(k.data_ptr(), v.data_ptr(), K.c(), V.c(), pt.c(), pt.n_slots, d, pos,
                                      residual_mode, _stream(k)), "append_kv_paged")


def decode_attention_entropy(q: torch.Tensor, K: Planes, V: Planes, seq_len: int, mode: int = MODE_COMPENSATED,
                             out: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Decode attention and, from the same pass, the per-head entropy of the softmax
    over binary scores (the reference's compute_head_entropy).  Returns (out fp16
    [n_heads, d], entropy fp32 [n_heads])."""
    _check_half(q, "Q")
    d = q.shape[-1]
    n_heads = q.numel() // d
    n_slots = K.n_slots
    group = n_heads // n_slots
    if group * n_slots != n_heads:
        raise RuntimeError("number of query heads must be a multiple of the number of KV slots")
    if out is None:
        out = torch.empty((n_heads, d), dtype=torch.float16, device=q.device)
    ent = torch.empty(n_heads, dtype=torch.float32, device=q.device)
    lib = _lib.load()
    st = _stream(q)
    wsb = lib.bc_decode_workspace_bytes(n_slots, group, seq_len, d)
    ws = _lib.workspace(q.device, st, wsb, ("decode", n_slots, group))
    _lib.check(lib.bc_decode_attention_entropy(q.data_ptr(), K.c(), V.c(), out.data_ptr(), None, ent.data_ptr(),
                                               n_slots, group, seq_len, K.kv_stride, d, mode, _lib.ptr(ws),
                                               ws.numel() if ws is not None else 0, st),
               "decode_attention_entropy")
    return out, ent


def select_positions_topk(K: Planes, V: Planes, seq_len: int, n_keep: int) -> torch.Tensor:
    """Per-position adaptive precision: uint8 keep mask [n_slots, kv_stride] of the n_keep
    positions per slot with the largest K + V residual energy (bc_select_positions_topk)."""
    if not (K.compensated and V.compensated):
        raise RuntimeError("select_positions_topk needs compensated (residual) caches")
    lib = _lib.load()
    st = _lib.stream_of(K.sign.device)
    keep = torch.zeros((K.n_slots, K.kv_stride), dtype=torch.uint8, device=K.sign.device)
    wsb = lib.bc_select_workspace_bytes(K.n_slots, K.kv_stride)
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=K.sign.device)
    _lib.check(lib.bc_select_positions_topk(K.c(), V.c(), K.n_slots, seq_len, K.kv_stride, K.head_dim, n_keep,
                                            keep.data_ptr(), ws.data_ptr(), ws.numel(), st),
               "select_positions_topk")
    return keep


def compact_adaptive(K: Planes, V: Planes, keep: torch.Tensor, seq_len: int, n_keep: int) -> tuple[Planes, Planes]:
    """Compact adaptive cache (bc_compact_adaptive): kept positions first with their
    residuals, the rest binary only from row round8(n_keep); the residual planes hold
    only the kept rows.  Returns (Kc, Vc); their sign planes' stride is kv_stride of
    the result, the residual planes' stride nib.shape[1]."""
    b0 = round_stride(n_keep)
    c_stride = round_stride(b0 + seq_len - n_keep)
    r_stride = max(8, b0)

    def mk(P: Planes) -> Planes:
        dev = P.sign.device
        return Planes(torch.zeros((P.n_slots, c_stride, P.head_dim // 32), dtype=torch.int32, device=dev),
                      torch.zeros((P.n_slots, c_stride), dtype=torch.float16, device=dev),
                      torch.full((P.n_slots, r_stride, P.head_dim // 2), 0x88, dtype=torch.uint8, device=dev),
                      torch.zeros((P.n_slots, r_stride), dtype=torch.float16, device=dev), P.head_dim)

    Kc, Vc = mk(K), mk(V)
    lib = _lib.load()
    _lib.check(lib.bc_compact_adaptive(K.c(), V.c(), keep.data_ptr(), K.n_slots, seq_len, K.kv_stride, K.head_dim,
                                       n_keep, Kc.c(), Vc.c(), c_stride, r_stride,
                                       _lib.stream_of(K.sign.device)), "compact_adaptive")
    return Kc, Vc


def decode_attention_adaptive(q: torch.Tensor, Kc: Planes, Vc: Planes, seq_len: int, n_keep: int,
                              out: torch.Tensor | None = None) -> torch.Tensor:
    """Decode attention over a compact adaptive cache (bc_decode_attention_adaptive).
    q and out may be pinned host tensors: q is staged to the device first
    (device_query), and the kernel writes out over the host link itself."""
    if out is not None:
        _check_half_dev_or_pinned(out, "out")
    q = device_query(q, Kc.sign.device)
    d = q.shape[-1]
    n_heads = q.numel() // d
    n_slots = Kc.n_slots
    group = n_heads // n_slots
    if group * n_slots != n_heads:
        raise RuntimeError("number of query heads must be a multiple of the number of KV slots")
    if out is None:
        out = torch.empty((n_heads, d), dtype=torch.float16, device=q.device)
    elif out.numel() < n_heads * d:
        raise RuntimeError(f"out holds {out.numel()} elements, the call writes {n_heads * d}")
    lib = _lib.load()
    st = _stream(q)
    wsb = lib.bc_decode_adaptive_workspace_bytes(n_slots, group, seq_len, n_keep, d)
    ws = _lib.workspace(q.device, st, wsb, ("decode", n_slots, group))
    _lib.check(lib.bc_decode_attention_adaptive(q.data_ptr(), Kc.c(), Vc.c(), out.data_ptr(), None, n_slots, group,
                                                seq_len, n_keep, Kc.kv_stride, Kc.nib.shape[1], d, _lib.ptr(ws),
                                                ws.numel() if ws is not None else 0, st),
               "decode_attention_adaptive")
    return out


def keep_count(seq_len: int, fraction: float) -> int:
    """Number of residuals kept per slot for a keep fraction (rounded to nearest, ties up)."""
    return int(seq_len * fraction + 0.5)


def select_residual_topk(P: Planes, seq_len: int, n_keep: int, apply: bool = True,
                         want_mask: bool = False) -> torch.Tensor | None:
    """Per-vector adaptive precision on one plane cache: keep the residuals of the n_keep
    vectors per slot with the largest residual energy (see bc_select_residual_topk);
    with apply, zero the others in place.  Returns the uint8 keep mask when asked."""
    if not P.compensated:
        raise RuntimeError("select_residual_topk needs a compensated (residual) cache")
    lib = _lib.load()
    st = _lib.stream_of(P.sign.device)
    keep = torch.zeros((P.n_slots, P.kv_stride), dtype=torch.uint8, device=P.sign.device) if want_mask else None
    wsb = lib.bc_select_workspace_bytes(P.n_slots, P.kv_stride)
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=P.sign.device)
    _lib.check(lib.bc_select_residual_topk(P.c(), P.n_slots, seq_len, P.kv_stride, P.head_dim, n_keep,
                                           _lib.ptr(keep), 1 if apply else 0, ws.data_ptr(), ws.numel(), st),
               "select_residual_topk")
    return keep


def stage_rows(pairs: list[tuple[torch.Tensor, torch.Tensor]]) -> None:
    """bc_stage_rows: copy each (pinned host src, device dst) pair of equally sized,
    16-byte aligned contiguous tensors with one kernel on the current stream of
    the destinations' device.  The sources are read before the kernel waits for
    the previous one in the stream, so no GPU work queued earlier may write them."""
    if not 0 < len(pairs) <= 4:
        raise RuntimeError("stage_rows takes 1 to 4 segments")
    segs = (_lib.CopySeg * len(pairs))()
    for i, (src, dst) in enumerate(pairs):
        if src.nbytes != dst.nbytes or not src.is_contiguous() or not dst.is_contiguous():
            raise RuntimeError("stage_rows: segments must be contiguous and of equal size")
        segs[i].src, segs[i].dst, segs[i].bytes = src.data_ptr(), dst.data_ptr(), src.nbytes
    _lib.check(_lib.load().bc_stage_rows(segs, len(pairs), _lib.stream_of(pairs[0][1].device)), "stage_rows")


def lse_merge(parts: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Merge partial triples float32 [n_parts, n_heads, head_dim + 2] -> fp16 [n_heads, head_dim]."""
    n_parts, n_heads, dp2 = parts.shape
    d = dp2 - 2
    parts = parts.contiguous()
    if out is None:
        out = torch.empty((n_heads, d), dtype=torch.float16, device=parts.device)
    lib = _lib.load()
    _lib.check(lib.bc_lse_merge(parts.data_ptr(), n_parts, n_heads, d, out.data_ptr(), _stream(parts)), "lse_merge")
    return out


def xnor_popcount(q: torch.Tensor, K: Planes, seq_len: int) -> torch.Tensor:
    """Integer XNOR popcount of each query head against its slot's keys: int32 [n_heads, seq_len]."""
    _check_half(q, "Q")
    d = q.shape[-1]
    n_heads = q.numel() // d
    group = n_heads // K.n_slots
    out = torch.empty((n_heads, seq_len), dtype=torch.int32, device=q.device)
    lib = _lib.load()
    _lib.check(lib.bc_xnor_popcount(q.data_ptr(), K.sign.data_ptr(), out.data_ptr(), K.n_slots, group, seq_len,
                                    K.kv_stride, d, _stream(q)), "xnor_popcount")
    return out


def head_entropy(q: torch.Tensor, K: Planes, seq_len: int) -> torch.Tensor:
    """Entropy of the binary-score softmax per head (query head h reads slot h)."""
    _check_half(q, "Q")
    d = q.shape[-1]
    n_heads = q.numel() // d
    out = torch.empty((n_heads,), dtype=torch.float32, device=q.device)
    lib = _lib.load()
    _lib.check(lib.bc_head_entropy_planes(q.data_ptr(), K.c(), out.data_ptr(), n_heads, seq_len, K.kv_stride, d,
                                          _stream(q)), "head_entropy")
    return out


def records_to_planes(bin_blob: torch.Tensor, res_blob: torch.Tensor | None, n_vecs: int, head_dim: int) -> Planes:
    """Reference BinaryVec/ResidualVec blobs (n_vecs records) -> flat planes [1, n_vecs_padded]."""
    P = Planes.empty(1, round_stride(n_vecs), head_dim, res_blob is not None, bin_blob.device)
    lib = _lib.load()
    _lib.check(lib.bc_records_to_planes(bin_blob.data_ptr(), _lib.ptr(res_blob), P.c(), n_vecs, head_dim,
                                        _stream(bin_blob)), "records_to_planes")
    return P


def planes_to_records(P: Planes, n_vecs: int) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Flat planes (first n_vecs rows of slot-major storage) -> reference record blobs."""
    lib = _lib.load()
    b = torch.empty(n_vecs * lib.bc_sizeof_binary_vec(), dtype=torch.uint8, device=P.sign.device)
    r = None
    if P.compensated:
        r = torch.empty(n_vecs * lib.bc_sizeof_residual_vec(), dtype=torch.uint8, device=P.sign.device)
    _lib.check(lib.bc_planes_to_records(P.c(), b.data_ptr(), _lib.ptr(r), n_vecs, P.head_dim, _stream(b)),
               "planes_to_records")
    return b, r
