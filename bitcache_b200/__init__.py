"""bitcache_b200: B200-native (sm_100a) binary KV cache with XNOR-popcount
scoring and INT4 residual correction.

Drop-in for the reference package ``bitcache`` (anishesg/bitcache):
``BitCache``, ``functional`` and the ``_C`` operator set keep the reference's
names and argument meaning; the kernels behind them are this package's own
(libbitcache_b200.so, C ABI in include/bitcache_b200.h).
"""
from __future__ import annotations

import torch
from torch import Tensor

from . import _lib


def __getattr__(name: str):
    # _HAS_EXTENSION (reference bitcache/__init__.py:14-19) is evaluated on
    # first use: importing the package (e.g. for its workload generators) maps
    # no native code; every operator loads the library and fails loudly when
    # it is missing.
    if name == "_HAS_EXTENSION":
        return _lib.available()
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")


def _require_extension() -> None:
    """Raise when the native library is missing (reference bitcache/__init__.py:22-26)."""
    if not _lib.available():
        raise RuntimeError(
            "bitcache_b200 native library not found. Run: python -m bitcache_b200.build")


from . import planes as _planes  # noqa: E402


class BitCache:
    """Binary KV cache for one transformer layer (reference bitcache/__init__.py:29-207).

    Encodes each appended K/V token to sign bits + mean |x| scale and, when
    ``compensated``, an INT4 residual; ``attend`` runs the fused B200 decode
    kernel over the cached positions.  Storage is the native plane layout
    (5*head_dim/8 + 4 bytes per vector instead of the reference's 166-byte
    record pair).

    Ring buffer: once ``max_seq`` tokens are cached the oldest position is
    overwritten.  Attention is invariant to key order, so every cached
    position is attended in place; there is no wrap-around copy.

    Args match the reference; ``n_kv_heads`` (default ``n_heads``) enables
    grouped-query caches where query head h reads KV head h // (n_heads / n_kv_heads).
    ``append`` takes K, V of shape [batch, n_kv_heads, head_dim].
    """

    def __init__(self, batch: int, n_heads: int, head_dim: int, max_seq: int, device: str = "cuda",
                 compensated: bool = True, n_kv_heads: int | None = None) -> None:
        _require_extension()
        assert head_dim % 32 == 0, "head_dim must be a multiple of 32"
        assert head_dim <= 256, "head_dim must be <= 256"
        n_kv_heads = n_heads if n_kv_heads is None else n_kv_heads
        assert n_heads % n_kv_heads == 0, "n_heads must be a multiple of n_kv_heads"
        assert max_seq > 0, "max_seq must be positive"
        self.batch = batch
        self.n_heads = n_heads
        self.n_kv_heads = n_kv_heads
        self.head_dim = head_dim
        self.max_seq = max_seq
        self.device = torch.device(device)
        self.compensated = compensated
        self._kv_stride = _planes.round_stride(max_seq)
        n_slots = batch * n_kv_heads
        self._K = _planes.Planes.empty(n_slots, self._kv_stride, head_dim, compensated, self.device)
        self._V = _planes.Planes.empty(n_slots, self._kv_stride, head_dim, compensated, self.device)
        self._res_mode = _planes.RES_FP32_SCALE if compensated else _planes.RES_NONE
        self._write_pos = 0
        self._filled = 0
        self._n_slots = n_slots
        # the planes never move: their C descriptors are built once
        self._Kc, self._Vc = self._K.c(), self._V.c()
        self._stage: Tensor | None = None  # device copy of a step's pinned Q, K, V
        self._segs = None
        self._ws_bytes: dict[int, int] = {}

    def _staging(self, nq: int, nkv: int):
        """The device buffer a step's pinned Q, K, V are staged into, and the
        bc_copy_seg array of that copy (sources filled in per call)."""
        if self._stage is None:
            self._stage = torch.empty(nq + 2 * nkv, dtype=torch.float16, device=self._K.sign.device)
            base = self._stage.data_ptr()
            self._stage_ptrs = (base, base + 2 * nq, base + 2 * (nq + nkv))
            self._segs = (_lib.CopySeg * 3)()
            for i, (dst, n) in enumerate(zip(self._stage_ptrs, (nq, nkv, nkv))):
                self._segs[i].dst, self._segs[i].bytes = dst, 2 * n
        return self._segs, self._stage_ptrs

    def _step_workspace(self, seq_len: int, dev: torch.device, stream: int) -> tuple[int | None, int]:
        """Split-K workspace of a step over seq_len keys (sizes cached per length)."""
        nbytes = self._ws_bytes.get(seq_len)
        if nbytes is None:
            nbytes = _lib.load().bc_decode_workspace_bytes(self._n_slots, self.n_heads // self.n_kv_heads, seq_len,
                                                           self.head_dim)
            self._ws_bytes[seq_len] = nbytes
        ws = _lib.workspace(dev, stream, nbytes, ("decode", self._n_slots, self.n_heads // self.n_kv_heads))
        return (None, 0) if ws is None else (ws.data_ptr(), ws.numel())

    # -- core API ------------------------------------------------------------
    def append(self, K: Tensor, V: Tensor) -> None:
        """Encode one new K/V token per (batch, kv head) into the ring buffer
        (online_encode.cu arithmetic; K and V in one launch)."""
        self._validate_kv(K, V)
        _planes.append_kv(K, V, self._K, self._V, self._write_pos, self._res_mode)
        self._write_pos = (self._write_pos + 1) % self.max_seq
        self._filled = min(self._filled + 1, self.max_seq)

    def prefill(self, K: Tensor, V: Tensor) -> None:
        """Encode a whole prompt at once: K, V fp16 [batch, n_kv_heads, seq, head_dim], seq <= max_seq,
        starting at position 0 (replaces the cache contents).  Uses the same
        arithmetic as ``append`` (residual against the fp32 scale)."""
        assert K.shape == V.shape and K.dim() == 4, "K and V must be [batch, n_kv_heads, seq, head_dim]"
        b, h, s, d = K.shape
        assert (b, h, d) == (self.batch, self.n_kv_heads, self.head_dim), "shape mismatch"
        assert s <= self.max_seq, "prefill longer than max_seq"
        _planes.encode_planes(K.reshape(b * h, s, d).contiguous(), self._K, self._res_mode)
        _planes.encode_planes(V.reshape(b * h, s, d).contiguous(), self._V, self._res_mode)
        self._write_pos = s % self.max_seq
        self._filled = s

    def attend(self, Q: Tensor) -> Tensor:
        """Attention of Q [batch, n_heads, head_dim] fp16 over the cached positions."""
        assert self._filled > 0, "cache is empty, call append() first"
        assert Q.shape == (self.batch, self.n_heads, self.head_dim), "Q shape mismatch"
        assert Q.dtype == torch.float16 and Q.is_cuda and Q.is_contiguous(), "Q must be contiguous fp16 CUDA"
        mode = _planes.MODE_COMPENSATED if self.compensated else _planes.MODE_BINARY
        out = _planes.decode_attention(Q.view(-1, self.head_dim), self._K, self._V, self._filled, mode)
        return out.view(self.batch, self.n_heads, self.head_dim)

    def step(self, Q: Tensor, K: Tensor, V: Tensor, out: Tensor | None = None) -> Tensor:
        """One decode step in one launch: ``append(K, V)`` followed by ``attend(Q)``
        (reference bitcache/__init__.py:95-148), with identical results and cache
        contents.  The new token is encoded inside the attention kernel and
        attended from the encoder's output.

        Q, K, V (and ``out``) may also be pinned host tensors.  The inputs then
        cross the host link once, staged into a device buffer by a small kernel
        launched ahead of the step (bc_stage_rows), instead of once per split
        CTA; the step kernel writes the output over the host link itself.  A
        host loop that rewrites the pinned inputs synchronises on the previous
        step first (it reads that step's output anyway)."""
        pinned = not Q.is_cuda
        kv_shape = (self.batch, self.n_kv_heads, self.head_dim)
        for t, name, shape in ((K, "K", kv_shape), (V, "V", kv_shape),
                               (Q, "Q", (self.batch, self.n_heads, self.head_dim))):
            assert t.shape == shape, f"{name} shape {tuple(t.shape)} != {shape}"
            assert t.dtype == torch.float16, f"{name} must be float16"
            assert t.is_contiguous(), f"{name} must be contiguous"
            assert (t.is_pinned() if pinned else t.is_cuda), f"{name}: all of Q, K, V on CUDA, or all pinned host"
        if out is None:
            out = (torch.empty(Q.shape, dtype=torch.float16).pin_memory() if pinned
                   else torch.empty(Q.shape, dtype=torch.float16, device=self.device))
        else:
            assert out.shape == Q.shape and out.dtype == torch.float16 and out.is_contiguous(), "out mismatch"
            assert out.is_cuda or out.is_pinned(), "out must be a CUDA tensor or pinned host memory"
        pos = self._write_pos
        filled = min(self._filled + 1, self.max_seq)
        lib = _lib.load()
        dev = self._K.sign.device
        st = _lib.stream_of(dev)
        qp, kp, vp = Q.data_ptr(), K.data_ptr(), V.data_ptr()
        if pinned and (qp | kp | vp) % 16 == 0:
            # one host-link crossing per step: stage Q, K, V on the device first
            segs, dev_ptrs = self._staging(Q.numel(), K.numel())
            segs[0].src, segs[1].src, segs[2].src = qp, kp, vp
            _lib.check(lib.bc_stage_rows(segs, 3, st), "stage_rows")
            qp, kp, vp = dev_ptrs
        ws, wsb = self._step_workspace(filled, dev, st)
        mode = _lib.BC_MODE_COMPENSATED if self.compensated else _lib.BC_MODE_BINARY
        _lib.check(lib.bc_decode_step(qp, kp, vp, self._Kc, self._Vc, out.data_ptr(), None, self._n_slots,
                                      self.n_heads // self.n_kv_heads, filled, self._kv_stride, self.head_dim, mode,
                                      pos, self._res_mode, ws, wsb, st), "decode_step")
        res = out
        self._write_pos = (pos + 1) % self.max_seq
        self._filled = filled
        return res.view(self.batch, self.n_heads, self.head_dim)

    def keep_residuals(self, fraction: float = 0.25) -> None:
        """Per-vector adaptive precision: keep the INT4 residual only for the given fraction
        of cached vectors (per K/V, per slot) with the largest residual energy; the rest
        become binary-only.  Applies to the positions cached so far."""
        assert self.compensated, "keep_residuals needs a compensated cache"
        n_keep = _planes.keep_count(self._filled, fraction)
        for P in (self._K, self._V):
            _planes.select_residual_topk(P, self._filled, n_keep, apply=True)

    def reset(self) -> None:
        """Clear the cache and the ring pointers."""
        self._K.zero_()
        self._V.zero_()
        self._write_pos = 0
        self._filled = 0

    # -- properties ----------------------------------------------------------
    @property
    def seq_len(self) -> int:
        return self._filled

    @property
    def memory_bytes(self) -> int:
        """Device bytes held by the K and V planes."""
        return self._K.nbytes() + self._V.nbytes()

    @property
    def compression_ratio(self) -> float:
        """fp16 KV bytes over binary (sign + scale) bytes, as in the reference
        (__init__.py:177-185) but with this layout's d/8 + 2 bytes per vector."""
        fp16 = 2 * self.batch * self.n_kv_heads * self.max_seq * self.head_dim * 2
        binary = 2 * self.batch * self.n_kv_heads * self.max_seq * _planes.vector_bytes(self.head_dim, False)
        return fp16 / binary

    @property
    def planes(self) -> tuple[_planes.Planes, _planes.Planes]:
        return self._K, self._V

    def _validate_kv(self, K: Tensor, V: Tensor) -> None:
        expected = (self.batch, self.n_kv_heads, self.head_dim)
        assert K.shape == torch.Size(expected), f"K shape {tuple(K.shape)} != {expected}"
        assert V.shape == torch.Size(expected), f"V shape {tuple(V.shape)} != {expected}"
        assert K.dtype == torch.float16, "K must be float16"
        assert V.dtype == torch.float16, "V must be float16"
        assert K.is_cuda and V.is_cuda, "K and V must be on CUDA"
        assert K.is_contiguous() and V.is_contiguous(), "K and V must be contiguous"

    def __repr__(self) -> str:
        mode = "compensated" if self.compensated else "binary"
        return (f"BitCache(batch={self.batch}, n_heads={self.n_heads}, n_kv_heads={self.n_kv_heads}, "
                f"head_dim={self.head_dim}, max_seq={self.max_seq}, filled={self._filled}, mode={mode}, "
                f"mem={self.memory_bytes / 1024:.1f}KB)")


from . import functional  # noqa: E402,F401
from . import _C  # noqa: E402,F401

__all__ = ["BitCache", "functional", "_C", "_require_extension"]
