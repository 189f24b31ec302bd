"""The reference's own CUDA kernels (oracle/_ref/libbitcache_ref.so, compiled
from the reference sources by oracle/build.py) -- TEST INFRASTRUCTURE ONLY.

Used by the GPU parity tests and the golden-vector generator as the
bit-exactness checker.  The reference attention kernels have no
batch*n_heads guard (compensated_attention.cu:52), so every per-(batch, head)
buffer is padded here to a multiple of 32 rows with zeros (zero records score
0 and contribute 0, so the padding rows compute finite values in bounds).
"""
from __future__ import annotations

import ctypes
import os

import torch

from . import build

_lib = None
P = ctypes.c_void_p
I = ctypes.c_int


def available() -> bool:
    return os.path.exists(build.REF_SO)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not available():
            raise RuntimeError(f"reference kernels not built: {build.REF_SO}")
        L = ctypes.CDLL(build.REF_SO)
        for name, args in {
            "ref_binary_encode": [P, P, I, I, P],
            "ref_residual_encode": [P, P, P, I, I, P],
            "ref_binary_attention": [P, P, P, P, I, I, I, I, P],
            "ref_compensated_attention": [P, P, P, P, P, P, I, I, I, I, P],
            "ref_online_encode_token": [P, P, P, I, I, I, I, I, P],
            "ref_compute_head_entropy": [P, P, P, I, I, I, I, P],
            "ref_adaptive_select": [P, P, I, I, ctypes.c_float, P],
            "ref_reference_attention": [P, P, P, P, I, I, I, I, P],
        }.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = I
        L.ref_sizeof_binary_vec.restype = I
        L.ref_sizeof_residual_vec.restype = I
        _lib = L
    return _lib


def _st(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _ok(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"reference {what} failed with cudaError {rc}")


def binary_encode(src: torch.Tensor) -> torch.Tensor:
    n, d = src.shape
    out = torch.zeros(n * 36, dtype=torch.uint8, device=src.device)
    _ok(lib().ref_binary_encode(src.data_ptr(), out.data_ptr(), n, d, _st(src)), "binary_encode")
    return out


def residual_encode(src: torch.Tensor, blob: torch.Tensor) -> torch.Tensor:
    n, d = src.shape
    out = torch.zeros(n * 130, dtype=torch.uint8, device=src.device)
    _ok(lib().ref_residual_encode(src.data_ptr(), blob.data_ptr(), out.data_ptr(), n, d, _st(src)), "residual_encode")
    return out


def _pad_rows(n_rows: int) -> int:
    return (n_rows + 31) // 32 * 32


def _pad(t: torch.Tensor, rows: int, per_row: int) -> torch.Tensor:
    out = torch.zeros(rows * per_row, dtype=t.dtype, device=t.device)
    out[: t.numel()] = t.reshape(-1)
    return out


def attention(q: torch.Tensor, kb: torch.Tensor, vb: torch.Tensor, kr: torch.Tensor | None, vr: torch.Tensor | None,
              batch: int, n_heads: int, seq_len: int, head_dim: int) -> torch.Tensor:
    """Reference binary (kr is None) or compensated attention; q [batch*n_heads, d] fp16."""
    bh = batch * n_heads
    rows = _pad_rows(bh)
    qp = _pad(q.reshape(-1), rows, head_dim)
    out = torch.zeros(rows * head_dim, dtype=torch.float16, device=q.device)
    kbp, vbp = _pad(kb, rows, seq_len * 36), _pad(vb, rows, seq_len * 36)
    if kr is None:
        _ok(lib().ref_binary_attention(qp.data_ptr(), kbp.data_ptr(), vbp.data_ptr(), out.data_ptr(), 1, rows,
                                       seq_len, head_dim, _st(q)), "binary_attention")
    else:
        krp, vrp = _pad(kr, rows, seq_len * 130), _pad(vr, rows, seq_len * 130)
        _ok(lib().ref_compensated_attention(qp.data_ptr(), kbp.data_ptr(), krp.data_ptr(), vbp.data_ptr(),
                                            vrp.data_ptr(), out.data_ptr(), 1, rows, seq_len, head_dim, _st(q)),
            "compensated_attention")
    return out[: bh * head_dim].view(bh, head_dim)


def online_encode_token(kv: torch.Tensor, bin_cache: torch.Tensor, res_cache: torch.Tensor, batch: int,
                        n_heads: int, head_dim: int, current_len: int, max_seq: int) -> None:
    _ok(lib().ref_online_encode_token(kv.data_ptr(), bin_cache.data_ptr(), res_cache.data_ptr(), batch, n_heads,
                                      head_dim, current_len, max_seq, _st(kv)), "online_encode_token")


def head_entropy(q: torch.Tensor, kb: torch.Tensor, batch: int, n_heads: int, seq_len: int,
                 head_dim: int) -> torch.Tensor:
    out = torch.zeros(batch * n_heads, dtype=torch.float32, device=q.device)
    _ok(lib().ref_compute_head_entropy(q.data_ptr(), kb.data_ptr(), out.data_ptr(), batch, n_heads, seq_len,
                                       head_dim, _st(q)), "compute_head_entropy")
    return out


def adaptive_select(ent: torch.Tensor, thr: float) -> torch.Tensor:
    out = torch.zeros(ent.numel(), dtype=torch.uint8, device=ent.device)
    _ok(lib().ref_adaptive_select(ent.data_ptr(), out.data_ptr(), 1, ent.numel(), thr, _st(ent)), "adaptive_select")
    return out


def reference_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, batch: int, n_heads: int, seq_len: int,
                        head_dim: int) -> torch.Tensor:
    bh = batch * n_heads
    rows = _pad_rows(bh)
    qp = _pad(q.reshape(-1), rows, head_dim)
    kp = _pad(k.reshape(-1), rows, seq_len * head_dim)
    vp = _pad(v.reshape(-1), rows, seq_len * head_dim)
    out = torch.zeros(rows * head_dim, dtype=torch.float16, device=q.device)
    _ok(lib().ref_reference_attention(qp.data_ptr(), kp.data_ptr(), vp.data_ptr(), out.data_ptr(), 1, rows, seq_len,
                                      head_dim, _st(q)), "reference_attention")
    return out[: bh * head_dim].view(bh, head_dim)
