"""Functional API, mirroring the reference's ``bitcache.functional``
(bitcache/functional.py:17-139): the same entry points, argument meaning and
assertion behaviour, over the B200 kernels.  Blobs hold the reference's
BinaryVec / ResidualVec records byte for byte.
"""
from __future__ import annotations

import torch
from torch import Tensor

from . import _C, _require_extension


def encode(src: Tensor) -> Tensor:
    """Binary-encode fp16 vectors [n_vecs, head_dim] -> BinaryVec blob (functional.py:17-35)."""
    _require_extension()
    assert src.is_cuda, "src must be on CUDA"
    assert src.is_contiguous(), "src must be contiguous"
    assert src.dtype == torch.float16, "src must be float16"
    assert src.dim() == 2, "src must be 2D [n_vecs, head_dim]"
    return _C.binary_encode(src)


def compute_residual(src: Tensor, binary_blob: Tensor) -> Tensor:
    """INT4 residual against the binary reconstruction -> ResidualVec blob (functional.py:38-56)."""
    _require_extension()
    assert src.is_cuda and binary_blob.is_cuda, "tensors must be on CUDA"
    assert src.is_contiguous() and binary_blob.is_contiguous(), "tensors must be contiguous"
    assert src.dtype == torch.float16, "src must be float16"
    return _C.residual_encode(src, binary_blob)


def binary_attention(Q: Tensor, K_bin: Tensor, V_bin: Tensor, batch: int, n_heads: int, seq_len: int,
                     head_dim: int) -> Tensor:
    """Binary-only attention (functional.py:59-88): Q [batch, n_heads, head_dim] fp16."""
    _require_extension()
    assert Q.is_cuda, "Q must be on CUDA"
    assert Q.is_contiguous(), "Q must be contiguous"
    assert Q.dtype == torch.float16, "Q must be float16"
    return _C.binary_attention(Q, K_bin, V_bin, batch, n_heads, seq_len, head_dim)


def compensated_attention(Q: Tensor, K_bin: Tensor, K_res: Tensor, V_bin: Tensor, V_res: Tensor, batch: int,
                          n_heads: int, seq_len: int, head_dim: int) -> Tensor:
    """Residual-compensated attention (functional.py:91-127)."""
    _require_extension()
    assert Q.is_cuda, "Q must be on CUDA"
    assert Q.is_contiguous(), "Q must be contiguous"
    assert Q.dtype == torch.float16, "Q must be float16"
    return _C.compensated_attention(Q, K_bin, K_res, V_bin, V_res, batch, n_heads, seq_len, head_dim)


def sizeof_binary_vec() -> int:
    """Size in bytes of one BinaryVec record (functional.py:130-133): 36."""
    _require_extension()
    return _C.sizeof_binary_vec()


def sizeof_residual_vec() -> int:
    """Size in bytes of one ResidualVec record (functional.py:136-139): 130."""
    _require_extension()
    return _C.sizeof_residual_vec()


__all__ = ["encode", "compute_residual", "binary_attention", "compensated_attention", "sizeof_binary_vec",
           "sizeof_residual_vec"]
