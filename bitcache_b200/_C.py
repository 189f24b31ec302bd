"""Operator mirror of the reference's ``bitcache._C`` torch binding
(src/torch_binding.cpp:17-177): same op names, argument order, output
allocation and validation, dispatching to the B200 kernels through the C ABI.

Blobs are opaque uint8 tensors of n * sizeof(BinaryVec) / n * sizeof(ResidualVec)
bytes holding the reference's record structs, byte for byte.

Deliberate differences (invalid input only): the attention ops check blob
sizes (the reference reads out of bounds on short blobs) and guard
batch*n_heads (the reference kernels write past the output when it is not a
multiple of 32).
"""
from __future__ import annotations

import torch

from . import _lib


def _check_input(x: torch.Tensor, name: str) -> None:
    # CHECK_INPUT, torch_binding.cpp:9-12
    if not x.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if not x.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")
    if x.dtype != torch.float16:
        raise RuntimeError(f"{name} must be float16")


def _check_blob(x: torch.Tensor, name: str) -> None:
    if not x.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if not x.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def _check_head_dim(head_dim: int) -> None:
    if head_dim % 32 != 0:
        raise RuntimeError("head_dim must be a multiple of 32")
    if head_dim > 256:
        raise RuntimeError("head_dim exceeds MAX_HEAD_DIM=256")


def _stream(t: torch.Tensor) -> int:
    return _lib.stream_of(t.device)


def sizeof_binary_vec() -> int:
    return int(_lib.load().bc_sizeof_binary_vec())


def sizeof_residual_vec() -> int:
    return int(_lib.load().bc_sizeof_residual_vec())


def binary_encode(src: torch.Tensor) -> torch.Tensor:
    """torch_binding.cpp:17-37: fp16 [n_vecs, head_dim] -> uint8 [n_vecs * sizeof(BinaryVec)]."""
    _check_input(src, "src")
    if src.dim() != 2:
        raise RuntimeError("src must be 2D [n_vecs, head_dim]")
    n, d = src.shape
    _check_head_dim(d)
    out = torch.empty(n * sizeof_binary_vec(), dtype=torch.uint8, device=src.device)
    _lib.check(_lib.load().bc_binary_encode(src.data_ptr(), out.data_ptr(), n, d, _stream(src)), "binary_encode")
    return out


def residual_encode(src: torch.Tensor, binary_blob: torch.Tensor) -> torch.Tensor:
    """torch_binding.cpp:40-65: fp16 + BinaryVec blob -> uint8 [n_vecs * sizeof(ResidualVec)]."""
    _check_input(src, "src")
    _check_blob(binary_blob, "binary_blob")
    n, d = src.shape
    _check_head_dim(d)
    if binary_blob.numel() != n * sizeof_binary_vec():
        raise RuntimeError("binary_blob size mismatch")
    out = torch.empty(n * sizeof_residual_vec(), dtype=torch.uint8, device=src.device)
    _lib.check(_lib.load().bc_residual_encode(src.data_ptr(), binary_blob.data_ptr(), out.data_ptr(), n, d,
                                              _stream(src)), "residual_encode")
    return out


def _check_records(blob: torch.Tensor, name: str, n: int, rec: int) -> None:
    _check_blob(blob, name)
    if blob.numel() < n * rec:
        raise RuntimeError(f"{name} holds {blob.numel()} bytes, needs {n * rec}")


def binary_attention(Q: torch.Tensor, K_bin: torch.Tensor, V_bin: torch.Tensor, batch: int, n_heads: int,
                     seq_len: int, head_dim: int) -> torch.Tensor:
    """torch_binding.cpp:68-89."""
    _check_input(Q, "Q")
    n = batch * n_heads * seq_len
    _check_records(K_bin, "K_bin", n, sizeof_binary_vec())
    _check_records(V_bin, "V_bin", n, sizeof_binary_vec())
    out = torch.empty_like(Q)
    lib = _lib.load()
    st = _stream(Q)
    ws = _lib.workspace(Q.device, st, lib.bc_attention_workspace_bytes(batch, n_heads, seq_len, head_dim),
                        ("records", batch * n_heads))
    _lib.check(lib.bc_binary_attention(Q.data_ptr(), K_bin.data_ptr(), V_bin.data_ptr(), out.data_ptr(), batch,
                                       n_heads, seq_len, head_dim, _lib.ptr(ws),
                                       ws.numel() if ws is not None else 0, st), "binary_attention")
    return out


def compensated_attention(Q: torch.Tensor, K_bin: torch.Tensor, K_res: torch.Tensor, V_bin: torch.Tensor,
                          V_res: torch.Tensor, batch: int, n_heads: int, seq_len: int,
                          head_dim: int) -> torch.Tensor:
    """torch_binding.cpp:92-117."""
    _check_input(Q, "Q")
    n = batch * n_heads * seq_len
    _check_records(K_bin, "K_bin", n, sizeof_binary_vec())
    _check_records(V_bin, "V_bin", n, sizeof_binary_vec())
    _check_records(K_res, "K_res", n, sizeof_residual_vec())
    _check_records(V_res, "V_res", n, sizeof_residual_vec())
    out = torch.empty_like(Q)
    lib = _lib.load()
    st = _stream(Q)
    ws = _lib.workspace(Q.device, st, lib.bc_attention_workspace_bytes(batch, n_heads, seq_len, head_dim),
                        ("records", batch * n_heads))
    _lib.check(lib.bc_compensated_attention(Q.data_ptr(), K_bin.data_ptr(), K_res.data_ptr(), V_bin.data_ptr(),
                                            V_res.data_ptr(), out.data_ptr(), batch, n_heads, seq_len, head_dim,
                                            _lib.ptr(ws), ws.numel() if ws is not None else 0, st),
               "compensated_attention")
    return out


def online_encode_token(kv: torch.Tensor, binary_cache: torch.Tensor, residual_cache: torch.Tensor | None,
                        batch: int, n_heads: int, head_dim: int, current_len: int, max_seq: int) -> None:
    """torch_binding.cpp:121-138 (in place).  residual_cache may be None for a binary-only cache."""
    _check_input(kv, "kv")
    _check_records(binary_cache, "binary_cache", batch * n_heads * max_seq, sizeof_binary_vec())
    if residual_cache is not None:
        _check_records(residual_cache, "residual_cache", batch * n_heads * max_seq, sizeof_residual_vec())
    _lib.check(_lib.load().bc_online_encode_token(kv.data_ptr(), binary_cache.data_ptr(), _lib.ptr(residual_cache),
                                                  batch, n_heads, head_dim, current_len, max_seq, _stream(kv)),
               "online_encode_token")


def compute_head_entropy(Q: torch.Tensor, K_bin: torch.Tensor, batch: int, n_heads: int, seq_len: int,
                         head_dim: int) -> torch.Tensor:
    """torch_binding.cpp:141-162: float32 [batch, n_heads]."""
    _check_input(Q, "Q")
    _check_records(K_bin, "K_bin", batch * n_heads * seq_len, sizeof_binary_vec())
    ent = torch.empty((batch, n_heads), dtype=torch.float32, device=Q.device)
    lib = _lib.load()
    st = _stream(Q)
    ws = _lib.workspace(Q.device, st, lib.bc_entropy_workspace_bytes(batch, n_heads, seq_len), ("entropy",))
    _lib.check(lib.bc_compute_head_entropy(Q.data_ptr(), K_bin.data_ptr(), ent.data_ptr(), batch, n_heads, seq_len,
                                           head_dim, _lib.ptr(ws), ws.numel() if ws is not None else 0, st),
               "compute_head_entropy")
    return ent


def adaptive_select(entropy: torch.Tensor, threshold: float) -> torch.Tensor:
    """launch_adaptive_select (adaptive_precision.cuh:42-49), which the reference binding does not
    expose: uint8 modes, 0 = BINARY where entropy >= threshold, else 1 = COMPENSATED."""
    if not entropy.is_cuda or entropy.dtype != torch.float32 or not entropy.is_contiguous():
        raise RuntimeError("entropy must be a contiguous float32 CUDA tensor")
    modes = torch.empty(entropy.shape, dtype=torch.uint8, device=entropy.device)
    n = entropy.numel()
    _lib.check(_lib.load().bc_adaptive_select(entropy.data_ptr(), modes.data_ptr(), 1, n, float(threshold),
                                              _stream(entropy)), "adaptive_select")
    return modes


__all__ = ["sizeof_binary_vec", "sizeof_residual_vec", "binary_encode", "residual_encode", "binary_attention",
           "compensated_attention", "online_encode_token", "compute_head_entropy", "adaptive_select"]
