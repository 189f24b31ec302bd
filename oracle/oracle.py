"""numpy front end of the C oracle (bitcache_oracle.c) -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module.  fp16 data is passed as uint16 bit patterns; encodings come back
as separate field arrays (sign words, binary scale, nibbles, residual scale),
whose values equal the reference BinaryVec / ResidualVec fields.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import build

_lib = None

P = ctypes.c_void_p
I64 = ctypes.c_int64
I32 = ctypes.c_int


class _Planes(ctypes.Structure):
    _fields_ = [("words", P), ("bscale", P), ("nib", P), ("rscale", P)]


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = build.build_oracle()
        L = ctypes.CDLL(path)
        L.orc_h2f.restype = ctypes.c_float
        L.orc_h2f.argtypes = [ctypes.c_uint16]
        L.orc_f2h.restype = ctypes.c_uint16
        L.orc_f2h.argtypes = [ctypes.c_float]
        L.orc_binary_encode.argtypes = [P, I64, I32, P, P]
        L.orc_residual_encode.argtypes = [P, P, P, I64, I32, P, P, P]
        L.orc_online_encode.argtypes = [P, I64, I32, P, P, P, P, P]
        L.orc_xnor_popcount.argtypes = [P, P, I64, I32, P]
        L.orc_attention.argtypes = [P, ctypes.POINTER(_Planes), ctypes.POINTER(_Planes), I64, I32, I32, I64, I32,
                                    I32, P, I32]
        L.orc_reference_attention.argtypes = [P, P, P, I64, I32, I32, P]
        L.orc_head_entropy.argtypes = [P, P, P, I64, I32, I64, I32, P]
        L.orc_adaptive_select.argtypes = [P, I64, ctypes.c_float, P]
        L.orc_select_residual_topk.argtypes = [P, P, I64, I32, I64, I32, I32, P]
        L.orc_lse_merge.argtypes = [P, I32, I64, I32, P]
        L.orc_num_threads.restype = I32
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(P)


def _u16(a: np.ndarray) -> np.ndarray:
    if a.dtype == np.float16:
        a = a.view(np.uint16)
    return np.ascontiguousarray(a, dtype=np.uint16)


def num_threads() -> int:
    return int(lib().orc_num_threads())


def binary_encode(src: np.ndarray):
    """src fp16/uint16 [n, d] -> (words uint32 [n, d/32], bscale uint16 [n])."""
    s = _u16(src)
    n, d = s.shape
    words = np.zeros((n, d // 32), np.uint32)
    sc = np.zeros(n, np.uint16)
    lib().orc_binary_encode(_p(s), n, d, _p(words), _p(sc))
    return words, sc


def residual_encode(src: np.ndarray, words: np.ndarray, bscale: np.ndarray):
    """residual.cu semantics -> (nib uint8 [n, d/2], rscale uint16 [n], pre float32 [n, d])."""
    s = _u16(src)
    n, d = s.shape
    nib = np.zeros((n, d // 2), np.uint8)
    rs = np.zeros(n, np.uint16)
    pre = np.zeros((n, d), np.float32)
    lib().orc_residual_encode(_p(s), _p(np.ascontiguousarray(words, np.uint32)),
                              _p(np.ascontiguousarray(bscale, np.uint16)), n, d, _p(nib), _p(rs), _p(pre))
    return nib, rs, pre


def online_encode(src: np.ndarray):
    """online_encode.cu semantics -> (words, bscale, nib, rscale, pre)."""
    s = _u16(src)
    n, d = s.shape
    words = np.zeros((n, d // 32), np.uint32)
    bs = np.zeros(n, np.uint16)
    nib = np.zeros((n, d // 2), np.uint8)
    rs = np.zeros(n, np.uint16)
    pre = np.zeros((n, d), np.float32)
    lib().orc_online_encode(_p(s), n, d, _p(words), _p(bs), _p(nib), _p(rs), _p(pre))
    return words, bs, nib, rs, pre


def xnor_popcount(q: np.ndarray, kwords: np.ndarray) -> np.ndarray:
    qq = _u16(q).reshape(-1)
    kw = np.ascontiguousarray(kwords, np.uint32)
    n = kw.shape[0]
    out = np.zeros(n, np.int32)
    lib().orc_xnor_popcount(_p(qq), _p(kw), n, qq.shape[0], _p(out))
    return out


def attention(q: np.ndarray, K: dict, V: dict, group: int, seq_len: int, kv_stride: int, compensated: bool,
              nthreads: int = 0) -> np.ndarray:
    """Reference two-pass decode attention. q [n_q, d]; K/V dicts of plane arrays
    words [slots, kv_stride, d/32], bscale [slots, kv_stride], nib, rscale. Returns fp16 bits [n_q, d]."""
    qq = _u16(q)
    n_q, d = qq.shape
    keep = []

    def mk(X):
        arrs = [np.ascontiguousarray(X["words"], np.uint32), np.ascontiguousarray(X["bscale"], np.uint16),
                None if X.get("nib") is None else np.ascontiguousarray(X["nib"], np.uint8),
                None if X.get("rscale") is None else np.ascontiguousarray(X["rscale"], np.uint16)]
        keep.append(arrs)
        return _Planes(_p(arrs[0]), _p(arrs[1]), _p(arrs[2]), _p(arrs[3]))

    kp, vp = mk(K), mk(V)
    out = np.zeros((n_q, d), np.uint16)
    lib().orc_attention(_p(qq), ctypes.byref(kp), ctypes.byref(vp), n_q, group, seq_len, kv_stride, d,
                        1 if compensated else 0, _p(out), nthreads)
    return out


def reference_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray) -> np.ndarray:
    """Exact fp32-accumulated attention from fp16 K/V [n_q, S, d] (reference_attention.cu)."""
    qq, kk, vv = _u16(q), _u16(k), _u16(v)
    n_q, s, d = kk.shape
    out = np.zeros((n_q, d), np.uint16)
    lib().orc_reference_attention(_p(qq), _p(kk), _p(vv), n_q, s, d, _p(out))
    return out


def head_entropy(q: np.ndarray, kwords: np.ndarray, kscale: np.ndarray, seq_len: int, kv_stride: int) -> np.ndarray:
    qq = _u16(q)
    n_q, d = qq.shape
    out = np.zeros(n_q, np.float32)
    lib().orc_head_entropy(_p(qq), _p(np.ascontiguousarray(kwords, np.uint32)),
                           _p(np.ascontiguousarray(kscale, np.uint16)), n_q, seq_len, kv_stride, d, _p(out))
    return out


def adaptive_select(entropy: np.ndarray, thr: float) -> np.ndarray:
    e = np.ascontiguousarray(entropy, np.float32)
    out = np.zeros(e.shape, np.uint8)
    lib().orc_adaptive_select(_p(e), e.size, thr, _p(out))
    return out


def select_residual_topk(nib: np.ndarray, rscale: np.ndarray, seq_len: int, n_keep: int) -> np.ndarray:
    """nib [slots, kv_stride, d/2], rscale [slots, kv_stride] -> keep uint8 [slots, kv_stride]."""
    nb = np.ascontiguousarray(nib, np.uint8)
    rs = np.ascontiguousarray(rscale, np.uint16)
    slots, stride, half_d = nb.shape
    keep = np.zeros((slots, stride), np.uint8)
    lib().orc_select_residual_topk(_p(nb), _p(rs), slots, seq_len, stride, 2 * half_d, n_keep, _p(keep))
    return keep


def residual_keys(nib_rows: np.ndarray, rscale: np.ndarray) -> np.ndarray:
    """Per-vector selection key fp32(rs*rs) * float(sum code^2) (the key of
    orc_select_residual_topk), from reference-format nibble rows [.., d/2] and fp16 bits."""
    lo = (nib_rows & 0x0F).astype(np.int64)
    hi = (nib_rows >> 4).astype(np.int64)
    lo = np.where(lo >= 8, lo - 16, lo)
    hi = np.where(hi >= 8, hi - 16, hi)
    ss = (lo * lo + hi * hi).sum(-1)
    rs = rscale.view(np.float16).astype(np.float32)
    return ((rs * rs).astype(np.float32) * ss.astype(np.float32)).astype(np.float32)


def select_positions_topk(k_nib: np.ndarray, k_rs: np.ndarray, v_nib: np.ndarray, v_rs: np.ndarray, seq_len: int,
                          n_keep: int) -> np.ndarray:
    """Joint per-position selection (the rule of bc_select_positions_topk): key =
    fp32(key_K + key_V); the n_keep largest per slot, ties to the lower position.
    Returns keep uint8 [slots, seq_len]."""
    key = (residual_keys(k_nib[:, :seq_len], k_rs[:, :seq_len]) +
           residual_keys(v_nib[:, :seq_len], v_rs[:, :seq_len])).astype(np.float32)
    keep = np.zeros(key.shape, np.uint8)
    for j in range(key.shape[0]):
        order = np.lexsort((np.arange(seq_len), -key[j].astype(np.float64)))
        keep[j, order[:n_keep]] = 1
    return keep


def lse_merge(parts: np.ndarray) -> np.ndarray:
    """parts float32 [n_parts, n_heads, d+2] -> float32 [n_heads, d]."""
    pp = np.ascontiguousarray(parts, np.float32)
    n_parts, n_heads, dp2 = pp.shape
    out = np.zeros((n_heads, dp2 - 2), np.float32)
    lib().orc_lse_merge(_p(pp), n_parts, n_heads, dp2 - 2, _p(out))
    return out


def f2h(x: np.ndarray) -> np.ndarray:
    """float32 -> fp16 bits, the oracle's RN-even converter (checked against numpy in tests)."""
    f = np.ascontiguousarray(x, np.float32).reshape(-1)
    L = lib()
    return np.array([L.orc_f2h(float(v)) for v in f], np.uint16).reshape(np.shape(x))


# Reference record views (BinaryVec 36 B, ResidualVec 130 B).
BINVEC = np.dtype([("words", "<u4", (8,)), ("scale", "<u2"), ("pad", "<u2")])
RESVEC = np.dtype([("nib", "u1", (128,)), ("scale", "<u2")])
assert BINVEC.itemsize == 36 and RESVEC.itemsize == 130


def split_binvec(blob: np.ndarray, d: int):
    r = np.frombuffer(np.ascontiguousarray(blob, np.uint8).tobytes(), BINVEC)
    return r["words"][:, : d // 32].copy(), r["scale"].copy()


def split_resvec(blob: np.ndarray, d: int):
    r = np.frombuffer(np.ascontiguousarray(blob, np.uint8).tobytes(), RESVEC)
    return r["nib"][:, : d // 2].copy(), r["scale"].copy()


def make_binvec(words: np.ndarray, scale: np.ndarray) -> np.ndarray:
    n, nw = words.shape
    r = np.zeros(n, BINVEC)
    r["words"][:, :nw] = words
    r["scale"] = scale
    return r.view(np.uint8).reshape(-1)


def make_resvec(nib: np.ndarray, scale: np.ndarray) -> np.ndarray:
    n, hd = nib.shape
    r = np.zeros(n, RESVEC)
    r["nib"][:, :hd] = nib
    r["scale"] = scale
    return r.view(np.uint8).reshape(-1)


def oracle_path() -> str:
    return os.path.abspath(build.ORACLE_SO)
