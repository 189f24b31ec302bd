"""ctypes binding to libbitcache_b200.so (the C ABI in include/bitcache_b200.h).

The shared library is built in-tree (``python -m bitcache_b200.build``) and
loaded from this package directory.  There is no fallback: if the library is
missing or a call fails, a RuntimeError is raised.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
# The in-tree build; BITCACHE_B200_LIB may name another build of the same library.
LIB_PATH = os.environ.get("BITCACHE_B200_LIB") or os.path.join(HERE, "libbitcache_b200.so")

BC_OK = 0
BC_ERR_WORKSPACE = 4
BC_RES_NONE, BC_RES_FP16_SCALE, BC_RES_FP32_SCALE = 0, 1, 2
BC_MODE_BINARY, BC_MODE_COMPENSATED = 0, 1
BC_DEVERR_TIMEOUT = 1
BC_DEVERR_PAGE = 2

c_void_p = ctypes.c_void_p
c_int = ctypes.c_int
c_int64 = ctypes.c_int64
c_size_t = ctypes.c_size_t
c_float = ctypes.c_float


class KVPlanes(ctypes.Structure):
    """bc_kv_planes: sign, nib, bscale, rscale device pointers."""

    _fields_ = [("sign", c_void_p), ("nib", c_void_p), ("bscale", c_void_p), ("rscale", c_void_p)]


class PageTable(ctypes.Structure):
    """bc_page_table: block table pointer and paging geometry."""

    _fields_ = [("pages", c_void_p), ("max_pages", ctypes.c_int32), ("page_size", ctypes.c_int32),
                ("n_pages", ctypes.c_int32)]


class CopySeg(ctypes.Structure):
    """bc_copy_seg: one host -> device segment of bc_stage_rows."""

    _fields_ = [("src", c_void_p), ("dst", c_void_p), ("bytes", ctypes.c_uint64)]


class Xchg(ctypes.Structure):
    """bc_xchg: every rank's exchange buffer as mapped here, world, rank, epoch, the
    poll limit of one exchange word (0: the library default) and the buffers' size."""

    _fields_ = [("bufs", c_void_p * 8), ("world", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("epoch", ctypes.c_uint32), ("spin_limit", ctypes.c_uint32), ("buf_bytes", ctypes.c_uint64)]


_SIGS = {
    "bc_status_string": (ctypes.c_char_p, [c_int]),
    "bc_get_device_error": (ctypes.c_uint, [c_int]),
    "bc_sizeof_binary_vec": (c_int64, []),
    "bc_sizeof_residual_vec": (c_int64, []),
    "bc_binary_encode": (c_int, [c_void_p, c_void_p, c_int64, c_int, c_void_p]),
    "bc_residual_encode": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_void_p]),
    "bc_online_encode_token": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p]),
    "bc_attention_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "bc_binary_attention": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                    c_void_p, c_size_t, c_void_p]),
    "bc_compensated_attention": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                         c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "bc_entropy_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "bc_compute_head_entropy": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_size_t,
                                        c_void_p]),
    "bc_head_entropy_planes": (c_int, [c_void_p, KVPlanes, c_void_p, c_int, c_int, c_int64, c_int, c_void_p]),
    "bc_adaptive_select": (c_int, [c_void_p, c_void_p, c_int, c_int, c_float, c_void_p]),
    "bc_encode_planes": (c_int, [c_void_p, KVPlanes, c_int, c_int, c_int64, c_int, c_int, c_void_p]),
    "bc_append_kv": (c_int, [c_void_p, c_void_p, KVPlanes, KVPlanes, c_int, c_int, c_int64, c_int64, c_int,
                             c_void_p]),
    "bc_decode_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "bc_decode_attention": (c_int, [c_void_p, KVPlanes, KVPlanes, c_void_p, c_void_p, c_int, c_int, c_int, c_int64,
                                    c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "bc_decode_step": (c_int, [c_void_p, c_void_p, c_void_p, KVPlanes, KVPlanes, c_void_p, c_void_p, c_int, c_int,
                               c_int, c_int64, c_int, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "bc_decode_attention_entropy": (c_int, [c_void_p, KVPlanes, KVPlanes, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                            c_int, c_int64, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "bc_select_positions_topk": (c_int, [KVPlanes, KVPlanes, c_int, c_int, c_int64, c_int, c_int, c_void_p,
                                         c_void_p, c_size_t, c_void_p]),
    "bc_compact_adaptive": (c_int, [KVPlanes, KVPlanes, c_void_p, c_int, c_int, c_int64, c_int, c_int, KVPlanes,
                                    KVPlanes, c_int64, c_int64, c_void_p]),
    "bc_decode_adaptive_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int]),
    "bc_decode_attention_adaptive": (c_int, [c_void_p, KVPlanes, KVPlanes, c_void_p, c_void_p, c_int, c_int, c_int,
                                             c_int, c_int64, c_int64, c_int, c_void_p, c_size_t, c_void_p]),
    "bc_xchg_bytes": (c_size_t, [c_int, c_int, c_int]),
    "bc_xchg_alloc": (c_int, [c_size_t, ctypes.POINTER(c_void_p)]),
    "bc_xchg_free": (c_int, [c_void_p]),
    "bc_ipc_handle": (c_int, [c_void_p, c_void_p]),
    "bc_ipc_open": (c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
    "bc_ipc_close": (c_int, [c_void_p]),
    "bc_decode_attention_xchg": (c_int, [c_void_p, KVPlanes, KVPlanes, c_void_p, c_int, c_int, c_int, c_int64, c_int,
                                         c_int, Xchg, c_void_p, c_size_t, c_void_p]),
    "bc_decode_step_paged": (c_int, [c_void_p, c_void_p, c_void_p, KVPlanes, KVPlanes, c_void_p, c_void_p, PageTable,
                                     c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "bc_append_kv_paged": (c_int, [c_void_p, c_void_p, KVPlanes, KVPlanes, PageTable, c_int, c_int, c_int64, c_int,
                                   c_void_p]),
    "bc_decode_noalloc_max_scratch_bytes": (c_size_t, []),
    "bc_decode_attention_noalloc": (c_int, [c_void_p, KVPlanes, KVPlanes, c_void_p, c_void_p, c_int, c_int, c_int,
                                            c_int64, c_int, c_int, c_void_p]),
    "bc_select_workspace_bytes": (c_size_t, [c_int, c_int64]),
    "bc_select_residual_topk": (c_int, [KVPlanes, c_int, c_int, c_int64, c_int, c_int, c_void_p, c_int, c_void_p,
                                        c_size_t, c_void_p]),
    "bc_lse_merge": (c_int, [c_void_p, c_int, c_int64, c_int, c_void_p, c_void_p]),
    "bc_stage_rows": (c_int, [c_void_p, c_int, c_void_p]),
    "bc_xnor_popcount": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int64, c_int, c_void_p]),
    "bc_records_to_planes": (c_int, [c_void_p, c_void_p, KVPlanes, c_int64, c_int, c_void_p]),
    "bc_planes_to_records": (c_int, [KVPlanes, c_void_p, c_void_p, c_int64, c_int, c_void_p]),
}

# Every symbol include/bitcache_b200.h declares.
EXPORTED = tuple(_SIGS)

_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load the shared library (once) and attach the C signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"bitcache_b200 native library not found at {LIB_PATH}; build it with "
                "`python -m bitcache_b200.build`")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            try:
                fn = getattr(lib, name)
            except AttributeError as e:
                raise RuntimeError(f"{LIB_PATH} lacks {name}; rebuild with `python -m bitcache_b200.build`") from e
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def available() -> bool:
    try:
        load()
        return True
    except (RuntimeError, OSError):
        return False


def check(status: int, what: str) -> None:
    if status != BC_OK:
        msg = load().bc_status_string(status).decode()
        raise RuntimeError(f"{what} failed: {msg} (status {status})")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


# Zero-filled split-K workspaces, one per (device, stream, shape key).  The
# kernels return their ticket counters to zero on completion, so a workspace
# is reused without clearing by later calls of the same (n_slots, group) on
# the same stream; a different shape gets its own buffer because its partials
# could land on this shape's counters.
_ws: dict[tuple, torch.Tensor] = {}


def workspace(device: torch.device, stream: int, nbytes: int, shape_key: tuple = ()) -> torch.Tensor | None:
    if nbytes <= 0:
        return None
    key = (device.index if device.index is not None else torch.cuda.current_device(), stream) + tuple(shape_key)
    t = _ws.get(key)
    if t is None or t.numel() < nbytes:
        t = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
        _ws[key] = t
    return t


def device_error(clear: bool = True) -> int:
    return int(load().bc_get_device_error(1 if clear else 0))
