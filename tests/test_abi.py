"""CPU: the C-ABI library loads, exports every symbol the header declares, and
rejects invalid arguments with the documented status codes before touching
the GPU.  Also the Python front ends' error behaviour on CPU tensors."""
import ctypes
import os
import re

import pytest
import torch

from bitcache_b200 import _lib, _C, functional, planes, workloads

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "bitcache_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = set(re.findall(r"\b(bc_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_symbols()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), f"{n} declared in bitcache_b200.h but not exported"
    assert set(names) == set(_lib.EXPORTED), "ctypes signature table out of sync with the header"


def test_record_sizes():
    lib = _lib.load()
    assert lib.bc_sizeof_binary_vec() == 36
    assert lib.bc_sizeof_residual_vec() == 130


@pytest.mark.parametrize("d", [0, 16, 33, 288, -32])
def test_bad_head_dim_rejected(d):
    lib = _lib.load()
    assert lib.bc_binary_encode(None, None, 4, d, None) == 1
    assert lib.bc_residual_encode(None, None, None, 4, d, None) == 1
    assert lib.bc_online_encode_token(None, None, None, 1, 1, d, 0, 8, None) == 1
    assert lib.bc_binary_attention(None, None, None, None, 1, 1, 8, d, None, 0, None) == 1
    assert lib.bc_compute_head_entropy(None, None, None, 1, 1, 8, d, None, 0, None) == 1
    P = _lib.KVPlanes()
    assert lib.bc_decode_attention(None, P, P, None, None, 1, 1, 8, 8, d, 1, None, 0, None) == 1


def test_argument_errors():
    lib = _lib.load()
    P = _lib.KVPlanes()
    assert lib.bc_binary_encode(None, None, -1, 128, None) == 2
    assert lib.bc_binary_encode(None, None, 0, 128, None) == 0  # empty is a no-op
    assert lib.bc_binary_encode(None, None, 3, 128, None) == 2  # null pointers
    assert lib.bc_decode_attention(None, P, P, None, None, 1, 3, 8, 8, 128, 1, None, 0, None) == 5  # group 3
    assert lib.bc_decode_attention(None, P, P, None, None, 1, 1, 16, 8, 128, 1, None, 0, None) == 2  # stride < seq
    assert lib.bc_decode_attention(None, P, P, None, None, 1, 1, 8, 8, 128, 7, None, 0, None) == 2  # mode
    assert lib.bc_decode_attention(None, P, P, None, None, 0, 1, 8, 8, 128, 1, None, 0, None) == 0  # no slots
    fake = _lib.KVPlanes(16, 16, 16, 16)
    assert lib.bc_decode_attention(16, fake, fake, 16, None, 1, 1, 8, 12, 128, 1, None, 0, None) == 3  # stride%8
    unaligned = _lib.KVPlanes(24, 16, 16, 16)
    assert lib.bc_decode_attention(16, unaligned, fake, 16, None, 1, 1, 8, 8, 128, 1, None, 0, None) == 3
    assert lib.bc_append_kv(16, 16, fake, fake, 1, 128, 8, 8, 2, None) == 2  # pos >= kv_stride
    assert lib.bc_lse_merge(None, 0, 1, 128, None, None) == 2


def test_status_strings():
    lib = _lib.load()
    assert b"head_dim" in lib.bc_status_string(1)
    assert b"workspace" in lib.bc_status_string(4)


def test_workspace_query():
    lib = _lib.load()
    assert lib.bc_decode_workspace_bytes(32, 1, 65536, 128) > 0
    assert lib.bc_decode_workspace_bytes(0, 1, 65536, 128) == 0
    assert lib.bc_decode_workspace_bytes(32, 3, 65536, 128) == 0
    # bounded by slots * splits * (d + 4 attention + 3 entropy) floats; compensated plans may
    # take up to four waves of splits (4 * 640 CTAs), so splits <= 2560 / slots
    assert lib.bc_decode_workspace_bytes(32, 1, 65536, 128) <= 32 * 80 * (132 + 3) * 4 + 4096


def test_python_front_ends_reject_cpu_tensors():
    x = torch.zeros(4, 128, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA"):
        _C.binary_encode(x)
    with pytest.raises(AssertionError):
        functional.encode(x)
    with pytest.raises(RuntimeError):
        planes.decode_attention(x, None, None, 1)


def test_vector_footprints():
    assert planes.vector_bytes(128) == 84
    assert planes.vector_bytes(128, False) == 18
    assert workloads.vector_footprint(128) == 82
    assert workloads.step_cache_bytes(1, 32, 65536, 128) == 343_932_928


def test_exchange_struct_and_size_check():
    """bc_xchg carries the buffers' size; a call whose heads would not fit is
    refused on the host (BC_ERR_ARG) before anything is launched."""
    lib = _lib.load()
    assert ctypes.sizeof(_lib.Xchg) == 88
    fake = _lib.KVPlanes(16, 16, 16, 16)
    x = _lib.Xchg()
    x.bufs[0] = 256
    x.world, x.rank, x.epoch = 1, 0, 1
    x.buf_bytes = lib.bc_xchg_bytes(4, 128, 1)  # sized for 4 heads
    assert lib.bc_decode_attention_xchg(16, fake, fake, 16, 8, 1, 64, 64, 128, 1, x, None, 0, None) == 2
    x.buf_bytes = 0
    assert lib.bc_decode_attention_xchg(16, fake, fake, 16, 4, 1, 64, 64, 128, 1, x, None, 0, None) == 2


def test_peer_exchange_refuses_other_shapes():
    """PeerExchange.decode checks the call's heads and head_dim against the
    sizes its buffers were allocated for, before any device work."""
    from types import SimpleNamespace

    from bitcache_b200 import dist as bdist

    x = object.__new__(bdist.PeerExchange)
    x._lib = _lib
    x.n_heads, x.head_dim = 4, 128
    K = SimpleNamespace(n_slots=8)
    with pytest.raises(RuntimeError, match="built for 4 heads of dim 128"):
        x.decode(torch.zeros(8, 128, dtype=torch.float16), K, K, 64, 1)
    with pytest.raises(RuntimeError, match="built for 4 heads of dim 128"):
        x.decode(torch.zeros(4, 64, dtype=torch.float16), SimpleNamespace(n_slots=4), K, 64, 1)


def test_host_operands_must_be_pinned():
    """Host-resident Q and output are read and written by the GPU directly, so
    the adaptive and exchange decodes refuse pageable host tensors (and a
    too-small output) before any device work."""
    from types import SimpleNamespace

    from bitcache_b200 import dist as bdist
    from bitcache_b200 import planes

    q = torch.zeros(4, 128, dtype=torch.float16)  # pageable host memory
    with pytest.raises(RuntimeError, match="pinned host tensor"):
        planes.device_query(q, torch.device("cpu"))
    x = object.__new__(bdist.PeerExchange)
    x._lib = _lib
    x.n_heads, x.head_dim = 4, 128
    K = SimpleNamespace(n_slots=4, sign=SimpleNamespace(device=torch.device("cpu")))
    with pytest.raises(RuntimeError, match="pinned host tensor"):
        x.decode(q, K, K, 64, 1)
    with pytest.raises(RuntimeError, match="pinned host tensor"):
        x.decode(q, K, K, 64, 1, out=torch.zeros(4, 128, dtype=torch.float16))


def test_bitcache_import_name():
    """The reference's import name gives this implementation."""
    import bitcache
    import bitcache.functional as F
    from bitcache import _C as C

    import bitcache_b200

    assert bitcache.BitCache is bitcache_b200.BitCache
    assert F.compensated_attention is functional.compensated_attention
    assert C.online_encode_token is _C.online_encode_token
    assert callable(bitcache._require_extension)


def test_stage_rows_argument_checks():
    """bc_stage_rows refuses unaligned segments and too many segments before launching."""
    lib = _lib.load()
    segs = (_lib.CopySeg * 5)()
    segs[0].src, segs[0].dst, segs[0].bytes = 16, 32, 24  # size not a multiple of 16
    assert lib.bc_stage_rows(segs, 1, None) == 3
    segs[0].src, segs[0].dst, segs[0].bytes = 8, 32, 32  # unaligned source
    assert lib.bc_stage_rows(segs, 1, None) == 3
    assert lib.bc_stage_rows(segs, 5, None) == 2  # at most 4 segments
    assert lib.bc_stage_rows(segs, 0, None) == 0  # nothing to do
