"""GPU: the allocation-free decode entry point (bc_decode_attention_noalloc),
called through the C ABI, gives the same attention as bc_decode_attention
with a caller workspace, on consecutive calls and across shapes that share
its fixed scratch array.  Collected last on purpose: it checks a shared
library-global array, so every other test has already run when it fails."""
import numpy as np
import pytest
import torch

from bitcache_b200 import _lib, planes

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-3
MIN_COS = 0.9999


def _close(got, want):
    g = got.float().cpu().numpy().astype(np.float64).ravel()
    w = want.float().cpu().numpy().astype(np.float64).ravel()
    assert np.max(np.abs(g - w)) <= MAX_ABS
    assert float(g @ w / (np.linalg.norm(g) * np.linalg.norm(w))) >= MIN_COS


def _case(cuda, slots, group, S, d, seed):
    g = torch.Generator().manual_seed(seed)
    K = planes.Planes.empty(slots, planes.round_stride(S), d, True, cuda)
    V = planes.Planes.empty(slots, planes.round_stride(S), d, True, cuda)
    planes.encode_planes((torch.randn(slots, S, d, generator=g) / d ** 0.5).half().to(cuda), K)
    planes.encode_planes((torch.randn(slots, S, d, generator=g) / d ** 0.5).half().to(cuda), V)
    q = (torch.randn(slots * group, d, generator=g) / d ** 0.5).half().to(cuda)
    return q, K, V, S


def _noalloc(q, K, V, S, mode=planes.MODE_COMPENSATED):
    lib = _lib.load()
    d = q.shape[-1]
    out = torch.empty_like(q)
    rc = lib.bc_decode_attention_noalloc(q.data_ptr(), K.c(), V.c(), out.data_ptr(), None, K.n_slots,
                                         q.shape[0] // K.n_slots, S, K.kv_stride, d, mode,
                                         torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.bc_status_string(rc).decode()
    return out


SHAPES = [(32, 1, 8192, 128), (4, 4, 3000, 64), (6, 2, 777, 256)]


@pytest.mark.parametrize("slots,group,S,d", SHAPES)
def test_noalloc_matches_workspace_entry_point(cuda, slots, group, S, d):
    q, K, V, S = _case(cuda, slots, group, S, d, slots + S)
    want = planes.decode_attention(q, K, V, S)
    first = _noalloc(q, K, V, S)
    second = _noalloc(q, K, V, S)
    torch.cuda.synchronize()
    _close(first, want)
    _close(second, want)


def test_noalloc_shapes_sharing_the_array(cuda):
    """Alternating shapes reuse the array; each call still matches its own reference."""
    cases = [_case(cuda, *shape, seed=i) for i, shape in enumerate(SHAPES)]
    wants = [planes.decode_attention(q, K, V, S) for q, K, V, S in cases]
    for _ in range(2):
        for (q, K, V, S), want in zip(cases, wants):
            _close(_noalloc(q, K, V, S), want)
    torch.cuda.synchronize()


def test_noalloc_rejects_shapes_beyond_its_scratch(cuda):
    lib = _lib.load()
    limit = lib.bc_decode_noalloc_max_scratch_bytes()
    assert limit == 4 << 20
    slots = 20000  # needs ~10 MB of split scratch
    assert lib.bc_decode_workspace_bytes(slots, 1, 64, 128) > limit
    P = _lib.KVPlanes()
    rc = lib.bc_decode_attention_noalloc(None, P, P, None, None, slots, 1, 64, 64, 128, 1, None)
    assert rc == 6  # BC_ERR_TOO_LARGE
    assert b"maximum" in lib.bc_status_string(rc)
