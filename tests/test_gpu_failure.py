"""GPU: the bounded waits give up instead of hanging, and the library stays
usable afterwards.  No GPU fault is provoked: the wait runs out because
nothing ever writes the words it waits for.

The peer exchange (bc_decode_attention_xchg) is called as rank 0 of a world
of 2 on one GPU, with both exchange buffers allocated on this GPU and no
rank 1: rank 0's kernel stores its triples into both buffers and then waits
for rank 1's, which never come.  With a short spin limit it must return
within milliseconds, raise BC_DEVERR_TIMEOUT, and leave the next calls
(plain decode, and an exchange of the next epoch) correct."""
import ctypes
import time

import pytest
import torch

from bitcache_b200 import _lib, planes
from bitcache_b200 import dist as bdist

pytestmark = pytest.mark.gpu


def _cache(cuda, slots, S, d, seed):
    g = torch.Generator().manual_seed(seed)
    K = planes.Planes.empty(slots, planes.round_stride(S), d, True, cuda)
    V = planes.Planes.empty(slots, planes.round_stride(S), d, True, cuda)
    planes.encode_planes((torch.randn(slots, S, d, generator=g) * 0.5).half().to(cuda), K)
    planes.encode_planes((torch.randn(slots, S, d, generator=g) * 0.5).half().to(cuda), V)
    q = (torch.randn(slots, d, generator=g) * 0.5).half().to(cuda)
    return q, K, V


@pytest.mark.parametrize("slots,S", [(4, 300), (32, 4096)])
def test_exchange_wait_gives_up_and_recovers(cuda, slots, S):
    lib = _lib.load()
    d = 128
    q, K, V = _cache(cuda, slots, S, d, seed=slots + S)
    want = planes.decode_attention(q, K, V, S)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    nbytes = lib.bc_xchg_bytes(slots, d, 2)
    bufs = []
    for _ in range(2):
        p = ctypes.c_void_p()
        _lib.check(lib.bc_xchg_alloc(nbytes, ctypes.byref(p)), "xchg_alloc")
        bufs.append(p.value)
    try:
        x = _lib.Xchg()
        x.bufs[0], x.bufs[1] = bufs
        x.world, x.rank, x.epoch, x.spin_limit, x.buf_bytes = 2, 0, 1, 20000, nbytes
        st = _lib.stream_of(cuda)
        wsb = lib.bc_decode_workspace_bytes(slots, 1, S, d)
        ws = torch.zeros(max(wsb, 16), dtype=torch.uint8, device=cuda)
        out = torch.zeros(slots, d, dtype=torch.float16, device=cuda)
        t0 = time.perf_counter()
        _lib.check(lib.bc_decode_attention_xchg(q.data_ptr(), K.c(), V.c(), out.data_ptr(), slots, 1, S, K.kv_stride,
                                                d, planes.MODE_COMPENSATED, x, ws.data_ptr(), ws.numel(), st),
                   "decode_attention_xchg")
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
        assert _lib.device_error(clear=True) & _lib.BC_DEVERR_TIMEOUT, "the wait for the missing rank did not give up"
        assert elapsed < 2.0, f"giving up took {elapsed:.2f} s"
        assert _lib.device_error() == 0
        # recovery: zero the workspace, then a plain decode and a one-rank exchange
        # of the next epoch through the same buffer are correct again
        ws.zero_()
        again = planes.decode_attention(q, K, V, S)
        x1 = _lib.Xchg()
        x1.bufs[0] = bufs[0]
        x1.world, x1.rank, x1.epoch, x1.spin_limit, x1.buf_bytes = 1, 0, 2, 20000, nbytes
        _lib.check(lib.bc_decode_attention_xchg(q.data_ptr(), K.c(), V.c(), out.data_ptr(), slots, 1, S, K.kv_stride,
                                                d, planes.MODE_COMPENSATED, x1, ws.data_ptr(), ws.numel(), st),
                   "decode_attention_xchg")
        torch.cuda.synchronize()
        assert _lib.device_error() == 0
        assert torch.equal(again, want)
        torch.testing.assert_close(out.float(), want.float(), atol=2e-3, rtol=0)
    finally:
        torch.cuda.synchronize()
        for p in bufs:
            lib.bc_xchg_free(p)


def test_exchange_refuses_calls_larger_than_its_buffers(cuda):
    """A call with more heads (or a larger head_dim) than the exchange buffers
    were sized for is refused before launch, in PeerExchange and in the C ABI."""
    lib = _lib.load()
    d = 128
    q, K, V = _cache(cuda, 8, 256, d, seed=3)
    x = bdist.PeerExchange(4, d)
    try:
        with pytest.raises(RuntimeError, match="built for 4 heads"):
            x.decode(q, K, V, 256, planes.MODE_COMPENSATED)
        c = _lib.Xchg()
        c.bufs[0] = x._own
        c.world, c.rank, c.epoch, c.buf_bytes = 1, 0, 1, lib.bc_xchg_bytes(4, d, 1)
        out = torch.empty(8, d, dtype=torch.float16, device=cuda)
        rc = lib.bc_decode_attention_xchg(q.data_ptr(), K.c(), V.c(), out.data_ptr(), 8, 1, 256, K.kv_stride, d,
                                          planes.MODE_COMPENSATED, c, None, 0, _lib.stream_of(cuda))
        assert rc == 2  # BC_ERR_ARG
        torch.cuda.synchronize()
        assert _lib.device_error() == 0
    finally:
        x.close()


def test_exchange_one_rank_with_pinned_host_query_and_output(cuda):
    """PeerExchange with one rank on pinned host Q and output (the end-to-end form
    of the sequence split): bit-identical to the same exchange on device tensors
    and to the plain decode, on consecutive epochs."""
    slots, S, d = 8, 2048, 128
    q, K, V = _cache(cuda, slots, S, d, seed=7)
    want = planes.decode_attention(q, K, V, S).cpu()
    x = bdist.PeerExchange(slots, d)
    try:
        dev_out = x.decode(q, K, V, S, planes.MODE_COMPENSATED).cpu()
        assert torch.equal(dev_out, want)
        qh = q.cpu().pin_memory()
        oh = torch.zeros(slots, d, dtype=torch.float16).pin_memory()
        for _ in range(2):
            oh.zero_()
            x.decode(qh, K, V, S, planes.MODE_COMPENSATED, out=oh)
            torch.cuda.synchronize()
            assert torch.equal(oh, want)
        assert _lib.device_error() == 0
    finally:
        x.close()
