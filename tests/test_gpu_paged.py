"""GPU: paged caches (block table over a page pool) against the contiguous
layout.  The decode plan depends only on the logical shape, so a paged cache
holding the same rows must give bit-identical outputs and, after an append,
bit-identical rows."""
import numpy as np
import pytest
import torch

from bitcache_b200 import _lib, planes

pytestmark = pytest.mark.gpu


def make(cuda, slots, S, d, comp, seed, page_size, spare=3):
    g = torch.Generator().manual_seed(seed)
    stride = planes.round_stride(max(S, 1))
    rm = planes.RES_FP32_SCALE if comp else planes.RES_NONE
    K = planes.Planes.empty(slots, stride + page_size, d, comp, cuda)
    V = planes.Planes.empty(slots, stride + page_size, d, comp, cuda)
    if S:
        planes.encode_planes((torch.randn(slots, S, d, generator=g) * 0.5).half().to(cuda), K, rm)
        planes.encode_planes((torch.randn(slots, S, d, generator=g) * 0.5).half().to(cuda), V, rm)
    max_pages = (stride + page_size) // page_size
    n_pages = slots * max_pages + spare
    perm = torch.randperm(n_pages, generator=g)[: slots * max_pages].to(torch.int32)
    pt = planes.PageTable(perm.view(slots, max_pages).contiguous().to(cuda), page_size, n_pages)
    Kp = planes.paginate(K, pt, max_pages * page_size)
    Vp = planes.paginate(V, pt, max_pages * page_size)
    return K, V, Kp, Vp, pt


def rows_equal(P, pool, pt, seq_len, comp):
    back = planes.Planes.empty(pt.n_slots, pt.pages.shape[1] * pt.page_size, P.head_dim, comp, P.sign.device)
    table = pt.pages.cpu()
    for s in range(pt.n_slots):
        for j in range(pt.pages.shape[1]):
            pg = int(table[s, j])
            for name in ("sign", "bscale", "nib", "rscale"):
                if getattr(P, name) is not None:
                    getattr(back, name)[s, j * pt.page_size:(j + 1) * pt.page_size].copy_(getattr(pool, name)[pg])
    n = planes.round_stride(seq_len)
    assert torch.equal(back.sign[:, :seq_len], P.sign[:, :seq_len])
    assert torch.equal(back.bscale[:, :seq_len], P.bscale[:, :seq_len])
    if comp:
        assert torch.equal(back.nib_rows()[:, :seq_len], P.nib_rows()[:, :seq_len])
        assert torch.equal(back.rscale[:, :seq_len], P.rscale[:, :seq_len])
    del n


@pytest.mark.parametrize("slots,group,S,d,comp,page", [
    (4, 1, 3000, 128, True, 128),
    (4, 1, 3000, 128, True, 512),
    (3, 4, 1100, 128, True, 256),
    (2, 8, 777, 64, False, 128),
    (2, 2, 300, 256, True, 128),
    (5, 1, 129, 32, True, 128),
])
def test_paged_attention_bit_identical(cuda, slots, group, S, d, comp, page):
    K, V, Kp, Vp, pt = make(cuda, slots, S, d, comp, seed=S + d, page_size=page)
    g = torch.Generator().manual_seed(7)
    q = (torch.randn(slots * group, d, generator=g) * 0.5).half().to(cuda)
    mode = planes.MODE_COMPENSATED if comp else planes.MODE_BINARY
    want = planes.decode_attention(q, K, V, S, mode)
    got = planes.decode_step_paged(q, None, None, Kp, Vp, pt, S, -1, mode)
    torch.cuda.synchronize()
    assert torch.equal(got, want)


@pytest.mark.parametrize("pos_kind", ["end", "inside", "page_start"])
@pytest.mark.parametrize("group", [1, 4])
def test_paged_step_equals_contiguous_step(cuda, pos_kind, group):
    slots, S0, d, page = 3, 900, 128, 256
    K, V, Kp, Vp, pt = make(cuda, slots, S0, d, True, seed=11, page_size=page)
    pos = {"end": S0, "inside": 333, "page_start": 512}[pos_kind]
    S = max(S0, pos + 1) if pos_kind == "end" else S0
    g = torch.Generator().manual_seed(13)
    q = (torch.randn(slots * group, d, generator=g) * 0.5).half().to(cuda)
    k = (torch.randn(slots, d, generator=g) * 0.5).half().to(cuda)
    v = (torch.randn(slots, d, generator=g) * 0.5).half().to(cuda)
    want = planes.decode_step(q, k, v, K, V, S, pos)
    got = planes.decode_step_paged(q, k, v, Kp, Vp, pt, S, pos)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    rows_equal(K, Kp, pt, S, True)
    rows_equal(V, Vp, pt, S, True)


def test_paged_append_equals_contiguous_append(cuda):
    slots, S0, d, page = 4, 200, 64, 128
    K, V, Kp, Vp, pt = make(cuda, slots, S0, d, True, seed=17, page_size=page)
    g = torch.Generator().manual_seed(19)
    for pos in (S0, 255, 0):
        k = (torch.randn(slots, d, generator=g) * 0.5).half().to(cuda)
        v = (torch.randn(slots, d, generator=g) * 0.5).half().to(cuda)
        planes.append_kv(k, v, K, V, pos)
        planes.append_kv_paged(k, v, Kp, Vp, pt, pos)
    torch.cuda.synchronize()
    rows_equal(K, Kp, pt, 256, True)
    rows_equal(V, Vp, pt, 256, True)


def test_paged_rejects_bad_geometry(cuda):
    K, V, Kp, Vp, pt = make(cuda, 2, 100, 128, True, seed=1, page_size=128)
    q = torch.zeros(2, 128, dtype=torch.float16, device=cuda)
    bad = planes.PageTable(pt.pages, 96, pt.n_pages)  # not a multiple of the 128-key tile
    with pytest.raises(RuntimeError):
        planes.decode_step_paged(q, None, None, Kp, Vp, bad, 100)
    with pytest.raises(RuntimeError):  # more keys than the table can address
        planes.decode_step_paged(q, None, None, Kp, Vp, pt, pt.pages.shape[1] * 128 + 1)


def test_out_of_pool_page_is_reported_not_dereferenced(cuda):
    """A block-table entry outside [0, n_pages) is checked in the kernel: the
    tile is not copied, BC_DEVERR_PAGE is raised, and the context stays usable."""
    K, V, Kp, Vp, pt = make(cuda, 2, 600, 128, True, seed=3, page_size=128)
    assert _lib.device_error() == 0
    pages = pt.pages.clone()
    pages[1, 2] = pt.n_pages + 5
    pages[0, 0] = -1
    bad = planes.PageTable(pages, pt.page_size, pt.n_pages)
    q = torch.zeros(2, 128, dtype=torch.float16, device=cuda)
    planes.decode_step_paged(q, None, None, Kp, Vp, bad, 600)
    assert _lib.device_error() & _lib.BC_DEVERR_PAGE
    k = torch.zeros(2, 128, dtype=torch.float16, device=cuda)
    planes.append_kv_paged(k, k, Kp, Vp, bad, 300)  # logical page 2 of slot 1 is bad
    assert _lib.device_error() & _lib.BC_DEVERR_PAGE
    _lib._ws.clear()  # aborted CTAs leave their split counters set
    ok = planes.decode_step_paged(q, None, None, Kp, Vp, pt, 600)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0 and torch.isfinite(ok.float()).all()
