"""GPU: encoders bit-exact against the reference's own kernels (oracle/_ref),
through the C ABI (via the _C / planes front ends)."""
import numpy as np
import pytest
import torch

import cases
from bitcache_b200 import _C, planes
from oracle import oracle as O
from oracle import refgpu

pytestmark = pytest.mark.gpu

D_ALL = [32, 64, 96, 128, 160, 192, 224, 256]


def src(n, d, seed, scale=0.5):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(n, d, generator=g) * scale).half()
    return x


def with_edges(x):
    d = x.shape[1]
    return torch.cat([x, cases.edge_vectors(d), cases.special_vectors(d)]).contiguous()


def fields_bin(blob, d):
    return O.split_binvec(blob.cpu().numpy(), d)


def fields_res(blob, d):
    return O.split_resvec(blob.cpu().numpy(), d)


@pytest.mark.parametrize("d", D_ALL)
def test_binary_encode_bit_exact(cuda, d):
    x = with_edges(src(3000, d, d)).to(cuda)
    mine = _C.binary_encode(x)
    ref = refgpu.binary_encode(x)
    torch.cuda.synchronize()
    wm, sm = fields_bin(mine, d)
    wr, sr = fields_bin(ref, d)
    assert np.array_equal(wm, wr)
    assert np.array_equal(sm, sr)
    # unused words and padding are zeroed in this implementation
    rec = np.frombuffer(mine.cpu().numpy().tobytes(), O.BINVEC)
    assert not rec["words"][:, d // 32:].any() and not rec["pad"].any()


@pytest.mark.parametrize("d", D_ALL)
def test_residual_encode_bit_exact(cuda, d):
    x = with_edges(src(3000, d, 100 + d)).to(cuda)
    rb = refgpu.binary_encode(x)
    mine = _C.residual_encode(x, rb)
    ref = refgpu.residual_encode(x, rb)
    chain = _C.residual_encode(x, _C.binary_encode(x))
    torch.cuda.synchronize()
    nm, sm = fields_res(mine, d)
    nr, sr = fields_res(ref, d)
    assert np.array_equal(nm, nr)
    assert np.array_equal(sm, sr)
    nc, sc = fields_res(chain, d)
    assert np.array_equal(nc, nr) and np.array_equal(sc, sr)


@pytest.mark.parametrize("d", [64, 128, 256])
def test_encode_matches_oracle(cuda, d):
    x = src(2000, d, 7 + d)
    xg = x.to(cuda)
    b = _C.binary_encode(xg)
    r = _C.residual_encode(xg, b)
    w, s = fields_bin(b, d)
    nib, rs = fields_res(r, d)
    ow, os_ = O.binary_encode(x.numpy())
    assert np.array_equal(w, ow) and np.array_equal(s, os_)
    on, ors, pre = O.residual_encode(x.numpy(), w, s)
    assert np.array_equal(rs, ors)
    from test_oracle_golden import check_codes

    check_codes(nib, on, pre, f"gpu-vs-oracle d={d}")


@pytest.mark.parametrize("d", D_ALL)
@pytest.mark.parametrize("mode", [planes.RES_FP16_SCALE, planes.RES_NONE])
def test_plane_encode_bit_exact(cuda, d, mode):
    slots, seq = 3, 203
    x = src(slots * seq, d, 300 + d).to(cuda)
    P = planes.Planes.empty(slots, planes.round_stride(seq) + 8, d, mode != planes.RES_NONE, cuda)
    planes.encode_planes(x.view(slots, seq, d), P, mode)
    rb = refgpu.binary_encode(x)
    wr, sr = fields_bin(rb, d)
    torch.cuda.synchronize()
    assert np.array_equal(P.sign[:, :seq].cpu().numpy().view(np.uint32).reshape(-1, d // 32), wr)
    assert np.array_equal(P.bscale[:, :seq].cpu().numpy().view(np.uint16).reshape(-1), sr)
    assert not P.sign[:, seq:].any()
    if mode != planes.RES_NONE:
        rr = refgpu.residual_encode(x, rb)
        nr, rsr = fields_res(rr, d)
        assert np.array_equal(P.nib_rows()[:, :seq].cpu().numpy().reshape(-1, d // 2), nr)
        assert np.array_equal(P.rscale[:, :seq].cpu().numpy().view(np.uint16).reshape(-1), rsr)


@pytest.mark.parametrize("d", [64, 128, 256, 96])
def test_online_encode_ring_bit_exact(cuda, d):
    B, H, max_seq, steps = 2, 3, 16, 21
    g = torch.Generator().manual_seed(d)
    toks = (torch.randn(steps, B * H, d, generator=g) * 0.5).half().to(cuda)
    n = B * H * max_seq
    mb = torch.zeros(n * 36, dtype=torch.uint8, device=cuda)
    mr = torch.zeros(n * 130, dtype=torch.uint8, device=cuda)
    rb = torch.zeros_like(mb)
    rr = torch.zeros_like(mr)
    for t in range(steps):
        _C.online_encode_token(toks[t], mb, mr, B, H, d, t, max_seq)
        refgpu.online_encode_token(toks[t], rb, rr, B, H, d, t, max_seq)
    torch.cuda.synchronize()
    assert np.array_equal(fields_bin(mb, d)[0], fields_bin(rb, d)[0])
    assert np.array_equal(fields_bin(mb, d)[1], fields_bin(rb, d)[1])
    assert np.array_equal(fields_res(mr, d)[0], fields_res(rr, d)[0])
    assert np.array_equal(fields_res(mr, d)[1], fields_res(rr, d)[1])


def test_online_encode_binary_only_cache(cuda):
    d, B, H, max_seq = 128, 1, 4, 8
    x = src(B * H, d, 5).to(cuda)
    mb = torch.zeros(B * H * max_seq * 36, dtype=torch.uint8, device=cuda)
    _C.online_encode_token(x, mb, None, B, H, d, 3, max_seq)
    rb = refgpu.binary_encode(x)
    w, s = fields_bin(mb, d)
    wr, sr = fields_bin(rb, d)
    idx = np.arange(B * H) * max_seq + 3
    assert np.array_equal(w[idx], wr) and np.array_equal(s[idx], sr)


@pytest.mark.parametrize("d", [64, 128, 256])
def test_append_kv_matches_online_records(cuda, d):
    slots, stride, pos = 5, 24, 17
    k = src(slots, d, 1).to(cuda)
    v = src(slots, d, 2).to(cuda)
    K = planes.Planes.empty(slots, stride, d, True, cuda)
    V = planes.Planes.empty(slots, stride, d, True, cuda)
    planes.append_kv(k, v, K, V, pos)
    for X, x in ((K, k), (V, v)):
        bb = torch.zeros(slots * stride * 36, dtype=torch.uint8, device=cuda)
        rr = torch.zeros(slots * stride * 130, dtype=torch.uint8, device=cuda)
        refgpu.online_encode_token(x, bb, rr, 1, slots, d, pos, stride)
        w, s = fields_bin(bb, d)
        nib, rs = fields_res(rr, d)
        torch.cuda.synchronize()
        assert np.array_equal(X.sign.cpu().numpy().view(np.uint32).reshape(-1, d // 32), w)
        assert np.array_equal(X.bscale.cpu().numpy().view(np.uint16).reshape(-1), s)
        assert np.array_equal(X.nib_rows().cpu().numpy().reshape(-1, d // 2), nib)
        assert np.array_equal(X.rscale.cpu().numpy().view(np.uint16).reshape(-1), rs)


@pytest.mark.parametrize("d", [64, 128, 256])
def test_record_plane_converters_roundtrip(cuda, d):
    x = src(777, d, 9).to(cuda)
    b = refgpu.binary_encode(x)
    r = refgpu.residual_encode(x, b)
    P = planes.records_to_planes(b, r, 777, d)
    b2, r2 = planes.planes_to_records(P, 777)
    torch.cuda.synchronize()
    for f in (0, 1):
        assert np.array_equal(fields_bin(b2, d)[f], fields_bin(b, d)[f])
        assert np.array_equal(fields_res(r2, d)[f], fields_res(r, d)[f])


@pytest.mark.parametrize("d", D_ALL)
@pytest.mark.parametrize("mode", [planes.RES_FP16_SCALE, planes.RES_FP32_SCALE, planes.RES_NONE])
def test_plane_encode_edge_vectors_bit_exact(cuda, d, mode):
    """Zero, -0, subnormal, huge, inf and NaN vectors through the prefill encoder
    (the lane-per-vector kernel at head_dim <= 128) against the reference kernels
    (FP16 scale: residual.cu) or the online encoder (FP32 scale: online_encode.cu)."""
    x = with_edges(src(61, d, 900 + d)).to(cuda)
    n = x.shape[0]
    P = planes.Planes.empty(1, planes.round_stride(n), d, mode != planes.RES_NONE, cuda)
    planes.encode_planes(x.view(1, n, d), P, mode)
    rb = refgpu.binary_encode(x)
    wr, sr = fields_bin(rb, d)
    torch.cuda.synchronize()
    assert np.array_equal(P.sign[0, :n].cpu().numpy().view(np.uint32), wr)
    assert np.array_equal(P.bscale[0, :n].cpu().numpy().view(np.uint16), sr)
    if mode == planes.RES_FP16_SCALE:
        nr, rsr = fields_res(refgpu.residual_encode(x, rb), d)
    elif mode == planes.RES_FP32_SCALE:
        bb = torch.zeros(n * 36, dtype=torch.uint8, device=cuda)
        rr = torch.zeros(n * 130, dtype=torch.uint8, device=cuda)
        refgpu.online_encode_token(x, bb, rr, 1, n, d, 0, 1)  # n slots of a 1-position ring
        nr, rsr = fields_res(rr, d)
    else:
        return
    torch.cuda.synchronize()
    assert np.array_equal(P.nib_rows()[0, :n].cpu().numpy(), nr)
    assert np.array_equal(P.rscale[0, :n].cpu().numpy().view(np.uint16), rsr)
