"""GPU: the fused decode step (bc_decode_step: append + attend in one launch)
against the two-launch path it replaces (bc_append_kv + bc_decode_attention)
and against the C oracle.  The planes must receive identical bytes; the
outputs must agree within the north-star tolerance (the step kernel may plan a
different split count, which only reorders the fp32 split-K sums)."""
import numpy as np
import pytest
import torch

from bitcache_b200 import BitCache, planes
from oracle import oracle as O

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-3
MIN_COS = 0.9999


def close(got, want, label=""):
    g = got.float().cpu().numpy().astype(np.float64).ravel()
    w = want.float().cpu().numpy().astype(np.float64).ravel() if torch.is_tensor(want) else want.astype(np.float64).ravel()
    err = float(np.max(np.abs(g - w))) if g.size else 0.0
    cos = float(g @ w / (np.linalg.norm(g) * np.linalg.norm(w) + 1e-30)) if g.size else 1.0
    assert err <= MAX_ABS, f"{label}: max-abs {err:.3g}"
    if np.linalg.norm(w) > 1e-6:
        assert cos >= MIN_COS, f"{label}: cosine {cos:.6f}"


def planes_equal(A, B, seq_len, comp):
    assert torch.equal(A.sign[:, :seq_len], B.sign[:, :seq_len])
    assert torch.equal(A.bscale[:, :seq_len], B.bscale[:, :seq_len])
    if comp:
        assert torch.equal(A.nib_rows()[:, :seq_len], B.nib_rows()[:, :seq_len])
        assert torch.equal(A.rscale[:, :seq_len], B.rscale[:, :seq_len])


def filled_pair(slots, stride, d, comp, S0, cuda, seed):
    g = torch.Generator().manual_seed(seed)
    x = [(torch.randn(slots, S0, d, generator=g) * 0.5).half().to(cuda) for _ in range(2)]
    out = []
    for _ in range(2):
        K = planes.Planes.empty(slots, stride, d, comp, cuda)
        V = planes.Planes.empty(slots, stride, d, comp, cuda)
        if S0:
            rm = planes.RES_FP32_SCALE if comp else planes.RES_NONE
            planes.encode_planes(x[0], K, rm)
            planes.encode_planes(x[1], V, rm)
        out.append((K, V))
    return out


# (slots, group, d, comp, S0 already cached, max_seq): the step appends at S0 (growing)
# or, with a full ring, at a position inside the range.
CASES = [
    (4, 1, 128, True, 1000, 4096),    # append at the end, several splits
    (4, 1, 128, True, 0, 64),         # first token: seq_len 1
    (2, 1, 64, True, 127, 512),       # append lands on a tile's last key
    (2, 1, 64, True, 128, 512),       # ... and on a tile's first key
    (3, 4, 128, True, 777, 1024),     # grouped-query: head groups 1.. patch without storing
    (2, 8, 128, False, 2047, 4096),   # binary, four heads per CTA
    (2, 2, 256, True, 300, 512),
    (3, 4, 64, True, 500, 1024),      # four heads per CTA at head_dim 64 (by-bit planes)
    (2, 4, 256, True, 200, 512),      # two head groups of two at head_dim 256
    (5, 1, 32, True, 4095, 8192),
    (1, 1, 128, False, 65, 128),
]


@pytest.mark.parametrize("slots,group,d,comp,S0,max_seq", CASES)
def test_step_equals_append_then_attend(cuda, slots, group, d, comp, S0, max_seq):
    stride = planes.round_stride(max_seq)
    (K1, V1), (K2, V2) = filled_pair(slots, stride, d, comp, S0, cuda, seed=S0 + d)
    g = torch.Generator().manual_seed(99 + S0)
    q = (torch.randn(slots * group, d, generator=g) * 0.5).half().to(cuda)
    k = (torch.randn(slots, d, generator=g) * 0.5).half().to(cuda)
    v = (torch.randn(slots, d, generator=g) * 0.5).half().to(cuda)
    mode = planes.MODE_COMPENSATED if comp else planes.MODE_BINARY
    rm = planes.RES_FP32_SCALE if comp else planes.RES_NONE
    S = S0 + 1
    got = planes.decode_step(q, k, v, K1, V1, S, S0, mode, rm)
    planes.append_kv(k, v, K2, V2, S0, rm)
    want = planes.decode_attention(q, K2, V2, S, mode)
    torch.cuda.synchronize()
    planes_equal(K1, K2, S, comp)
    planes_equal(V1, V2, S, comp)
    close(got, want, f"step slots{slots} g{group} d{d} comp={comp} S0={S0}")


@pytest.mark.parametrize("pos", [0, 5, 128, 999, 1023])
@pytest.mark.parametrize("group", [1, 4])
def test_step_full_ring_overwrites_inside_range(cuda, pos, group):
    """Full ring: the appended row replaces a cached one; every other CTA must
    keep reading the old rows, the owner of pos must attend the new one."""
    slots, d, S = 3, 128, 1024
    (K1, V1), (K2, V2) = filled_pair(slots, S, d, True, S, cuda, seed=pos)
    g = torch.Generator().manual_seed(pos + 7)
    q = (torch.randn(slots * group, d, generator=g) * 0.5).half().to(cuda)
    k = (torch.randn(slots, d, generator=g) * 2.0).half().to(cuda)  # a large row: its effect is visible
    v = (torch.randn(slots, d, generator=g) * 2.0).half().to(cuda)
    got = planes.decode_step(q, k, v, K1, V1, S, pos)
    before = planes.decode_attention(q, K2, V2, S)
    planes.append_kv(k, v, K2, V2, pos)
    want = planes.decode_attention(q, K2, V2, S)
    torch.cuda.synchronize()
    planes_equal(K1, K2, S, True)
    planes_equal(V1, V2, S, True)
    close(got, want, f"ring pos={pos} group={group}")
    assert (got.float() - before.float()).abs().max() > 1e-3  # the new row did change the answer


def test_step_res_fp16_scale_and_no_append(cuda):
    slots, d, S0 = 4, 64, 300
    (K1, V1), (K2, V2) = filled_pair(slots, 512, d, True, S0, cuda, seed=3)
    g = torch.Generator().manual_seed(4)
    q = (torch.randn(slots, d, generator=g) * 0.5).half().to(cuda)
    k = (torch.randn(slots, d, generator=g) * 0.5).half().to(cuda)
    v = (torch.randn(slots, d, generator=g) * 0.5).half().to(cuda)
    got = planes.decode_step(q, k, v, K1, V1, S0 + 1, S0, residual_mode=planes.RES_FP16_SCALE)
    planes.append_kv(k, v, K2, V2, S0, planes.RES_FP16_SCALE)
    want = planes.decode_attention(q, K2, V2, S0 + 1)
    torch.cuda.synchronize()
    planes_equal(K1, K2, S0 + 1, True)
    close(got, want, "fp16-scale append")
    # append_pos = -1: plain attention, planes untouched
    snap = K1.sign.clone()
    plain = planes.decode_step(q, None, None, K1, V1, S0 + 1, -1)
    torch.cuda.synchronize()
    assert torch.equal(K1.sign, snap)
    close(plain, want, "no append")


def test_step_rejects_bad_arguments(cuda):
    K = planes.Planes.empty(1, 64, 128, True, cuda)
    V = planes.Planes.empty(1, 64, 128, True, cuda)
    q = torch.zeros(1, 128, dtype=torch.float16, device=cuda)
    k = torch.zeros(1, 128, dtype=torch.float16, device=cuda)
    with pytest.raises(RuntimeError):
        planes.decode_step(q, k, k, K, V, 10, 10)  # pos outside [0, seq_len)
    with pytest.raises(RuntimeError):  # compensated attention needs the appended residual
        planes.decode_step(q, k, k, K, V, 10, 3, residual_mode=planes.RES_NONE)


def test_step_rejects_pageable_host_operands(cuda):
    """The kernel reads host operands through unified addressing, which only
    pinned memory has: the C ABI refuses pageable pointers (status, no launch)."""
    from bitcache_b200 import _lib
    lib = _lib.load()
    K = planes.Planes.empty(1, 64, 128, True, cuda)
    V = planes.Planes.empty(1, 64, 128, True, cuda)
    out = torch.empty(1, 128, dtype=torch.float16, device=cuda)
    qd = torch.zeros(1, 128, dtype=torch.float16, device=cuda)
    pageable = torch.zeros(1, 128, dtype=torch.float16)  # ordinary host memory
    assert not pageable.is_pinned()
    ws = torch.empty(1 << 20, dtype=torch.uint8, device=cuda)
    st = _lib.stream_of(cuda)
    for q, k in ((pageable, qd), (qd, pageable)):
        rc = lib.bc_decode_step(q.data_ptr(), k.data_ptr(), k.data_ptr(), K.c(), V.c(), out.data_ptr(), None, 1, 1,
                                10, K.kv_stride, 128, planes.MODE_COMPENSATED, 3, _lib.BC_RES_FP32_SCALE,
                                ws.data_ptr(), ws.numel(), st)
        assert rc == 2, f"pageable operand accepted (status {rc})"  # BC_ERR_ARG
    torch.cuda.synchronize()
    assert _lib.device_error() == 0


def test_bitcache_step_matches_append_attend_and_oracle(cuda):
    """BitCache.step over a ring that wraps, against append+attend on a twin
    cache (bit-identical planes) and the oracle on the final contents."""
    B, H, Hkv, d, max_seq, steps = 2, 8, 2, 128, 200, 230
    g = torch.Generator().manual_seed(17)
    ks = (torch.randn(steps, B, Hkv, d, generator=g) * 0.5).half()
    vs = (torch.randn(steps, B, Hkv, d, generator=g) * 0.5).half()
    qs = (torch.randn(steps, B, H, d, generator=g) * 0.5).half()
    a = BitCache(B, H, d, max_seq=max_seq, n_kv_heads=Hkv)
    b = BitCache(B, H, d, max_seq=max_seq, n_kv_heads=Hkv)
    for t in range(steps):
        kt, vt, qt = ks[t].to(cuda), vs[t].to(cuda), qs[t].to(cuda)
        got = a.step(qt, kt, vt)
        b.append(kt, vt)
        want = b.attend(qt)
        if t in (0, 1, 150, max_seq - 1, max_seq, steps - 1):
            close(got.view(-1, d), want.view(-1, d), f"t={t}")
    torch.cuda.synchronize()
    assert a.seq_len == b.seq_len == max_seq
    for X, Y in zip(a.planes, b.planes):
        planes_equal(X, Y, max_seq, True)
    # oracle on the final ring contents: positions hold tokens t with t % max_seq == pos
    order = [(steps - max_seq + i) for i in range(max_seq)]
    pos = [t % max_seq for t in order]
    kk = torch.empty(max_seq, B, Hkv, d, dtype=torch.float16)
    vv = torch.empty_like(kk)
    for t, p in zip(order, pos):
        kk[p] = ks[t]
        vv[p] = vs[t]
    n = B * Hkv
    kf = kk.permute(1, 2, 0, 3).reshape(-1, d).numpy()
    vf = vv.permute(1, 2, 0, 3).reshape(-1, d).numpy()
    ow, obs, onb, ors, _ = O.online_encode(kf)
    vw, vbs, vnb, vrs, _ = O.online_encode(vf)
    Kp = {"words": ow.reshape(n, max_seq, -1), "bscale": obs.reshape(n, max_seq),
          "nib": onb.reshape(n, max_seq, -1), "rscale": ors.reshape(n, max_seq)}
    Vp = {"words": vw.reshape(n, max_seq, -1), "bscale": vbs.reshape(n, max_seq),
          "nib": vnb.reshape(n, max_seq, -1), "rscale": vrs.reshape(n, max_seq)}
    want = O.attention(qs[-1].reshape(-1, d).numpy(), Kp, Vp, H // Hkv, max_seq, max_seq, True)
    close(got.view(-1, d), want.view(np.float16).astype(np.float32), "BitCache.step vs oracle")


def test_bitcache_step_with_pinned_host_operands(cuda):
    """Q, K, V and the output in pinned host memory (read and written by the
    kernel directly) give the same result and cache as device tensors."""
    B, H, Hkv, d, max_seq = 2, 8, 4, 128, 300
    g = torch.Generator().manual_seed(23)
    a = BitCache(B, H, d, max_seq=max_seq, n_kv_heads=Hkv)
    b = BitCache(B, H, d, max_seq=max_seq, n_kv_heads=Hkv)
    pre_k = (torch.randn(B, Hkv, 200, d, generator=g) * 0.5).half().to(cuda)
    pre_v = (torch.randn(B, Hkv, 200, d, generator=g) * 0.5).half().to(cuda)
    a.prefill(pre_k, pre_v)
    b.prefill(pre_k, pre_v)
    qh = torch.empty(B, H, d, dtype=torch.float16).pin_memory()
    kh = torch.empty(B, Hkv, d, dtype=torch.float16).pin_memory()
    vh = torch.empty(B, Hkv, d, dtype=torch.float16).pin_memory()
    oh = torch.empty(B, H, d, dtype=torch.float16).pin_memory()
    for t in range(5):
        qh.copy_((torch.randn(B, H, d, generator=g) * 0.5).half())
        kh.copy_((torch.randn(B, Hkv, d, generator=g) * 0.5).half())
        vh.copy_((torch.randn(B, Hkv, d, generator=g) * 0.5).half())
        got = a.step(qh, kh, vh, out=oh)
        want = b.step(qh.to(cuda), kh.to(cuda), vh.to(cuda))
        torch.cuda.synchronize()
        assert got.data_ptr() == oh.data_ptr() and not got.is_cuda
        assert torch.equal(got, want.cpu())
    for X, Y in zip(a.planes, b.planes):
        planes_equal(X, Y, 205, True)


def test_step_mixed_host_and_device_rows_wait_for_the_previous_kernel(cuda):
    """new_k in pinned host memory, new_v a device tensor written by the
    kernel queued just ahead (a decode whose output is that tensor).  The step
    may read host-resident rows before it waits for the previous kernel, but
    only when both rows are host-resident: here new_v must be read after the
    previous decode has written it.  The result equals the same step run after
    a full synchronisation."""
    d, slots, S0 = 128, 8, 3000
    g = torch.Generator().manual_seed(31)
    big = [(torch.randn(slots, 32768, d, generator=g) * 0.5).half().to(cuda) for _ in range(2)]
    Kb = planes.Planes.empty(slots, 32768, d, True, cuda)
    Vb = planes.Planes.empty(slots, 32768, d, True, cuda)
    planes.encode_planes(big[0], Kb)
    planes.encode_planes(big[1], Vb)
    qb = (torch.randn(slots, d, generator=g) * 0.5).half().to(cuda)
    (Ka, Va), (Kc, Vc) = filled_pair(slots, 4096, d, True, S0, cuda, seed=32)
    q = (torch.randn(slots, d, generator=g) * 0.5).half().to(cuda)
    kh = (torch.randn(slots, d, generator=g) * 0.5).half().pin_memory()
    for trial in range(3):
        vdev = torch.zeros(slots, d, dtype=torch.float16, device=cuda)
        torch.cuda.synchronize()
        planes.decode_attention(qb, Kb, Vb, 32768, out=vdev)  # writes new_v in its final epilogue
        got = planes.decode_step(q, kh, vdev, Ka, Va, S0 + 1, S0)
        torch.cuda.synchronize()
        want = planes.decode_step(q, kh.to(cuda), vdev.clone(), Kc, Vc, S0 + 1, S0)
        torch.cuda.synchronize()
        assert vdev.abs().sum() > 0
        assert torch.equal(got, want), f"trial {trial}: the step read new_v before the previous kernel wrote it"
        planes_equal(Ka, Kc, S0 + 1, True)
        planes_equal(Va, Vc, S0 + 1, True)


def test_stage_rows_copies_host_segments(cuda):
    """bc_stage_rows copies pinned host segments to device memory exactly, with
    the sources read ahead of the previous kernel and written after it."""
    g = torch.Generator().manual_seed(41)
    srcs = [torch.randint(0, 256, (n,), generator=g, dtype=torch.uint8).pin_memory() for n in (4096, 16, 80000)]
    dsts = [torch.zeros(s.numel(), dtype=torch.uint8, device=cuda) for s in srcs]
    # a long kernel ahead in the stream that also writes the destinations: the
    # staged values must land after it
    for d in dsts:
        d.fill_(7)
    torch.cuda._sleep(1_000_000)
    for d in dsts:
        d.fill_(9)
    planes.stage_rows(list(zip(srcs, dsts)))
    torch.cuda.synchronize()
    for s, d in zip(srcs, dsts):
        assert torch.equal(d.cpu(), s)
