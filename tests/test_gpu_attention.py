"""GPU: decode attention (record drop-ins and the fused plane kernel), scores,
entropy and BitCache against the reference's own kernels and the C oracle.
Tolerance for fp outputs: max-abs 2e-3 and cosine >= 0.9999."""
import numpy as np
import pytest
import torch

import cases
from bitcache_b200 import BitCache, _C, _lib, functional, planes, workloads
from oracle import oracle as O
from oracle import refgpu

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-3
MIN_COS = 0.9999


def close(got, want, label=""):
    g = got.float().cpu().numpy().astype(np.float64).ravel()
    w = want.float().cpu().numpy().astype(np.float64).ravel() if torch.is_tensor(want) else want.astype(np.float64).ravel()
    err = np.max(np.abs(g - w)) if g.size else 0.0
    cos = float(g @ w / (np.linalg.norm(g) * np.linalg.norm(w) + 1e-30)) if g.size else 1.0
    assert err <= MAX_ABS, f"{label}: max-abs {err:.3g}"
    if np.linalg.norm(w) > 1e-6:
        assert cos >= MIN_COS, f"{label}: cosine {cos:.6f}"


def records(k, v):
    kb = _C.binary_encode(k)
    kr = _C.residual_encode(k, kb)
    vb = _C.binary_encode(v)
    vr = _C.residual_encode(v, vb)
    return kb, kr, vb, vr


SMALL = [(1, 8, 1024, 128), (2, 3, 300, 64), (1, 2, 77, 256), (1, 4, 513, 32), (3, 1, 4096, 128), (1, 1, 1, 128)]


@pytest.mark.parametrize("B,H,S,d", SMALL)
@pytest.mark.parametrize("comp", [False, True])
def test_record_attention_vs_reference(cuda, B, H, S, d, comp):
    g = torch.Generator().manual_seed(B * 1000 + S + d)
    q = (torch.randn(B, H, d, generator=g) * 0.5).half().to(cuda)
    k = (torch.randn(B * H * S, d, generator=g) * 0.5).half().to(cuda)
    v = (torch.randn(B * H * S, d, generator=g) * 0.5).half().to(cuda)
    kb, kr, vb, vr = records(k, v)
    if comp:
        mine = functional.compensated_attention(q, kb, kr, vb, vr, B, H, S, d)
        ref = refgpu.attention(q.view(B * H, d), kb, vb, kr, vr, B, H, S, d)
    else:
        mine = functional.binary_attention(q, kb, vb, B, H, S, d)
        ref = refgpu.attention(q.view(B * H, d), kb, vb, None, None, B, H, S, d)
    close(mine.view(B * H, d), ref, f"records B{B} H{H} S{S} d{d} comp={comp}")


@pytest.mark.parametrize("B,H,S,d", SMALL)
@pytest.mark.parametrize("comp", [False, True])
def test_plane_attention_vs_reference(cuda, B, H, S, d, comp):
    g = torch.Generator().manual_seed(7 * B + S + d)
    q = (torch.randn(B * H, d, generator=g) * 0.5).half().to(cuda)
    k = (torch.randn(B * H, S, d, generator=g) * 0.5).half().to(cuda)
    v = (torch.randn(B * H, S, d, generator=g) * 0.5).half().to(cuda)
    stride = planes.round_stride(S) + 16
    K = planes.Planes.empty(B * H, stride, d, True, cuda)
    V = planes.Planes.empty(B * H, stride, d, True, cuda)
    planes.encode_planes(k, K, planes.RES_FP16_SCALE)
    planes.encode_planes(v, V, planes.RES_FP16_SCALE)
    mode = planes.MODE_COMPENSATED if comp else planes.MODE_BINARY
    mine = planes.decode_attention(q, K, V, S, mode)
    kb, kr, vb, vr = records(k.view(-1, d), v.view(-1, d))
    ref = refgpu.attention(q, kb, vb, kr if comp else None, vr if comp else None, B, H, S, d)
    close(mine, ref, f"planes B{B} H{H} S{S} d{d} comp={comp}")


def test_c1_golden_vs_kernels(cuda):
    """The committed reference outputs of config C1 are reproduced by both kernels."""
    fx = cases.load_fixture("c1")
    q, k, v = cases.attn_inputs("c1")
    b, h, s, d, _, _ = cases.ATTN_CASES["c1"]
    kb, kr, vb, vr = records(k.to(cuda), v.to(cuda))
    assert np.array_equal(O.split_binvec(kb.cpu().numpy(), d)[0], fx["k_words"])
    assert np.array_equal(O.split_resvec(vr.cpu().numpy(), d)[0], fx["v_nib"])
    out = functional.compensated_attention(q.view(b, h, d).to(cuda), kb, kr, vb, vr, b, h, s, d)
    close(out.view(b * h, d), fx["comp_out"].view(np.float16).astype(np.float32), "c1 golden")


@pytest.mark.parametrize("group", [2, 4, 8])
@pytest.mark.parametrize("d", [32, 64, 128, 256])
@pytest.mark.parametrize("comp", [True, False])
def test_gqa_vs_oracle(cuda, group, d, comp):
    """Grouped-query heads, several per CTA: the tensor-core value phase (heads as
    MMA columns) for compensated caches at d = 64, 128, 256 and binary ones at
    d = 128; 16-dim f32x2 value lanes elsewhere."""
    slots, S = 3, 700
    g = torch.Generator().manual_seed(group * 10 + d)
    q = (torch.randn(slots * group, d, generator=g) * 0.5).half()
    k = (torch.randn(slots, S, d, generator=g) * 0.5).half()
    v = (torch.randn(slots, S, d, generator=g) * 0.5).half()
    stride = planes.round_stride(S)
    K = planes.Planes.empty(slots, stride, d, True, cuda)
    V = planes.Planes.empty(slots, stride, d, True, cuda)
    planes.encode_planes(k.to(cuda), K, planes.RES_FP16_SCALE)
    planes.encode_planes(v.to(cuda), V, planes.RES_FP16_SCALE)
    mode = planes.MODE_COMPENSATED if comp else planes.MODE_BINARY
    mine = planes.decode_attention(q.to(cuda), K, V, S, mode)

    def host(X):
        return {"words": X.sign.cpu().numpy().view(np.uint32), "bscale": X.bscale.cpu().numpy().view(np.uint16),
                "nib": X.nib_rows().cpu().numpy(), "rscale": X.rscale.cpu().numpy().view(np.uint16)}

    want = O.attention(q.numpy(), host(K), host(V), group, S, stride, comp).view(np.float16).astype(np.float32)
    close(mine, want, f"gqa g={group} d={d} comp={comp}")


@pytest.mark.parametrize("pattern", ["score_ramp", "value_jump"])
@pytest.mark.parametrize("group", [1, 2])
@pytest.mark.parametrize("d", [64, 128, 256])
def test_growing_coefficients_vs_oracle(cuda, pattern, group, d):
    """Key coefficients that grow within a split: the tensor-core value phase
    must move its fixed-point unit and shift the accumulators down exactly.
    score_ramp: scores rise by ~30 log2 units over every 256 positions (a
    sawtooth, so every period's top keys carry equal weight); value_jump: the
    first half of every period holds values 2^12 times smaller."""
    slots, S = 32, 8192
    g = torch.Generator().manual_seed(5 + group + d)
    q = (torch.randn(slots * group, d, generator=g) * 0.5).half()
    pos = torch.arange(S, dtype=torch.float32)
    phase = (pos % 256) / 256.0
    k = torch.randn(slots, S, d, generator=g) * 0.3
    v = torch.randn(slots, S, d, generator=g) * 0.5
    if pattern == "score_ramp":
        k += (8.0 * phase)[None, :, None] * q.float().view(slots, group, d)[:, 0][:, None, :]
    else:
        v *= torch.where(phase < 0.5, 2.0 ** -12, 1.0)[None, :, None]
    k, v = k.half(), v.half()
    K = planes.Planes.empty(slots, S, d, True, cuda)
    V = planes.Planes.empty(slots, S, d, True, cuda)
    planes.encode_planes(k.to(cuda), K, planes.RES_FP32_SCALE)
    planes.encode_planes(v.to(cuda), V, planes.RES_FP32_SCALE)
    mine = planes.decode_attention(q.to(cuda), K, V, S)

    def host(X):
        return {"words": X.sign.cpu().numpy().view(np.uint32), "bscale": X.bscale.cpu().numpy().view(np.uint16),
                "nib": X.nib_rows().cpu().numpy(), "rscale": X.rscale.cpu().numpy().view(np.uint16)}

    want = O.attention(q.numpy(), host(K), host(V), group, S, S, True).view(np.float16).astype(np.float32)
    close(mine, want, f"{pattern} group={group} d={d}")


@pytest.mark.parametrize("S", [0, 1, 7, 8, 9, 129, 1000])
def test_seq_len_edges_and_masking(cuda, S):
    """Positions past seq_len hold garbage and must not contribute; seq_len 0 gives zeros."""
    d, slots = 128, 2
    stride = planes.round_stride(max(S, 1)) + 32
    g = torch.Generator().manual_seed(S + 1)
    full = (torch.randn(slots, stride, d, generator=g) * 0.5).half().to(cuda)
    vfull = (torch.randn(slots, stride, d, generator=g) * 3.0).half().to(cuda)
    K = planes.Planes.empty(slots, stride, d, True, cuda)
    V = planes.Planes.empty(slots, stride, d, True, cuda)
    planes.encode_planes(full, K, planes.RES_FP16_SCALE)
    planes.encode_planes(vfull, V, planes.RES_FP16_SCALE)
    q = (torch.randn(slots, d, generator=g) * 0.5).half().to(cuda)
    out = planes.decode_attention(q, K, V, S)
    if S == 0:
        assert not out.any()
        return
    kb, kr, vb, vr = records(full[:, :S].reshape(-1, d).contiguous(), vfull[:, :S].reshape(-1, d).contiguous())
    ref = refgpu.attention(q, kb, vb, kr, vr, 1, slots, S, d)
    close(out, ref, f"S={S}")


def test_c3_full_size_vs_reference(cuda):
    """Headline shape (S=65536, H=32, d=128, outlier channels) against the reference kernel."""
    w = workloads.make("C3", device=cuda)
    S, d, H = w.seq_len, w.head_dim, w.n_heads
    K = planes.Planes.empty(H, S, d, True, cuda)
    V = planes.Planes.empty(H, S, d, True, cuda)
    planes.encode_planes(w.k.view(H, S, d), K, planes.RES_FP16_SCALE)
    planes.encode_planes(w.v.view(H, S, d), V, planes.RES_FP16_SCALE)
    q = w.q.view(H, d)
    mine = planes.decode_attention(q, K, V, S)
    kb, kr, vb, vr = records(w.k.view(-1, d), w.v.view(-1, d))
    ref = refgpu.attention(q, kb, vb, kr, vr, 1, H, S, d)
    close(mine, ref, "C3 planes")
    rec = functional.compensated_attention(w.q, kb, kr, vb, vr, 1, H, S, d)
    close(rec.view(H, d), ref, "C3 records")
    # sequence split property: two halves merged == whole
    half = S // 2
    parts = torch.empty(2, H, d + 2, dtype=torch.float32, device=cuda)
    Kh = [planes.Planes(K.sign[:, a:b].contiguous(), K.bscale[:, a:b].contiguous(), K.nib[:, a:b].contiguous(),
                        K.rscale[:, a:b].contiguous(), d) for a, b in ((0, half), (half, S))]
    Vh = [planes.Planes(V.sign[:, a:b].contiguous(), V.bscale[:, a:b].contiguous(), V.nib[:, a:b].contiguous(),
                        V.rscale[:, a:b].contiguous(), d) for a, b in ((0, half), (half, S))]
    for i in range(2):
        planes.decode_attention(q, Kh[i], Vh[i], half, partial=parts[i], want_out=False)
    merged = planes.lse_merge(parts)
    close(merged, mine, "C3 split-merge")


def test_partial_output_consistent(cuda):
    d, slots, S = 128, 4, 3000
    g = torch.Generator().manual_seed(3)
    k = (torch.randn(slots, S, d, generator=g) * 0.5).half().to(cuda)
    v = (torch.randn(slots, S, d, generator=g) * 0.5).half().to(cuda)
    q = (torch.randn(slots, d, generator=g) * 0.5).half().to(cuda)
    K = planes.Planes.empty(slots, planes.round_stride(S), d, True, cuda)
    V = planes.Planes.empty(slots, planes.round_stride(S), d, True, cuda)
    planes.encode_planes(k, K)
    planes.encode_planes(v, V)
    part = torch.zeros(slots, d + 2, dtype=torch.float32, device=cuda)
    out = planes.decode_attention(q, K, V, S, partial=part)
    o2 = (part[:, 2:] / part[:, 1:2]).half()
    close(o2, out, "partial vs out")
    merged = planes.lse_merge(part[None])
    close(merged, out, "merge of one part")


@pytest.mark.parametrize("d", [64, 128, 256])
def test_popcount_scores_exact(cuda, d):
    slots, S, group = 2, 333, 2
    g = torch.Generator().manual_seed(d)
    q = (torch.randn(slots * group, d, generator=g)).half()
    k = (torch.randn(slots, S, d, generator=g)).half()
    K = planes.Planes.empty(slots, planes.round_stride(S), d, False, cuda)
    planes.encode_planes(k.to(cuda), K, planes.RES_NONE)
    got = planes.xnor_popcount(q.to(cuda), K, S).cpu().numpy()
    words = K.sign.cpu().numpy().view(np.uint32)
    for h in range(slots * group):
        want = O.xnor_popcount(q[h].numpy(), words[h // group, :S])
        assert np.array_equal(got[h], want)


@pytest.mark.parametrize("B,H,S,d", [(1, 8, 1024, 128), (2, 3, 300, 64), (1, 2, 77, 256)])
def test_entropy_and_select_vs_reference(cuda, B, H, S, d):
    g = torch.Generator().manual_seed(S)
    q = (torch.randn(B, H, d, generator=g) * 0.5).half().to(cuda)
    k = (torch.randn(B * H * S, d, generator=g) * 0.5).half().to(cuda)
    kb = _C.binary_encode(k)
    mine = _C.compute_head_entropy(q, kb, B, H, S, d)
    ref = refgpu.head_entropy(q.view(-1, d), kb, B, H, S, d)
    torch.testing.assert_close(mine.view(-1), ref, rtol=1e-4, atol=1e-4)
    K = planes.Planes.empty(B * H, planes.round_stride(S), d, False, cuda)
    planes.encode_planes(k.view(B * H, S, d), K, planes.RES_NONE)
    torch.testing.assert_close(planes.head_entropy(q.view(-1, d), K, S), ref, rtol=1e-4, atol=1e-4)
    thr = float(ref.median())
    assert torch.equal(_C.adaptive_select(ref, thr), refgpu.adaptive_select(ref, thr))


def test_bitcache_decode_loop_vs_reference(cuda):
    """BitCache.append/attend against the reference functional path on a full ring."""
    B, H, d, S = 2, 4, 128, 96
    g = torch.Generator().manual_seed(11)
    toks_k = (torch.randn(S, B, H, d, generator=g) * 0.5).half().to(cuda)
    toks_v = (torch.randn(S, B, H, d, generator=g) * 0.5).half().to(cuda)
    cache = BitCache(B, H, d, max_seq=S, device="cuda", compensated=True)
    rb = torch.zeros(B * H * S * 36, dtype=torch.uint8, device=cuda)
    rr = torch.zeros(B * H * S * 130, dtype=torch.uint8, device=cuda)
    vb = torch.zeros_like(rb)
    vr = torch.zeros_like(rr)
    for t in range(S):
        cache.append(toks_k[t], toks_v[t])
        refgpu.online_encode_token(toks_k[t], rb, rr, B, H, d, t, S)
        refgpu.online_encode_token(toks_v[t], vb, vr, B, H, d, t, S)
    q = (torch.randn(B, H, d, generator=g) * 0.5).half().to(cuda)
    mine = cache.attend(q)
    ref = refgpu.attention(q.view(-1, d), rb, vb, rr, vr, B, H, S, d)
    close(mine.view(-1, d), ref, "BitCache")
    assert cache.seq_len == S


def test_bitcache_ring_wrap_and_binary_mode(cuda):
    B, H, d, max_seq, steps = 1, 2, 64, 16, 40
    g = torch.Generator().manual_seed(5)
    ks = (torch.randn(steps, B, H, d, generator=g) * 0.5).half()
    vs = (torch.randn(steps, B, H, d, generator=g) * 0.5).half()
    for comp in (True, False):
        cache = BitCache(B, H, d, max_seq=max_seq, compensated=comp)
        for t in range(steps):
            cache.append(ks[t].to(cuda), vs[t].to(cuda))
        q = (torch.randn(B, H, d, generator=g) * 0.5).half()
        got = cache.attend(q.to(cuda)).view(-1, d)
        # last max_seq tokens, any order
        kk = ks[steps - max_seq:].permute(1, 2, 0, 3).reshape(-1, d)
        vv = vs[steps - max_seq:].permute(1, 2, 0, 3).reshape(-1, d)
        w, s = O.online_encode(kk.numpy())[:2]
        nb, rs = O.online_encode(kk.numpy())[2:4]
        vw, vsc, vnb, vrs, _ = O.online_encode(vv.numpy())
        Kp = {"words": w.reshape(B * H, max_seq, -1), "bscale": s.reshape(B * H, max_seq),
              "nib": nb.reshape(B * H, max_seq, -1), "rscale": rs.reshape(B * H, max_seq)}
        Vp = {"words": vw.reshape(B * H, max_seq, -1), "bscale": vsc.reshape(B * H, max_seq),
              "nib": vnb.reshape(B * H, max_seq, -1), "rscale": vrs.reshape(B * H, max_seq)}
        want = O.attention(q.view(-1, d).numpy(), Kp, Vp, 1, max_seq, max_seq, comp)
        close(got, want.view(np.float16).astype(np.float32), f"ring comp={comp}")
        assert cache.seq_len == max_seq


def test_bitcache_prefill_then_decode(cuda):
    w = workloads.make("C4", batch=2, seq_len=512, steps=3)
    cache = BitCache(w.batch, w.n_heads, w.head_dim, max_seq=600, n_kv_heads=w.n_kv_heads)
    cache.prefill(w.k.to(cuda), w.v.to(cuda))
    for t in range(3):
        cache.append(w.extra["k_new"][t].to(cuda), w.extra["v_new"][t].to(cuda))
    out = cache.attend(w.q.to(cuda))
    kk = torch.cat([w.k, w.extra["k_new"].permute(1, 2, 0, 3)], 2).reshape(-1, w.head_dim)
    vv = torch.cat([w.v, w.extra["v_new"].permute(1, 2, 0, 3)], 2).reshape(-1, w.head_dim)
    S = 515
    ow, obs, onb, ors, _ = O.online_encode(kk.numpy())
    vw, vbs, vnb, vrs, _ = O.online_encode(vv.numpy())
    n = w.batch * w.n_kv_heads
    Kp = {"words": ow.reshape(n, S, -1), "bscale": obs.reshape(n, S), "nib": onb.reshape(n, S, -1),
          "rscale": ors.reshape(n, S)}
    Vp = {"words": vw.reshape(n, S, -1), "bscale": vbs.reshape(n, S), "nib": vnb.reshape(n, S, -1),
          "rscale": vrs.reshape(n, S)}
    want = O.attention(w.q.reshape(-1, w.head_dim).numpy(), Kp, Vp, w.group, S, S, True)
    close(out.view(-1, w.head_dim), want.view(np.float16).astype(np.float32), "prefill+decode GQA")


@pytest.mark.parametrize("slots,group", [(32, 1), (3, 4), (5, 8)])
def test_workspace_counters_left_zero_and_no_device_error(cuda, slots, group):
    d, S = 128, 2048
    g = torch.Generator().manual_seed(slots)
    K = planes.Planes.empty(slots, S, d, True, cuda)
    V = planes.Planes.empty(slots, S, d, True, cuda)
    planes.encode_planes((torch.randn(slots, S, d, generator=g) * 0.1).half().to(cuda), K)
    planes.encode_planes((torch.randn(slots, S, d, generator=g) * 0.1).half().to(cuda), V)
    q = (torch.randn(slots * group, d, generator=g) * 0.1).half().to(cuda)
    first = planes.decode_attention(q, K, V, S)
    for _ in range(3):  # reuse of the same workspace gives the same answer
        assert torch.equal(planes.decode_attention(q, K, V, S), first)
    torch.cuda.synchronize()
    key = (cuda.index or 0, _lib.stream_of(cuda), "decode", slots, group)
    n_cnt = slots * group  # upper bound of the counter region (one head per CTA)
    assert not _lib._ws[key][: 4 * n_cnt].any(), "split-K ticket counters not returned to zero"
    assert _lib.device_error() == 0


@pytest.mark.parametrize("slots,group,S,d,comp", [
    (8, 1, 1024, 128, True),      # C1 shape
    (32, 1, 4096, 128, True),     # several splits per slot
    (3, 4, 700, 64, True),        # grouped-query heads
    (2, 8, 333, 128, False),
    (4, 1, 1, 256, True),
    (5, 2, 2049, 32, False),
])
def test_fused_entropy_matches_reference(cuda, slots, group, S, d, comp):
    """Entropy computed inside the attention pass equals the reference's
    compute_head_entropy (its own kernel, on records) and the attention output
    equals the plain kernel's."""
    g = torch.Generator().manual_seed(S + d + group)
    q = (torch.randn(slots * group, d, generator=g) * 0.5).half().to(cuda)
    k = (torch.randn(slots, S, d, generator=g) * 0.5).half().to(cuda)
    v = (torch.randn(slots, S, d, generator=g) * 0.5).half().to(cuda)
    stride = planes.round_stride(S)
    K = planes.Planes.empty(slots, stride, d, True, cuda)
    V = planes.Planes.empty(slots, stride, d, True, cuda)
    planes.encode_planes(k, K, planes.RES_FP16_SCALE)
    planes.encode_planes(v, V, planes.RES_FP16_SCALE)
    mode = planes.MODE_COMPENSATED if comp else planes.MODE_BINARY
    out, ent = planes.decode_attention_entropy(q, K, V, S, mode)
    plain = planes.decode_attention(q, K, V, S, mode)
    # reference kernel: one record row per query head (the KV slot repeated for the group)
    kb = _C.binary_encode(k.repeat_interleave(group, 0).reshape(-1, d).contiguous())
    ref = refgpu.head_entropy(q, kb, 1, slots * group, S, d)
    torch.cuda.synchronize()
    torch.testing.assert_close(ent, ref, rtol=1e-4, atol=1e-4)
    close(out, plain, f"entropy variant output slots={slots} g={group}")


@pytest.mark.parametrize("slots,group,S", [(32, 1, 4096), (3, 4, 700), (2, 1, 100)])
def test_peer_exchange_single_rank_equals_decode(cuda, slots, group, S):
    """The fused exchange path on one rank (the buffer is its own; flags go to
    itself) gives the plain decode's output, step after step."""
    from bitcache_b200 import dist as bdist

    d = 128
    g = torch.Generator().manual_seed(S + group)
    K = planes.Planes.empty(slots, planes.round_stride(S), d, True, cuda)
    V = planes.Planes.empty(slots, planes.round_stride(S), d, True, cuda)
    planes.encode_planes((torch.randn(slots, S, d, generator=g) * 0.5).half().to(cuda), K)
    planes.encode_planes((torch.randn(slots, S, d, generator=g) * 0.5).half().to(cuda), V)
    x = bdist.PeerExchange(slots * group, d)
    try:
        for step in range(4):
            q = (torch.randn(slots * group, d, generator=g) * 0.5).half().to(cuda)
            got = x.decode(q, K, V, S, planes.MODE_COMPENSATED)
            want = planes.decode_attention(q, K, V, S)
            torch.cuda.synchronize()
            close(got, want, f"xchg step {step}")
        assert _lib.device_error() == 0
    finally:
        x.close()
