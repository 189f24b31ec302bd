"""GPU: parity at the full BASELINE configurations C2, C4 and C5, against the
reference's own kernels (oracle/_ref, compiled from the reference sources) on
the same seeded inputs, and the reference's own quality gate through BitCache.

* Encodings (sign words, INT4 codes, both scales) are compared bit for bit
  with the reference encoders.
* Attention outputs must stay within max-abs 2e-3 and cosine >= 0.9999 of the
  reference's compensated_attention kernel.

The reference kernels have no grouped-query heads, so for C4 every KV slot's
records are repeated for the query heads of its group.
"""
import math

import numpy as np
import pytest
import torch

from bitcache_b200 import BitCache, _lib, planes, workloads
from oracle import oracle as O
from oracle import refgpu

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-3
MIN_COS = 0.9999
BIN, RES = 36, 130  # reference record sizes (binary_encode.cuh:13-18, residual.cuh:11-16)


def close(got, want, label=""):
    g = got.float().flatten().double()
    w = want.float().flatten().double().to(g.device)
    err = float((g - w).abs().max()) if g.numel() else 0.0
    cos = float(g @ w / (g.norm() * w.norm() + 1e-30)) if g.numel() else 1.0
    assert err <= MAX_ABS, f"{label}: max-abs {err:.3g}"
    if float(w.norm()) > 1e-6:
        assert cos >= MIN_COS, f"{label}: cosine {cos:.6f}"


def planes_equal_records(P, kb, kr, n_vecs, d, label):
    """Every field of the planes (flat, first n_vecs rows) equals the reference records."""
    rb, rr = planes.planes_to_records(P, n_vecs)
    nw = d // 32
    a = rb.view(n_vecs, BIN)
    b = kb.view(n_vecs, BIN)
    assert torch.equal(a[:, :4 * nw], b[:, :4 * nw]), f"{label}: sign words differ"
    assert torch.equal(a[:, 32:34], b[:, 32:34]), f"{label}: binary scales differ"
    if kr is not None:
        a = rr.view(n_vecs, RES)
        b = kr.view(n_vecs, RES)
        assert torch.equal(a[:, :d // 2], b[:, :d // 2]), f"{label}: INT4 codes differ"
        assert torch.equal(a[:, 128:130], b[:, 128:130]), f"{label}: residual scales differ"


def rows(blob, n, per):
    return blob.view(n, -1, per)


# ---------------------------------------------------------------------------
# C2: B=1, H=32, S=4096, d=128, 32 keys per head correlated 0.25 with Q
# ---------------------------------------------------------------------------
def test_c2_full_config(cuda):
    w = workloads.make("C2", device=cuda)
    n, S, d = w.n_slots, w.seq_len, w.head_dim
    k, v, q = w.k.reshape(n * S, d), w.v.reshape(n * S, d), w.q.reshape(n, d)
    kb, vb = refgpu.binary_encode(k), refgpu.binary_encode(v)
    kr, vr = refgpu.residual_encode(k, kb), refgpu.residual_encode(v, vb)
    K = planes.Planes.empty(n, S, d, True, cuda)
    V = planes.Planes.empty(n, S, d, True, cuda)
    planes.encode_planes(w.k.reshape(n, S, d), K, planes.RES_FP16_SCALE)
    planes.encode_planes(w.v.reshape(n, S, d), V, planes.RES_FP16_SCALE)
    planes_equal_records(K, kb, kr, n * S, d, "C2 K")
    planes_equal_records(V, vb, vr, n * S, d, "C2 V")
    want = refgpu.attention(q, kb, vb, kr, vr, 1, n, S, d)
    close(planes.decode_attention(q, K, V, S), want, "C2 compensated")
    want_b = refgpu.attention(q, kb, vb, None, None, 1, n, S, d)
    close(planes.decode_attention(q, K, V, S, planes.MODE_BINARY), want_b, "C2 binary")
    assert _lib.device_error() == 0


# ---------------------------------------------------------------------------
# C4: B=16, Hq=32, Hkv=8, S=32768 prefilled, then 64 steps of append + attend
# ---------------------------------------------------------------------------
def _ref_online_records(x, n, per_slot, max_seq, d):
    """The reference's online_encode_token arithmetic (residual against the fp32
    scale, online_encode.cu:56-119) for x [n, per_slot, d], placed at record
    slot*max_seq + p.  One launch encodes every vector: the kernel is given one
    "head" per vector and max_seq 1, so vector i lands at record i."""
    m = n * per_slot
    tb = torch.zeros(m * BIN, dtype=torch.uint8, device=x.device)
    tr = torch.zeros(m * RES, dtype=torch.uint8, device=x.device)
    refgpu.online_encode_token(x.reshape(m, d).contiguous(), tb, tr, 1, m, d, 0, 1)
    kb = torch.zeros(n * max_seq * BIN, dtype=torch.uint8, device=x.device)
    kr = torch.zeros(n * max_seq * RES, dtype=torch.uint8, device=x.device)
    rows(kb, n, BIN)[:, :per_slot] = rows(tb, n, BIN)
    rows(kr, n, RES)[:, :per_slot] = rows(tr, n, RES)
    return kb, kr


def _ref_attention_gqa(q, kb, vb, kr, vr, n, G, stride, seq_len, d):
    """Reference compensated attention over positions [0, seq_len) of records laid
    out [n][stride]; each slot's records repeated for its G query heads."""
    def rep(blob, per):
        return rows(blob, n, per)[:, :seq_len].repeat_interleave(G, 0).contiguous().view(-1)

    return refgpu.attention(q, rep(kb, BIN), rep(vb, BIN), rep(kr, RES), rep(vr, RES), 1, n * G, seq_len, d)


def test_c4_full_config_64_steps(cuda):
    """Prefill S=32768, then all 64 BitCache.step calls (the fused append +
    attend launch).  The final cache is bit-exact against 64 launches of the
    reference's online_encode_token; the first and last steps' outputs, and a
    plain decode over the final cache (the multi-wave split plan this shape
    selects), match the reference kernel."""
    w = workloads.make("C4", device=cuda)
    B, H, Hkv, S, d, G = w.batch, w.n_heads, w.n_kv_heads, w.seq_len, w.head_dim, w.group
    n, steps = w.n_slots, w.extra["steps"]
    max_seq = S + steps
    q = w.q.reshape(B, H, d)
    cache = BitCache(B, H, d, max_seq=max_seq, n_kv_heads=Hkv)
    cache.prefill(w.k, w.v)
    outs = {}
    for t in range(steps):
        o = cache.step(q, w.extra["k_new"][t], w.extra["v_new"][t])
        if t in (0, steps - 1):
            outs[t] = o.clone()
    assert cache.seq_len == max_seq
    # reference: the prefill through online_encode_token, then one launch per step
    kb, kr = _ref_online_records(w.k.reshape(n, S, d), n, S, max_seq, d)
    vb, vr = _ref_online_records(w.v.reshape(n, S, d), n, S, max_seq, d)
    del w.k, w.v
    torch.cuda.empty_cache()
    wants = {}
    for t in range(steps):
        refgpu.online_encode_token(w.extra["k_new"][t].reshape(n, d), kb, kr, B, Hkv, d, S + t, max_seq)
        refgpu.online_encode_token(w.extra["v_new"][t].reshape(n, d), vb, vr, B, Hkv, d, S + t, max_seq)
        if t == 0:
            wants[0] = _ref_attention_gqa(q.reshape(-1, d), kb, vb, kr, vr, n, G, max_seq, S + 1, d)
    Kp, Vp = cache.planes
    assert Kp.kv_stride == max_seq
    planes_equal_records(Kp, kb, kr, n * max_seq, d, "C4 K after 64 steps")
    planes_equal_records(Vp, vb, vr, n * max_seq, d, "C4 V after 64 steps")
    wants[steps - 1] = _ref_attention_gqa(q.reshape(-1, d), kb, vb, kr, vr, n, G, max_seq, max_seq, d)
    close(outs[0].reshape(-1, d), wants[0], "C4 step 0")
    close(outs[steps - 1].reshape(-1, d), wants[steps - 1], "C4 step 63")
    plain = planes.decode_attention(q.reshape(-1, d), Kp, Vp, max_seq)
    close(plain, wants[steps - 1], "C4 plain decode over the final cache")
    assert _lib.device_error() == 0


# ---------------------------------------------------------------------------
# C5: B=64, H=32, S=8192, d in {64, 128, 256}, Student-t K/V, 25% of residuals kept
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("d", [64, 128, 256])
def test_c5_full_config_adaptive(cuda, d):
    """Compact adaptive cache at the full C5 shape: encodings bit-exact against
    the reference encoders, the keep mask equal to the oracle's (on a sample of
    slots), and the output within tolerance of the reference's compensated
    kernel run on records whose unkept residuals are zeroed."""
    w = workloads.make("C5", device=cuda, head_dim=d)
    n, S = w.n_slots, w.seq_len
    k, v = w.k.reshape(n, S, d), w.v.reshape(n, S, d)
    q = w.q.reshape(n, d)
    K = planes.Planes.empty(n, S, d, True, cuda)
    V = planes.Planes.empty(n, S, d, True, cuda)
    planes.encode_planes(k, K, planes.RES_FP16_SCALE)
    planes.encode_planes(v, V, planes.RES_FP16_SCALE)
    kb, vb = refgpu.binary_encode(k.reshape(-1, d)), refgpu.binary_encode(v.reshape(-1, d))
    kr, vr = refgpu.residual_encode(k.reshape(-1, d), kb), refgpu.residual_encode(v.reshape(-1, d), vb)
    del w, k, v
    torch.cuda.empty_cache()
    planes_equal_records(K, kb, kr, n * S, d, f"C5 d={d} K")
    planes_equal_records(V, vb, vr, n * S, d, f"C5 d={d} V")
    n_keep = planes.keep_count(S, 0.25)
    keep = planes.select_positions_topk(K, V, S, n_keep)
    assert (keep[:, :S].sum(1) == n_keep).all()
    sample = list(range(0, n, 97))
    hk = {"nib": planes.nib_rows(K.nib[sample], d).cpu().numpy(), "rscale": K.rscale[sample].cpu().numpy()}
    hv = {"nib": planes.nib_rows(V.nib[sample], d).cpu().numpy(), "rscale": V.rscale[sample].cpu().numpy()}
    want_keep = O.select_positions_topk(hk["nib"], hk["rscale"].view(np.uint16), hv["nib"],
                                        hv["rscale"].view(np.uint16), S, n_keep)
    assert np.array_equal(keep[sample, :S].cpu().numpy(), want_keep)
    Kc, Vc = planes.compact_adaptive(K, V, keep, S, n_keep)
    got = planes.decode_attention_adaptive(q, Kc, Vc, S, n_keep)
    drop = (keep[:, :S] == 0).reshape(-1)
    for r in (kr, vr):
        r.view(n * S, RES)[drop] = 0  # code 0 and scale 0: the record contributes exactly nothing
    want = refgpu.attention(q, kb, vb, kr, vr, 1, n, S, d)
    close(got, want, f"C5 d={d} adaptive")
    assert _lib.device_error() == 0


# ---------------------------------------------------------------------------
# The reference's own quality gate (tests/test_python.py:63-179 of the
# reference), through BitCache.append / attend on the B200 kernels: decode
# simulation one token at a time; cosine against fp32 sdpa > 0.85 at every
# checkpoint, and compensated >= binary - 0.01.
#
# The same cosine is computed for the reference's own kernels on the same
# tokens, encoded into correct records by its online_encode_token, and ours
# must match it within 1e-3.  The 0.85 gate is asserted wherever the
# reference's kernels meet it.  They do not always: binary-only attention
# over 32 keys at head_dim 64 (the first checkpoint of the first config)
# measures about 0.79 with the reference kernels as with ours.  The
# reference's own BitCache in binary mode passes its binary blob as the
# residual cache (bitcache/__init__.py:104-111), so its 130-byte residual
# records are written at index*130 into a buffer of 36*max_seq bytes,
# beyond its end; its own run of this gate therefore measures corrupted
# records, not the algorithm.
# ---------------------------------------------------------------------------
def _sdpa(Q, K, V):
    return torch.nn.functional.scaled_dot_product_attention(
        Q.float().unsqueeze(2), K.float(), V.float(), scale=1.0 / math.sqrt(Q.shape[-1])).squeeze(2).half()


def _cos(a, b):
    a, b = a.float().flatten(), b.float().flatten()
    return float(a @ b / (a.norm() * b.norm() + 1e-12))


def _ref_cache_attend(Q, ks, vs, t, compensated):
    """The reference kernels over tokens ks[:t], vs[:t] ([batch, heads, d] each),
    encoded with the reference's online_encode_token into [batch*heads][t] records."""
    b, h, d = Q.shape
    n = b * h
    kb, kr = _ref_online_records(torch.stack(ks[:t], 2).reshape(n, t, d), n, t, t, d)
    vb, vr = _ref_online_records(torch.stack(vs[:t], 2).reshape(n, t, d), n, t, t, d)
    if not compensated:
        kr = vr = None
    return refgpu.attention(Q.reshape(n, d), kb, vb, kr, vr, b, h, t, d).view(b, h, d)


@pytest.mark.parametrize("batch,n_heads,head_dim,seq_len,compensated", [
    (1, 1, 64, 128, False),
    (1, 1, 64, 128, True),
    (1, 1, 128, 256, True),
    (1, 4, 128, 512, True),
    (2, 4, 64, 256, True),
    (1, 1, 128, 1024, True),
])
def test_reference_quality_gate_through_bitcache(cuda, batch, n_heads, head_dim, seq_len, compensated):
    torch.manual_seed(42 + seq_len + head_dim)
    cache = BitCache(batch, n_heads, head_dim, max_seq=seq_len + 8, device=str(cuda), compensated=compensated)
    ks, vs = [], []
    for _ in range(seq_len):
        kt = torch.randn(batch, n_heads, head_dim, device=cuda, dtype=torch.float16) * 0.5
        vt = torch.randn(batch, n_heads, head_dim, device=cuda, dtype=torch.float16) * 0.5
        cache.append(kt, vt)
        ks.append(kt)
        vs.append(vt)
    K_full, V_full = torch.stack(ks, 2), torch.stack(vs, 2)
    for t in sorted({seq_len // 4, seq_len // 2, seq_len}):
        Q = torch.randn(batch, n_heads, head_dim, device=cuda, dtype=torch.float16) * 0.5
        ref = _sdpa(Q, K_full[:, :, :t], V_full[:, :, :t])
        sub = BitCache(batch, n_heads, head_dim, max_seq=t + 4, device=str(cuda), compensated=compensated)
        for s in range(t):
            sub.append(ks[s], vs[s])
        cos = _cos(ref, sub.attend(Q))
        cos_ref = _cos(ref, _ref_cache_attend(Q, ks, vs, t, compensated))
        assert abs(cos - cos_ref) <= 1e-3, f"t={t}: cosine {cos:.4f}, reference kernels {cos_ref:.4f}"
        if cos_ref > 0.85:
            assert cos > 0.85, f"cosine {cos:.4f} below 0.85 at t={t}"
    if compensated:
        binc = BitCache(batch, n_heads, head_dim, max_seq=seq_len + 4, device=str(cuda), compensated=False)
        for s in range(seq_len):
            binc.append(ks[s], vs[s])
        Q = torch.randn(batch, n_heads, head_dim, device=cuda, dtype=torch.float16) * 0.5
        ref = _sdpa(Q, K_full, V_full)
        cos_bin, cos_comp = _cos(ref, binc.attend(Q)), _cos(ref, cache.attend(Q))
        assert cos_comp >= cos_bin - 0.01, f"compensated {cos_comp:.4f} below binary {cos_bin:.4f} - 0.01"
    assert _lib.device_error() == 0
