"""GPU: per-vector adaptive precision (keep the INT4 residual of the top
vectors by residual energy) against the C oracle: exact keep masks (ties to
the lower position), and compensated attention after the unselected
residuals are dropped."""
import numpy as np
import pytest
import torch

from bitcache_b200 import BitCache, planes, workloads
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def host(P):
    return {"words": P.sign.cpu().numpy().view(np.uint32), "bscale": P.bscale.cpu().numpy().view(np.uint16),
            "nib": P.nib_rows().cpu().numpy(), "rscale": P.rscale.cpu().numpy().view(np.uint16)}


def build(cuda, slots, S, stride, d, seed, dup=False):
    w = workloads.make("C5", batch=1, n_heads=slots, n_kv_heads=slots, seq_len=S, head_dim=d, seed=seed)
    k = w.k.reshape(slots, S, d).clone()
    if dup:  # repeated vectors give equal keys: exercises the tie rule
        k[:, S // 2:S // 2 + 20] = k[:, 3:4]
    P = planes.Planes.empty(slots, stride, d, True, cuda)
    planes.encode_planes(k.to(cuda), P)
    return P, w


@pytest.mark.parametrize("d", [64, 128, 256])
@pytest.mark.parametrize("frac", [0.0, 0.25, 0.5, 1.0])
def test_keep_mask_matches_oracle(cuda, d, frac):
    slots, S, stride = 3, 300, 320
    P, _ = build(cuda, slots, S, stride, d, seed=d, dup=True)
    n_keep = planes.keep_count(S, frac)
    h = host(P)
    keep = planes.select_residual_topk(P, S, n_keep, apply=False, want_mask=True).cpu().numpy()
    want = O.select_residual_topk(h["nib"], h["rscale"], S, n_keep)
    assert np.array_equal(keep[:, :S], want[:, :S])
    assert (keep[:, :S].sum(1) == n_keep).all()


def test_apply_then_attention_matches_oracle(cuda):
    slots, S, d, group = 4, 777, 128, 2
    P_k, w = build(cuda, slots, S, planes.round_stride(S), d, seed=1)
    P_v, _ = build(cuda, slots, S, planes.round_stride(S), d, seed=2)
    n_keep = planes.keep_count(S, 0.25)
    hk0, hv0 = host(P_k), host(P_v)
    mk = O.select_residual_topk(hk0["nib"], hk0["rscale"], S, n_keep).astype(bool)
    mv = O.select_residual_topk(hv0["nib"], hv0["rscale"], S, n_keep).astype(bool)
    planes.select_residual_topk(P_k, S, n_keep, apply=True)
    planes.select_residual_topk(P_v, S, n_keep, apply=True)
    for h0, m in ((hk0, mk), (hv0, mv)):
        h0["rscale"] = np.where(m, h0["rscale"], 0).astype(np.uint16)
        h0["nib"] = np.where(m[..., None], h0["nib"], 0).astype(np.uint8)
    hk, hv = host(P_k), host(P_v)
    assert np.array_equal(hk["rscale"][:, :S], hk0["rscale"][:, :S]) and np.array_equal(hk["nib"][:, :S], hk0["nib"][:, :S])
    g = torch.Generator().manual_seed(5)
    q = (torch.randn(slots * group, d, generator=g) / d ** 0.5).half()
    got = planes.decode_attention(q.to(cuda), P_k, P_v, S).float().cpu().numpy()
    want = O.attention(q.numpy(), hk0, hv0, group, S, P_k.kv_stride, True).view(np.float16).astype(np.float32)
    assert np.max(np.abs(got - want)) <= 2e-3
    assert float((got * want).sum() / (np.linalg.norm(got) * np.linalg.norm(want))) >= 0.9999


def test_bitcache_keep_residuals(cuda):
    """BitCache.keep_residuals keeps exactly the requested count per slot, and the
    adaptive output's quality against exact attention lies between binary-only and
    full compensated attention."""
    B, H, d, S = 1, 4, 128, 512
    g = torch.Generator().manual_seed(9)
    k = (torch.randn(B, H, S, d, generator=g) / d ** 0.5).half()
    v = (torch.randn(B, H, S, d, generator=g) / d ** 0.5).half()
    q = (torch.randn(B, H, d, generator=g) / d ** 0.5).half()
    exact = torch.softmax((q.float()[:, :, None] @ k.float().transpose(-1, -2)).squeeze(2) / d ** 0.5, -1)
    exact = (exact[:, :, None] @ v.float()).squeeze(2).flatten()
    cache = BitCache(B, H, d, max_seq=S)
    cache.prefill(k.to(cuda), v.to(cuda))
    full = cache.attend(q.to(cuda)).float().cpu().flatten()
    K, V = cache.planes
    binary = planes.decode_attention(q.view(-1, d).to(cuda), K, V, S, planes.MODE_BINARY).float().cpu().flatten()
    cache.keep_residuals(0.25)
    n_keep = planes.keep_count(S, 0.25)
    assert ((K.rscale[:, :S] != 0).sum(1) <= n_keep).all() and ((V.rscale[:, :S] != 0).sum(1) <= n_keep).all()
    part = cache.attend(q.to(cuda)).float().cpu().flatten()
    cos = lambda a: float(torch.nn.functional.cosine_similarity(a, exact, dim=0))  # noqa: E731
    assert cos(binary) - 0.01 <= cos(part) <= cos(full) + 0.01


# ---- compact adaptive caches: joint K+V selection per position, kept rows first ----

def host_rows(P, rows_stride=None):
    """Host copy with per-row nibbles (reference byte order) even when the residual
    planes have their own row stride."""
    return {"words": P.sign.cpu().numpy().view(np.uint32), "bscale": P.bscale.cpu().numpy().view(np.uint16),
            "nib": planes.nib_rows(P.nib, P.head_dim).cpu().numpy(), "rscale": P.rscale.cpu().numpy().view(np.uint16)}


@pytest.mark.parametrize("slots,group,S,d,frac", [
    (4, 1, 777, 128, 0.25),
    (3, 2, 1000, 64, 0.25),
    (2, 4, 513, 256, 0.5),
    (2, 4, 900, 64, 0.25),
    (5, 1, 300, 128, 0.0),
    (2, 1, 129, 128, 1.0),
    (3, 8, 2048, 128, 0.25),
])
def test_compact_adaptive_matches_zeroed_oracle(cuda, slots, group, S, d, frac):
    stride = planes.round_stride(S)
    K, _ = build(cuda, slots, S, stride, d, seed=S + d, dup=True)
    V, _ = build(cuda, slots, S, stride, d, seed=S + d + 1)
    n_keep = planes.keep_count(S, frac)
    hk, hv = host(K), host(V)
    keep = planes.select_positions_topk(K, V, S, n_keep)
    want_keep = O.select_positions_topk(hk["nib"], hk["rscale"], hv["nib"], hv["rscale"], S, n_keep)
    assert np.array_equal(keep[:, :S].cpu().numpy(), want_keep)
    Kc, Vc = planes.compact_adaptive(K, V, keep, S, n_keep)
    # rows moved as a stable partition: kept first, the rest from round8(n_keep)
    b0 = planes.round_stride(n_keep)
    hkc, hvc = host_rows(Kc), host_rows(Vc)
    for j in range(slots):
        kept = np.nonzero(want_keep[j])[0]
        rest = np.nonzero(want_keep[j] == 0)[0]
        for h0, hc in ((hk, hkc), (hv, hvc)):
            assert np.array_equal(hc["words"][j, :n_keep], h0["words"][j, kept])
            assert np.array_equal(hc["words"][j, b0:b0 + len(rest)], h0["words"][j, rest])
            assert np.array_equal(hc["bscale"][j, b0:b0 + len(rest)], h0["bscale"][j, rest])
            assert np.array_equal(hc["nib"][j, :n_keep], h0["nib"][j, kept])
            assert np.array_equal(hc["rscale"][j, :n_keep], h0["rscale"][j, kept])
    # attention: equal (within tolerance) to compensated attention with the unkept residuals zeroed
    g = torch.Generator().manual_seed(S)
    q = (torch.randn(slots * group, d, generator=g) / d ** 0.5).half()
    got = planes.decode_attention_adaptive(q.to(cuda), Kc, Vc, S, n_keep).float().cpu().numpy()
    m = want_keep.astype(bool)
    for h0 in (hk, hv):
        h0["rscale"] = h0["rscale"].copy()
        h0["nib"] = h0["nib"].copy()
        h0["rscale"][:, :S] = np.where(m, h0["rscale"][:, :S], 0)
        h0["nib"][:, :S] = np.where(m[..., None], h0["nib"][:, :S], 0)
    want = O.attention(q.numpy(), hk, hv, group, S, stride, True).view(np.float16).astype(np.float32)
    assert np.max(np.abs(got - want)) <= 2e-3
    if np.linalg.norm(want) > 1e-6:
        assert float((got * want).sum() / (np.linalg.norm(got) * np.linalg.norm(want))) >= 0.9999


def test_compact_adaptive_c5_shape_bytes(cuda):
    """C5-like slot count at a short length: the compact cache stores the residual
    planes for the kept quarter only."""
    slots, S, d = 64, 512, 128
    K, _ = build(cuda, slots, S, S, d, seed=5)
    V, _ = build(cuda, slots, S, S, d, seed=6)
    n_keep = planes.keep_count(S, 0.25)
    keep = planes.select_positions_topk(K, V, S, n_keep)
    assert (keep[:, :S].sum(1) == n_keep).all()
    Kc, Vc = planes.compact_adaptive(K, V, keep, S, n_keep)
    assert Kc.nib.shape[1] == planes.round_stride(n_keep)
    q = (torch.randn(slots, d) / d ** 0.5).half().to(cuda)
    out = planes.decode_attention_adaptive(q, Kc, Vc, S, n_keep)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()


@pytest.mark.parametrize("slots,S", [(3, 1000), (64, 512)])
def test_adaptive_with_pinned_host_query_and_output(cuda, slots, S):
    """Pinned host Q and output (the end-to-end form of the call): Q is staged to
    the device by one launch and the kernel writes the output over the host link;
    the result is bit-identical to the all-device call, twice in a row."""
    d, group = 128, 2
    K, _ = build(cuda, slots, S, S, d, seed=11)
    V, _ = build(cuda, slots, S, S, d, seed=12)
    n_keep = planes.keep_count(S, 0.25)
    keep = planes.select_positions_topk(K, V, S, n_keep)
    Kc, Vc = planes.compact_adaptive(K, V, keep, S, n_keep)
    g = torch.Generator().manual_seed(slots)
    q = (torch.randn(slots * group, d, generator=g) / d ** 0.5).half()
    want = planes.decode_attention_adaptive(q.to(cuda), Kc, Vc, S, n_keep).cpu()
    qh = q.pin_memory()
    oh = torch.zeros(slots * group, d, dtype=torch.float16).pin_memory()
    for _ in range(2):
        oh.zero_()
        planes.decode_attention_adaptive(qh, Kc, Vc, S, n_keep, out=oh)
        torch.cuda.synchronize()
        assert torch.equal(oh, want)
    with pytest.raises(RuntimeError):
        planes.decode_attention_adaptive(qh, Kc, Vc, S, n_keep, out=torch.empty(4, d, dtype=torch.float16).pin_memory())
    with pytest.raises(RuntimeError):
        planes.decode_attention_adaptive(q, Kc, Vc, S, n_keep)  # pageable host Q
