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
