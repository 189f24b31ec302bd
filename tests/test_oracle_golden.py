"""CPU: the C oracle against golden vectors produced by the reference's own
CUDA kernels (tests/golden/make_golden.py).  Pins the oracle before it is
used as the checker of the B200 kernels."""
import numpy as np
import pytest

import cases
from oracle import oracle as O

POW2 = {32, 64, 128, 256}


def codes(nib: np.ndarray) -> np.ndarray:
    lo = (nib & 0x0F).astype(np.int16)
    hi = (nib >> 4).astype(np.int16)
    lo = np.where(lo >= 8, lo - 16, lo)
    hi = np.where(hi >= 8, hi - 16, hi)
    out = np.empty(nib.shape[:-1] + (nib.shape[-1] * 2,), np.int16)
    out[..., 0::2] = lo
    out[..., 1::2] = hi
    return out


def check_codes(got_nib, want_nib, pre, label):
    """INT4 codes must match exactly, except single-step differences where the
    oracle's IEEE value r*(7/absmax) sits next to a rounding tie (the reference
    divides with --use_fast_math)."""
    a, b = codes(got_nib), codes(want_nib)
    bad = a != b
    n_bad = int(bad.sum())
    if n_bad:
        assert np.all(np.abs(a[bad] - b[bad]) == 1), f"{label}: code differs by more than 1"
        p = np.abs(pre.reshape(a.shape)[bad])
        dist_to_tie = np.abs(p - np.floor(p) - 0.5)
        # within ~2 ulp of the tie: explained by a 2-ulp difference in 7/absmax
        assert np.all(dist_to_tie <= 3e-7 * np.maximum(1.0, p)), f"{label}: mismatch not at a rounding tie"
        assert n_bad <= 2 + a.size // 10000, f"{label}: {n_bad} tie-adjacent mismatches"
    return n_bad


def half_bits_equal(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    fa, fb = a.view(np.float16), b.view(np.float16)
    return (a == b) | (np.isnan(fa) & np.isnan(fb))


def fixture(name):
    fx = cases.load_fixture(name)
    assert fx is not None, f"golden fixture {name}.npz missing (run tests/golden/make_golden.py on a GPU)"
    return fx


@pytest.mark.parametrize("name", list(cases.ATTN_CASES))
def test_encodings_match_reference(name):
    fx = fixture(name)
    q, k, v = cases.attn_inputs(name)
    assert cases.sha256(q, k, v) == str(fx["sha256"]), "input generator drift"
    d = q.shape[1]
    for pre, x in (("k_", k), ("v_", v)):
        xs = x.numpy()
        w, s = O.binary_encode(xs)
        assert np.array_equal(w, fx[pre + "words"]), "sign words differ"
        if d in POW2:
            assert np.array_equal(s, fx[pre + "bscale"]), "binary scale differs"
        else:  # fast-math x/d vs IEEE for non-power-of-two d: at most one fp16 ulp, rarely
            diff = np.abs(s.astype(np.int32) - fx[pre + "bscale"].astype(np.int32))
            assert diff.max() <= 1 and (diff > 0).sum() <= max(2, s.size // 1000)
        nib, rs, prepre = O.residual_encode(xs, fx[pre + "words"], fx[pre + "bscale"])
        assert np.array_equal(rs, fx[pre + "rscale"]), "residual scale differs"
        check_codes(nib, fx[pre + "nib"], prepre, f"{name}/{pre}")


def _planes_from_fixture(fx, pre, slots, seq, d):
    return {"words": fx[pre + "words"].reshape(slots, seq, d // 32), "bscale": fx[pre + "bscale"].reshape(slots, seq),
            "nib": fx[pre + "nib"].reshape(slots, seq, d // 2), "rscale": fx[pre + "rscale"].reshape(slots, seq)}


def cosine(a, b):
    a = a.astype(np.float64).ravel()
    b = b.astype(np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-30))


@pytest.mark.parametrize("name", list(cases.ATTN_CASES))
@pytest.mark.parametrize("compensated", [False, True])
def test_attention_matches_reference(name, compensated):
    fx = fixture(name)
    b, h, s, d, _, _ = cases.ATTN_CASES[name]
    q, _, _ = cases.attn_inputs(name)
    K = _planes_from_fixture(fx, "k_", b * h, s, d)
    V = _planes_from_fixture(fx, "v_", b * h, s, d)
    out = O.attention(q.numpy(), K, V, 1, s, s, compensated).view(np.float16).astype(np.float32)
    want = fx["comp_out" if compensated else "bin_out"].view(np.float16).astype(np.float32)
    assert np.max(np.abs(out - want)) <= 2e-3
    assert cosine(out, want) >= 0.9999


@pytest.mark.parametrize("name", list(cases.ATTN_CASES))
def test_entropy_and_select_match_reference(name):
    fx = fixture(name)
    b, h, s, d, _, _ = cases.ATTN_CASES[name]
    q, _, _ = cases.attn_inputs(name)
    ent = O.head_entropy(q.numpy(), fx["k_words"], fx["k_bscale"], s, s)
    np.testing.assert_allclose(ent, fx["entropy"], rtol=1e-4, atol=1e-4)
    assert np.array_equal(O.adaptive_select(fx["entropy"], float(fx["select_thr"])), fx["modes"])


@pytest.mark.parametrize("name", list(cases.ATTN_CASES))
def test_reference_quality_thresholds(name):
    """The reference's own asserted quality bars (tests/test_python.py:136, :158) hold on the fixtures."""
    fx = fixture(name)
    exact = fx["exact_out"].view(np.float16).astype(np.float32)
    cb = cosine(fx["bin_out"].view(np.float16).astype(np.float32), exact)
    cc = cosine(fx["comp_out"].view(np.float16).astype(np.float32), exact)
    assert cc > 0.85
    assert cc >= cb - 0.01


def test_exact_attention_matches_reference():
    fx = fixture("c1")
    q, k, v = cases.attn_inputs("c1")
    b, h, s, d, _, _ = cases.ATTN_CASES["c1"]
    out = O.reference_attention(q.numpy(), k.numpy().reshape(b * h, s, d), v.numpy().reshape(b * h, s, d))
    got = out.view(np.float16).astype(np.float32)
    want = fx["exact_out"].view(np.float16).astype(np.float32)
    assert np.max(np.abs(got - want)) <= 1e-3


@pytest.mark.parametrize("name,gen", [("edge", cases.edge_vectors), ("special", cases.special_vectors)])
def test_edge_vectors_match_reference(name, gen):
    fx = fixture(name)
    x = gen()
    assert cases.sha256(x) == str(fx["sha256"])
    xs = x.numpy()
    w, s = O.binary_encode(xs)
    assert np.array_equal(w, fx["words"])
    assert np.all(half_bits_equal(s, fx["bscale"]))
    nib, rs, pre = O.residual_encode(xs, fx["words"], fx["bscale"])
    assert np.all(half_bits_equal(rs, fx["rscale"]))
    check_codes(nib, fx["nib"], np.nan_to_num(pre), name)


def test_online_ring_matches_reference():
    fx = fixture("online")
    c = cases.ONLINE_CASE
    toks = cases.online_inputs()
    assert cases.sha256(toks) == str(fx["sha256"])
    n, ms, d = c["batch"] * c["n_heads"], c["max_seq"], c["head_dim"]
    words = np.zeros((n * ms, d // 32), np.uint32)
    bs = np.zeros(n * ms, np.uint16)
    nib = np.zeros((n * ms, d // 2), np.uint8)
    rs = np.zeros(n * ms, np.uint16)
    pre_all = np.zeros((n * ms, d), np.float32)
    for t in range(c["steps"]):
        w, b, nb, r, pre = O.online_encode(toks[t].numpy())
        idx = np.arange(n) * ms + t % ms
        words[idx], bs[idx], nib[idx], rs[idx], pre_all[idx] = w, b, nb, r, pre
    assert np.array_equal(words, fx["words"])
    assert np.array_equal(bs, fx["bscale"])
    assert np.array_equal(rs, fx["rscale"])
    check_codes(nib, fx["nib"], pre_all, "online")
