"""Golden-vector cases: seeded inputs shared by make_golden.py (which runs the
reference's own kernels on a GPU to produce the expected outputs) and the CPU
tests (which regenerate the inputs and check the oracle against them).

Inputs are drawn with a CPU torch.Generator; each fixture stores the SHA-256
of the input bytes so that generator drift is detected instead of masked.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from bitcache_b200 import workloads  # noqa: E402

# name -> (batch, n_heads, seq_len, head_dim, distribution, seed)
ATTN_CASES = {
    "c1": (1, 8, 1024, 128, "C1", 0),
    "d64_uniform": (1, 4, 512, 64, "uniform", 618),
    "d256_ragged": (2, 2, 300, 256, "randn", 7),
    "d96_small": (1, 3, 77, 96, "randn", 9),
    "d32_tiny": (1, 2, 64, 32, "randn", 11),
}

ONLINE_CASE = dict(batch=2, n_heads=3, head_dim=128, max_seq=16, steps=20, seed=21)


def attn_inputs(name: str):
    """-> q [B*H, d], k [B*H*S, d], v [B*H*S, d] as fp16 CPU tensors."""
    b, h, s, d, dist, seed = ATTN_CASES[name]
    if dist == "C1":
        w = workloads.make("C1")
        return (w.q.reshape(b * h, d).contiguous(), w.k.reshape(-1, d).contiguous(), w.v.reshape(-1, d).contiguous())
    g = torch.Generator().manual_seed(seed)
    shape_q, shape_kv = (b * h, d), (b * h * s, d)
    if dist == "uniform":  # test_correctness.cu:26-31: uniform [-1, 1] * 0.5
        mk = lambda shp: ((torch.rand(shp, generator=g) * 2 - 1) * 0.5).half()  # noqa: E731
    else:  # test_python.py:92: randn * 0.5
        mk = lambda shp: (torch.randn(shp, generator=g) * 0.5).half()  # noqa: E731
    q = mk(shape_q)
    k = mk(shape_kv)
    v = mk(shape_kv)
    return q, k, v


def edge_vectors(d: int = 128) -> torch.Tensor:
    """Encode-only special vectors: zeros, -0.0, extremes, fp16 subnormals, one-hot, ties, inf/nan."""
    rows = []
    z = torch.zeros(d, dtype=torch.float16)
    rows.append(z.clone())
    rows.append(torch.full((d,), -0.0, dtype=torch.float16))
    rows.append(torch.full((d,), 65504.0, dtype=torch.float16))
    alt = torch.full((d,), 65504.0, dtype=torch.float16)
    alt[1::2] = -65504.0
    rows.append(alt)
    sub = torch.arange(d, dtype=torch.int32).remainder(1024).to(torch.int16).view(torch.float16)  # subnormals
    rows.append(sub.clone())
    neg_sub = sub.clone()
    neg_sub[::3] = -neg_sub[::3]
    rows.append(neg_sub)
    oh = z.clone()
    oh[d // 3] = 1.0
    rows.append(oh)
    ohn = z.clone()
    ohn[5] = -3.5
    rows.append(ohn)
    lin = torch.linspace(-1, 1, d).half()
    rows.append(lin)
    ramp = (torch.arange(d, dtype=torch.float32) - d / 2).half()
    rows.append(ramp)
    allneg = -torch.linspace(0.01, 2.0, d).half()
    rows.append(allneg)
    g = torch.Generator().manual_seed(123)
    for _ in range(5):  # values spanning magnitudes
        e = torch.randint(-14, 15, (d,), generator=g).float()
        rows.append((torch.randn(d, generator=g) * torch.pow(2.0, e)).half())
    return torch.stack(rows).contiguous()


def special_vectors(d: int = 128) -> torch.Tensor:
    """inf / nan carrying vectors (encode only)."""
    g = torch.Generator().manual_seed(321)
    base = (torch.randn(4, d, generator=g) * 0.3).half()
    base[0, 7] = float("inf")
    base[1, 9] = float("-inf")
    base[2, 11] = float("nan")
    base[3, :] = float("nan")
    return base.contiguous()


def online_inputs():
    c = ONLINE_CASE
    g = torch.Generator().manual_seed(c["seed"])
    n = c["batch"] * c["n_heads"]
    toks = (torch.randn(c["steps"], n, c["head_dim"], generator=g) * 0.5).half()
    return toks


def sha256(*ts: torch.Tensor) -> str:
    h = hashlib.sha256()
    for t in ts:
        h.update(t.contiguous().view(-1).view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def fixture_path(name: str) -> str:
    return os.path.join(HERE, f"{name}.npz")


def load_fixture(name: str):
    p = fixture_path(name)
    if not os.path.exists(p):
        return None
    return dict(np.load(p, allow_pickle=False))
