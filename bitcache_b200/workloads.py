"""Seeded synthetic workloads for the five benchmark/parity configurations.

No public dataset is involved: every tensor is drawn from a torch Generator
seeded per config, in fp32, then cast to fp16, in the order Q, K, V.

C1  B=1,  H=8,  S=1024,  d=128: Q, K, V ~ N(0, 1/128)                  (CPU-runnable case)
C2  B=1,  H=32, S=4096,  d=128: per head 32 keys correlated 0.25 with Q
C3  B=1,  H=32, S=65536, d=128: K, V ~ N(0, 1/128), 1% of channels x8   (headline)
C4  B=16, Hq=32, Hkv=8, S=32768 prefilled + 64 appended tokens, d=128
C5  B=64, H=32, S=8192, d in {64, 128, 256}: K, V Student-t(5) scaled to variance 1/d
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch


@dataclass
class Workload:
    name: str
    batch: int
    n_heads: int
    n_kv_heads: int
    seq_len: int
    head_dim: int
    q: torch.Tensor          # [B, Hq, d] fp16
    k: torch.Tensor          # [B, Hkv, S, d] fp16
    v: torch.Tensor          # [B, Hkv, S, d] fp16
    extra: dict = field(default_factory=dict)

    @property
    def n_slots(self) -> int:
        return self.batch * self.n_kv_heads

    @property
    def group(self) -> int:
        return self.n_heads // self.n_kv_heads


CONFIGS = {
    "C1": dict(batch=1, n_heads=8, n_kv_heads=8, seq_len=1024, head_dim=128),
    "C2": dict(batch=1, n_heads=32, n_kv_heads=32, seq_len=4096, head_dim=128),
    "C3": dict(batch=1, n_heads=32, n_kv_heads=32, seq_len=65536, head_dim=128),
    "C4": dict(batch=16, n_heads=32, n_kv_heads=8, seq_len=32768, head_dim=128, steps=64),
    "C5": dict(batch=64, n_heads=32, n_kv_heads=32, seq_len=8192, head_dim=128, keep=0.25),
}


def _normal(shape, std: float, g: torch.Generator, device) -> torch.Tensor:
    return torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std


def _student_t5(shape, g: torch.Generator, device) -> torch.Tensor:
    # z / sqrt(chi2_5 / 5), in place so that at most three full-size fp32
    # tensors are alive (C5 at head_dim 256 is 4.3 G elements per tensor)
    z = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
    chi2 = torch.zeros(shape, device=device, dtype=torch.float32)
    for _ in range(5):
        t = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
        chi2 += t.square_()
        del t
    return z.div_(chi2.div_(5.0).sqrt_())


def make(name: str, device: str | torch.device = "cpu", seed: int | None = None, **over) -> Workload:
    """Build config `name` (C1..C5) with optional shape overrides (e.g. seq_len=...)."""
    cfg = dict(CONFIGS[name])
    cfg.update(over)
    b, hq, hkv, s, d = cfg["batch"], cfg["n_heads"], cfg["n_kv_heads"], cfg["seq_len"], cfg["head_dim"]
    seed = {"C1": 0, "C2": 2, "C3": 3, "C4": 4, "C5": 5}[name] if seed is None else seed
    device = torch.device(device)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    std = 1.0 / math.sqrt(d)
    extra: dict = {}
    if name == "C5":
        q = _normal((b, hq, d), std, g, device)
        scale = math.sqrt(3.0 / (5.0 * d))
        k = _student_t5((b, hkv, s, d), g, device).mul_(scale).half()
        v = _student_t5((b, hkv, s, d), g, device).mul_(scale).half()
        extra["keep"] = cfg.get("keep", 0.25)
    else:
        q = _normal((b, hq, d), std, g, device)
        k = _normal((b, hkv, s, d), std, g, device)
        v = _normal((b, hkv, s, d), std, g, device)
        if name == "C2":
            # Per (batch, head): 32 keys built as 0.25*q + sqrt(1-0.25^2)*z.
            rho = 0.25
            grp = hq // hkv
            for bi in range(b):
                for h in range(hkv):
                    pos = torch.randperm(s, generator=g, device=device)[:32]
                    z = _normal((32, d), std, g, device)
                    k[bi, h, pos] = rho * q[bi, h * grp] + math.sqrt(1 - rho * rho) * z
        elif name == "C3":
            n_out = max(1, math.ceil(0.01 * d))
            for bi in range(b):
                for h in range(hkv):
                    ch = torch.randperm(d, generator=g, device=device)[:n_out]
                    k[bi, h, :, ch] *= 8.0
                    v[bi, h, :, ch] *= 8.0
        elif name == "C4":
            steps = cfg.get("steps", 64)
            extra["steps"] = steps
            extra["k_new"] = _normal((steps, b, hkv, d), std, g, device).half()
            extra["v_new"] = _normal((steps, b, hkv, d), std, g, device).half()
    return Workload(name, b, hq, hkv, s, d, q.half(), k.half().contiguous(), v.half().contiguous(), extra)


def vector_footprint(head_dim: int, compensated: bool = True) -> int:
    """Algorithmic cache bytes per K or V vector used for GB/s figures: the
    reference README's 82 B at head_dim 128 (README.md:42), 5d/8 + 4 otherwise;
    binary only d/8 + 2."""
    if not compensated:
        return head_dim // 8 + 2
    return 82 if head_dim == 128 else 5 * head_dim // 8 + 4


def adaptive_step_bytes(batch: int, n_kv_heads: int, seq_len: int, head_dim: int, keep: float) -> int:
    """Algorithmic bytes of one decode step over a compact adaptive cache: sign and scale
    of every vector, the residual (d/2 + 2 B) of the kept fraction only; 34.5 B per
    vector at head_dim 128 and keep 0.25."""
    per = (head_dim // 8 + 2) + keep * (head_dim // 2 + 2)
    return int(round(2 * batch * n_kv_heads * seq_len * per))


def step_cache_bytes(batch: int, n_kv_heads: int, seq_len: int, head_dim: int, compensated: bool = True) -> int:
    """Algorithmic bytes of one decode step: K and V of every (batch, kv head, position) read once."""
    return 2 * batch * n_kv_heads * seq_len * vector_footprint(head_dim, compensated)
