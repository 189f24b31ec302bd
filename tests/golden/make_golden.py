"""Generate the golden fixtures in tests/golden/ by running the REFERENCE's own
CUDA kernels (oracle/_ref/libbitcache_ref.so, built from the reference sources
by oracle/build.py) on the seeded inputs of cases.py.  Needs a GPU:

    python tests/golden/make_golden.py --out tests/golden

Each fixture holds the reference record fields (sign words, binary scale,
INT4 nibbles, residual scale) for K and V, the binary and compensated
attention outputs, the exact fp16 attention, the head entropy, and the
SHA-256 of the inputs.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, HERE)

import cases  # noqa: E402
from oracle import oracle as O  # noqa: E402
from oracle import refgpu  # noqa: E402


def fields(bin_blob: torch.Tensor, res_blob: torch.Tensor | None, d: int):
    w, s = O.split_binvec(bin_blob.cpu().numpy(), d)
    out = {"words": w, "bscale": s}
    if res_blob is not None:
        nib, rs = O.split_resvec(res_blob.cpu().numpy(), d)
        out["nib"] = nib
        out["rscale"] = rs
    return out


def attn_case(name: str) -> dict:
    b, h, s, d, _, _ = cases.ATTN_CASES[name]
    q, k, v = cases.attn_inputs(name)
    res = {"sha256": np.array(cases.sha256(q, k, v))}
    qg, kg, vg = q.cuda(), k.cuda(), v.cuda()
    kb = refgpu.binary_encode(kg)
    kr = refgpu.residual_encode(kg, kb)
    vb = refgpu.binary_encode(vg)
    vr = refgpu.residual_encode(vg, vb)
    for pre, bb, rr in (("k_", kb, kr), ("v_", vb, vr)):
        for key, val in fields(bb, rr, d).items():
            res[pre + key] = val
    res["bin_out"] = refgpu.attention(qg, kb, vb, None, None, b, h, s, d).cpu().numpy().view(np.uint16)
    res["comp_out"] = refgpu.attention(qg, kb, vb, kr, vr, b, h, s, d).cpu().numpy().view(np.uint16)
    res["exact_out"] = refgpu.reference_attention(qg, kg, vg, b, h, s, d).cpu().numpy().view(np.uint16)
    res["entropy"] = refgpu.head_entropy(qg, kb, b, h, s, d).cpu().numpy()
    thr = float(np.median(res["entropy"]))
    res["select_thr"] = np.array(thr, np.float32)
    res["modes"] = refgpu.adaptive_select(torch.from_numpy(res["entropy"]).cuda(), thr).cpu().numpy()
    torch.cuda.synchronize()
    return res


def encode_only(name: str, x: torch.Tensor) -> dict:
    d = x.shape[1]
    xg = x.cuda()
    b = refgpu.binary_encode(xg)
    r = refgpu.residual_encode(xg, b)
    out = {"sha256": np.array(cases.sha256(x))}
    out.update(fields(b, r, d))
    return out


def online_case() -> dict:
    c = cases.ONLINE_CASE
    toks = cases.online_inputs()
    n = c["batch"] * c["n_heads"]
    binc = torch.zeros(n * c["max_seq"] * 36, dtype=torch.uint8, device="cuda")
    resc = torch.zeros(n * c["max_seq"] * 130, dtype=torch.uint8, device="cuda")
    for t in range(c["steps"]):
        refgpu.online_encode_token(toks[t].cuda(), binc, resc, c["batch"], c["n_heads"], c["head_dim"], t,
                                   c["max_seq"])
    torch.cuda.synchronize()
    out = {"sha256": np.array(cases.sha256(toks))}
    out.update(fields(binc, resc, c["head_dim"]))
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    os.makedirs(args.out, exist_ok=True)
    for name in cases.ATTN_CASES:
        np.savez_compressed(os.path.join(args.out, f"{name}.npz"), **attn_case(name))
        print("wrote", name)
    np.savez_compressed(os.path.join(args.out, "edge.npz"), **encode_only("edge", cases.edge_vectors()))
    np.savez_compressed(os.path.join(args.out, "special.npz"), **encode_only("special", cases.special_vectors()))
    np.savez_compressed(os.path.join(args.out, "online.npz"), **online_case())
    print("done")


if __name__ == "__main__":
    main()
