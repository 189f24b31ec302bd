"""The C++ launcher API (include/bitcache_b200_compat.cuh, the reference's
src/*.cuh launch_* signatures) called from a C++ program, as the reference's
own C++ tests call it (tests/test_correctness.cu:109-117 of the reference).

CPU: the caller compiles against the header and links against the library.
GPU: it runs, and its encodings are bit-exact against the reference's own
kernels on the same inputs, its attention outputs within max-abs 2e-3 and
cosine >= 0.9999 of the reference kernels, its entropy within 1e-4, its
precision modes equal, and its online-encoded ring bit-exact."""
import os
import shutil
import subprocess

import numpy as np
import pytest
import torch

from bitcache_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "cpp", "launchers_caller.cpp")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def build_caller(out_dir: str) -> str:
    exe = os.path.join(out_dir, "launchers_caller")
    libdir = os.path.dirname(_lib.LIB_PATH)
    cmd = ["g++", "-std=c++17", "-O2", "-I", os.path.join(ROOT, "include"), "-I", os.path.join(CUDA, "include"),
           SRC, "-o", exe, "-L", libdir, "-lbitcache_b200", f"-Wl,-rpath,{libdir}",
           "-L", os.path.join(CUDA, "lib64"), "-lcudart", f"-Wl,-rpath,{os.path.join(CUDA, 'lib64')}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, f"compiling the C++ caller failed:\n{r.stderr}"
    return exe


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_cpp_caller_compiles_and_links(tmp_path):
    _lib.load()  # the library must be built
    exe = build_caller(str(tmp_path))
    assert os.path.exists(exe)


@pytest.mark.gpu
@pytest.mark.parametrize("B,H,S,D", [(1, 8, 1024, 128), (2, 3, 300, 64), (1, 32, 4096, 128), (1, 2, 77, 256)])
def test_cpp_launchers_match_reference_kernels(cuda, tmp_path, B, H, S, D):
    from oracle import oracle as O
    from oracle import refgpu

    exe = build_caller(str(tmp_path))
    g = torch.Generator().manual_seed(B * 100 + H + S + D)
    q = (torch.randn(B * H, D, generator=g) * 0.5).half()
    k = (torch.randn(B * H * S, D, generator=g) * 0.5).half()
    v = (torch.randn(B * H * S, D, generator=g) * 0.5).half()
    tok = (torch.randn(B * H, D, generator=g) * 0.5).half()
    for name, t in (("q", q), ("k", k), ("v", v), ("tok", tok)):
        t.numpy().tofile(os.path.join(tmp_path, name + ".bin"))
    r = subprocess.run([exe, str(tmp_path), str(B), str(H), str(S), str(D)], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, f"C++ caller failed ({r.returncode}): {r.stderr}"

    def got(name, dtype=np.uint8):
        return np.fromfile(os.path.join(tmp_path, name + ".bin"), dtype=dtype)

    kd, vd, qd = k.to(cuda), v.to(cuda), q.to(cuda)
    kb, vb = refgpu.binary_encode(kd), refgpu.binary_encode(vd)
    kr, vr = refgpu.residual_encode(kd, kb), refgpu.residual_encode(vd, vb)
    for mine, ref, split in (("kb", kb, O.split_binvec), ("vb", vb, O.split_binvec),
                             ("kr", kr, O.split_resvec), ("vr", vr, O.split_resvec)):
        a, b = split(got(mine), D), split(ref.cpu().numpy(), D)
        for x, y in zip(a, b):
            assert np.array_equal(x, y), f"{mine} differs from the reference encoder"

    def close(mine, ref, label):
        m = got(mine, np.float16).astype(np.float64)
        w = ref.float().cpu().numpy().astype(np.float64).ravel()
        assert np.max(np.abs(m - w)) <= 2e-3, label
        assert float(m @ w / (np.linalg.norm(m) * np.linalg.norm(w) + 1e-30)) >= 0.9999, label

    close("out_bin", refgpu.attention(qd, kb, vb, None, None, B, H, S, D), "launch_binary_attention")
    close("out_comp", refgpu.attention(qd, kb, vb, kr, vr, B, H, S, D), "launch_compensated_attention")
    ent = refgpu.head_entropy(qd, kb, B, H, S, D)
    np.testing.assert_allclose(got("ent", np.float32), ent.cpu().numpy(), rtol=1e-4, atol=1e-4)
    assert np.array_equal(got("modes"), refgpu.adaptive_select(ent, 5.0).cpu().numpy())
    ring = 8
    rb = torch.zeros(B * H * ring * 36, dtype=torch.uint8, device=cuda)
    rr = torch.zeros(B * H * ring * 130, dtype=torch.uint8, device=cuda)
    for cur in (0, 1, 10):
        refgpu.online_encode_token(qd if cur == 1 else tok.to(cuda), rb, rr, B, H, D, cur, ring)
    torch.cuda.synchronize()
    assert np.array_equal(got("ring_b"), rb.cpu().numpy()), "online-encoded binary ring differs"
    assert np.array_equal(got("ring_r"), rr.cpu().numpy()), "online-encoded residual ring differs"
