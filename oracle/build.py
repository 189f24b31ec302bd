"""Build recipe for the checkers under oracle/ -- TEST INFRASTRUCTURE ONLY.

* ``oracle/libbitcache_oracle.so``: the C restatement (bitcache_oracle.c),
  gcc -O3 -fopenmp, strict IEEE (no FP contraction) so that it computes the
  reference's expressions term by term.
* ``oracle/_ref/libbitcache_ref.so``: the reference's own CUDA kernels,
  compiled for sm_100a from their sources where they lie (the reference
  checkout's ``src/``, named by ``BITCACHE_REF_SRC`` or, as its root, by
  ``BITCACHE_REF_ROOT``) with the
  reference's own nvcc flags (setup.py:7-17 of the reference) plus
  ref_shim.cu.  Built only where those sources exist; the prebuilt .so travels
  with the repository snapshot to the GPU box.

Usage: ``python oracle/build.py [--oracle] [--ref] [--ref-root <reference checkout>]``
(both by default).
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "libbitcache_oracle.so")
REF_DIR = os.path.join(HERE, "_ref")
REF_SO = os.path.join(REF_DIR, "libbitcache_ref.so")

# The reference's kernel sources (src/*.cu of anishesg/bitcache).
REF_SOURCES = [
    "binary_encode.cu",
    "residual.cu",
    "binary_attention.cu",
    "compensated_attention.cu",
    "online_encode.cu",
    "adaptive_precision.cu",
    "reference_attention.cu",
]


def ref_src_dir() -> str | None:
    """The reference's src/ directory: BITCACHE_REF_SRC, else the `src` folder of
    a reference checkout named by BITCACHE_REF_ROOT; None when neither is set."""
    if os.environ.get("BITCACHE_REF_SRC"):
        return os.environ["BITCACHE_REF_SRC"]
    if os.environ.get("BITCACHE_REF_ROOT"):
        return os.path.join(os.environ["BITCACHE_REF_ROOT"], "src")
    return None


def _up_to_date(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return False
    t = os.path.getmtime(target)
    return all(os.path.getmtime(d) <= t for d in deps if os.path.exists(d))


def build_oracle(force: bool = False) -> str:
    src = os.path.join(HERE, "bitcache_oracle.c")
    if not force and _up_to_date(ORACLE_SO, [src, __file__]):
        return ORACLE_SO
    cmd = [
        "gcc", "-O3", "-std=c11", "-fPIC", "-shared", "-fopenmp",
        "-ffp-contract=off", "-fno-fast-math", "-march=x86-64-v2",
        src, "-o", ORACLE_SO + ".tmp", "-lm",
    ]
    subprocess.run(cmd, check=True)
    os.replace(ORACLE_SO + ".tmp", ORACLE_SO)
    return ORACLE_SO


def build_ref(force: bool = False) -> str | None:
    """Compile the reference kernels; returns the .so path, or None when the
    reference sources are not present on this machine."""
    sdir = ref_src_dir()
    srcs = [os.path.join(sdir, s) for s in REF_SOURCES] if sdir else []
    if not srcs or not all(os.path.exists(s) for s in srcs):
        return REF_SO if os.path.exists(REF_SO) else None
    shim = os.path.join(HERE, "ref_shim.cu")
    if not force and _up_to_date(REF_SO, srcs + [shim, __file__]):
        return REF_SO
    os.makedirs(REF_DIR, exist_ok=True)
    nvcc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    cmd = [
        nvcc, "-O3", "--use_fast_math", "--expt-relaxed-constexpr", "--expt-extended-lambda", "-std=c++17",
        "-gencode=arch=compute_100a,code=sm_100a", "-lineinfo",
        "-shared", "-Xcompiler", "-fPIC", "-I", sdir,
        *srcs, shim, "-o", REF_SO + ".tmp",
    ]
    subprocess.run(cmd, check=True)
    os.replace(REF_SO + ".tmp", REF_SO)
    return REF_SO


if __name__ == "__main__":
    args = sys.argv[1:]
    if "--ref-root" in args:  # the reference checkout to compile the checker from
        i = args.index("--ref-root")
        os.environ["BITCACHE_REF_ROOT"] = args[i + 1]
        del args[i:i + 2]
    want = set(args) or {"--oracle", "--ref"}
    if "--oracle" in want:
        print(build_oracle(force=True))
    if "--ref" in want:
        print(build_ref(force=True))
