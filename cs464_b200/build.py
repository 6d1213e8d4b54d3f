"""Ahead-of-time build of the sm_100a GEMM library `cs464_b200/libb2g.so` (nvcc, in-tree).

The reference compiles each Triton config on first use (kernels/triton_matmul.py:38-82, ~0.13 s per config, plus a
prebuilt-cubin bundle to hide it, kernels/bundle.py). Here the whole config space is one runtime-parameterised kernel,
compiled once from source by this script; first-use compile cost is zero by construction.

`python -m cs464_b200.build` rebuilds when any source or flag changed (the source hash is baked into the library and
returned by `b2g_source_hash()`).
"""
from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB_PATH = PKG / "libb2g.so"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-O2", "-shared"]


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def source_hash() -> str:
    """sha256 (16 hex) of every CUDA source, header and build flag: what a stored config key compiles to."""
    h = hashlib.sha256()
    files = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    for f in files:
        h.update(f.name.encode())
        h.update(f.read_bytes())
    h.update(" ".join(ARCH_FLAGS + NVCC_FLAGS).encode())
    return h.hexdigest()[:16]


def nvcc() -> str:
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(exe).exists():
        raise RuntimeError("nvcc not found: the sm_100a library cannot be built")
    return exe


def _stamp() -> Path:
    return PKG / ".libb2g.hash"


def up_to_date() -> bool:
    return LIB_PATH.exists() and _stamp().exists() and _stamp().read_text().strip() == source_hash()


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library for sm_100a unless it is already built from the current sources."""
    if not force and up_to_date():
        return LIB_PATH
    digest = source_hash()
    tmp = LIB_PATH.with_suffix(f".so.tmp{os.getpid()}")
    cmd = [nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", f'-DB2G_SOURCE_HASH="{digest}"',
           *map(str, sources()), "-o", str(tmp)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        tmp.unlink(missing_ok=True)
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(r.stderr, file=sys.stderr)
    os.replace(tmp, LIB_PATH)
    _stamp().write_text(digest + "\n")
    return LIB_PATH


if __name__ == "__main__":
    p = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(p)
