"""Build recipe for libwfd_b200.so (the C-ABI library) — nvcc, sm_100a only.

    python wavefront-decoding_b200/build.py [--force]

The library is built in-tree under `_lib/` so it travels with the source tree;
nothing is installed into site-packages and no JIT cache is used.
"""
from __future__ import annotations

import hashlib
import os
import pathlib
import subprocess
import sys

PKG_DIR = pathlib.Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
INCLUDE = PKG_DIR.parent / "include"
OUT_DIR = PKG_DIR / "_lib"
LIB_PATH = OUT_DIR / "libwfd_b200.so"
STAMP = OUT_DIR / "libwfd_b200.stamp"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
]


def _sources() -> list[pathlib.Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h")))


def _digest() -> str:
    h = hashlib.sha256()
    for p in _sources():
        h.update(p.name.encode())
        h.update(p.read_bytes())
    h.update(" ".join(NVCC_FLAGS).encode())
    return h.hexdigest()


def nvcc() -> str:
    cand = os.environ.get("NVCC") or "/usr/local/cuda/bin/nvcc"
    return cand if pathlib.Path(cand).exists() else "nvcc"


def build(force: bool = False, verbose: bool = False) -> pathlib.Path:
    """Compile csrc/wfd_abi.cu (which includes every kernel) into LIB_PATH.
    Skips the compile when the sources are unchanged since the last build."""
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    digest = _digest()
    if not force and LIB_PATH.exists() and STAMP.exists() and STAMP.read_text().strip() == digest:
        return LIB_PATH
    cmd = [nvcc(), *NVCC_FLAGS, "-I", str(INCLUDE), str(CSRC / "wfd_abi.cu"), "-o", str(LIB_PATH) + ".tmp"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(str(LIB_PATH) + ".tmp", LIB_PATH)
    STAMP.write_text(digest + "\n")
    return LIB_PATH


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(path)
