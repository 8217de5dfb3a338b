"""Build libtrcuda.so in-tree with nvcc for sm_100a (B200).

``python -m turbo_roformer_b200._build`` or ``build()``; the library lands next to this file so that it
travels with the source tree. nvcc cross-compiles: no GPU is needed to build.
"""

from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
LIB_NAME = "libtrcuda.so"
LIB_PATH = os.path.join(HERE, LIB_NAME)
SOURCES = ("api.cu", "tc.cu", "dsp.cu", "pack.cu", "ola_noalloc.cu")
ARCH_FLAGS = ("-gencode", "arch=compute_100a,code=sm_100a")


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put the CUDA toolkit on PATH)")


def _source_hash() -> str:
    h = hashlib.sha256()
    for d in (CSRC, INCLUDE):
        for name in sorted(os.listdir(d)):
            if name.endswith((".cu", ".cuh", ".h")):
                with open(os.path.join(d, name), "rb") as f:
                    h.update(name.encode())
                    h.update(f.read())
    h.update(" ".join(ARCH_FLAGS).encode())
    return h.hexdigest()[:16]


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the CUDA sources into ``turbo_roformer_b200/libtrcuda.so`` (skipped when up to date)."""
    stamp = LIB_PATH + ".hash"
    digest = _source_hash()
    if not force and os.path.exists(LIB_PATH) and os.path.exists(stamp):
        with open(stamp) as f:
            if f.read().strip() == digest:
                return LIB_PATH
    cmd = [
        _nvcc(),
        *ARCH_FLAGS,
        "-lineinfo",
        "-O3",
        "-std=c++17",
        "-Xcompiler",
        "-fPIC",
        "-shared",
        "-I",
        INCLUDE,
        "-o",
        LIB_PATH + ".tmp",
        *(os.path.join(CSRC, s) for s in SOURCES),
    ]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(LIB_PATH + ".tmp", LIB_PATH)
    with open(stamp, "w") as f:
        f.write(digest + "\n")
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
