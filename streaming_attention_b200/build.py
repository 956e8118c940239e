"""Build libsa_b200.so in-tree from csrc/*.cu for sm_100a.

    python -m streaming_attention_b200.build        # or build() from Python

The library is written next to this file so that it travels with the source
tree; objects go to ``_build/`` at the repository root.  Rebuilds only when the
sources, headers or flags differ from those the library was built from (a
content hash kept beside it, so that a copied tree with new file times does
not rebuild).
"""

from __future__ import annotations

import glob
import hashlib
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libsa_b200.so")
STAMP = LIB + ".stamp"
BUILD_DIR = os.path.join(ROOT, "_build")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O3",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-warn-spills",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libsa_b200.so")


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h")))


def source_hash() -> str:
    h = hashlib.sha256()
    h.update(" ".join(NVCC_FLAGS).encode())
    for p in sources() + headers() + [__file__]:
        h.update(os.path.relpath(p, ROOT).encode())
        with open(p, "rb") as f:
            h.update(f.read())
    return h.hexdigest()


def needs_build() -> bool:
    if not os.path.exists(LIB) or not os.path.exists(STAMP):
        return True
    with open(STAMP) as f:
        return f.read().strip() != source_hash()


def build(force: bool = False, verbose: bool = False, jobs: int = 8) -> str:
    """Compile every csrc/*.cu for sm_100a and link libsa_b200.so."""
    if not force and not needs_build():
        return LIB
    nvcc = _nvcc()
    os.makedirs(BUILD_DIR, exist_ok=True)
    procs, objs = [], []
    for src in sources():
        obj = os.path.join(BUILD_DIR, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        cmd = [nvcc, *NVCC_FLAGS, "-I", os.path.join(ROOT, "include"), "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
        if len(procs) >= jobs:
            _drain(procs)
    _drain(procs)
    tmp = LIB + ".tmp"
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", tmp, *objs]
    if verbose:
        print(" ".join(cmd), flush=True)
    out = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if out.returncode != 0:
        raise RuntimeError("link failed:\n" + out.stdout)
    os.replace(tmp, LIB)
    with open(STAMP, "w") as f:
        f.write(source_hash() + "\n")
    return LIB


def _drain(procs):
    errors = []
    for cmd, p in procs:
        text = p.communicate()[0]
        if p.returncode != 0:
            errors.append(" ".join(cmd) + "\n" + text)
        elif text.strip():
            sys.stderr.write(text)
    procs.clear()
    if errors:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errors))


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
