"""Build libsa_b200.so in-tree from csrc/*.cu for sm_100a.

    python -m streaming_attention_b200.build        # or build() from Python

The library is written next to this file so that it travels with the source
tree; objects go to ``_build/`` at the repository root.  Rebuilds only when the
sources, headers or flags differ from those the library was built from (a
content hash kept beside it, so that a copied tree with new file times does
not rebuild).

``build(checks=True)`` makes libsa_b200_checks.so, the same sources with
``-DSA_DEVICE_CHECKS``: device-side index checks that record a failure in the
launch status word and skip the access (the stand-in for a memory checker;
``SA_DEVICE_CHECKS=1`` in the environment makes the package load it).
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
LIB_CHECKS = os.path.join(PKG, "libsa_b200_checks.so")
BUILD_DIR = os.path.join(ROOT, "_build")
CHECKS_FLAGS = ["-DSA_DEVICE_CHECKS"]

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


def source_hash(checks: bool = False) -> str:
    h = hashlib.sha256()
    h.update(" ".join(NVCC_FLAGS + (CHECKS_FLAGS if checks else [])).encode())
    for p in sources() + headers() + [__file__]:
        h.update(os.path.relpath(p, ROOT).encode())
        with open(p, "rb") as f:
            h.update(f.read())
    return h.hexdigest()


def needs_build(checks: bool = False) -> bool:
    lib = LIB_CHECKS if checks else LIB
    stamp = lib + ".stamp"
    if not os.path.exists(lib) or not os.path.exists(stamp):
        return True
    with open(stamp) as f:
        return f.read().strip() != source_hash(checks)


def build(force: bool = False, verbose: bool = False, jobs: int = 8, checks: bool = False) -> str:
    """Compile every csrc/*.cu for sm_100a and link libsa_b200.so (or, with
    `checks`, libsa_b200_checks.so)."""
    lib = LIB_CHECKS if checks else LIB
    stamp = lib + ".stamp"
    if not force and not needs_build(checks):
        return lib
    nvcc = _nvcc()
    bdir = os.path.join(BUILD_DIR, "checks") if checks else BUILD_DIR
    os.makedirs(bdir, exist_ok=True)
    flags = NVCC_FLAGS + (CHECKS_FLAGS if checks else [])
    procs, objs = [], []
    for src in sources():
        obj = os.path.join(bdir, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        cmd = [nvcc, *flags, "-I", os.path.join(ROOT, "include"), "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
        if len(procs) >= jobs:
            _drain(procs)
    _drain(procs)
    tmp = lib + ".tmp"
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", tmp, *objs]
    if verbose:
        print(" ".join(cmd), flush=True)
    out = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if out.returncode != 0:
        raise RuntimeError("link failed:\n" + out.stdout)
    os.replace(tmp, lib)
    with open(stamp, "w") as f:
        f.write(source_hash(checks) + "\n")
    return lib


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
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv, checks=True))
