"""Device-side index checks: libsa_b200_checks.so, the build with -DSA_DEVICE_CHECKS.

A failed check records its code (900..999) in the launch status word and the
offending index beside it, and skips the access it guards; sa_workspace_status
then returns SA_ERR_DEVICE_CHECK.  This is the stand-in for a memory checker:
the GPU parity tests run again on the checks build with every call's status
read back, and one bad index planted on the host (a perms-table entry outside
its block) must come back as SA_ERR_DEVICE_CHECK.
"""

import ctypes
import os
import subprocess
import sys

import pytest

from conftest import ROOT
from test_capi import declared_symbols

PKG = os.path.join(ROOT, "streaming_attention_b200")
CHECKS_LIB = os.path.join(PKG, "libsa_b200_checks.so")


def _env():
    env = dict(os.environ)
    env["SA_DEVICE_CHECKS"] = "1"
    env["SA_CHECK_STATUS"] = "1"
    env["PYTHONPATH"] = ROOT + os.pathsep + env.get("PYTHONPATH", "")
    return env


def test_checks_build_exports_every_declared_symbol():
    assert os.path.exists(CHECKS_LIB), "build() makes libsa_b200_checks.so beside libsa_b200.so"
    lib = ctypes.CDLL(CHECKS_LIB)
    for s in declared_symbols():
        assert hasattr(lib, s), f"{s} missing from the checks build"
    assert lib.sa_device_checks_enabled() == 1
    assert ctypes.CDLL(os.path.join(PKG, "libsa_b200.so")).sa_device_checks_enabled() == 0


def test_environment_selects_the_checks_build():
    code = ("from streaming_attention_b200 import _lib; "
            "assert _lib.LIB_PATH.endswith('libsa_b200_checks.so'), _lib.LIB_PATH; "
            "assert _lib.load().sa_device_checks_enabled() == 1")
    subprocess.run([sys.executable, "-c", code], env=_env(), check=True, timeout=120)


@pytest.mark.gpu
def test_parity_suite_passes_on_the_checks_build():
    # the config-shaped, golden-fixture, edge-shape and determinism cases; the
    # full-length ones are left to the ordinary build
    r = subprocess.run([sys.executable, "-m", "pytest", os.path.join(ROOT, "tests", "test_gpu_parity.py"),
                        "-m", "gpu", "-x", "-q", "-p", "no:cacheprovider", "-k", "not full_length and not full_size"],
                       env=_env(), cwd=ROOT, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert " passed" in r.stdout


PLANTED = r"""
import torch
import streaming_attention_b200 as sa
from streaming_attention_b200 import _lib, fast

assert _lib.load().sa_device_checks_enabled() == 1, "not the checks build"
bs = 64
orig = fast.draw_tables


def planted(**kw):
    t = orig(**dict(kw, cache=False))   # a copy of its own: the cached tables stay intact
    t.perms[0, 1, 3] = bs + 5           # a key index outside its block
    return t


fast.draw_tables = planted
g = torch.Generator().manual_seed(0)
q, k, v = (torch.randn(1, 2, 300, 32, generator=g).cuda() for _ in range(3))
try:
    sa.fast_article_causal_attention(q, k, v, degree=2, block_size=bs, scale=None, compressor="random", seed=0)
except _lib.SAError as e:
    assert "device check 901" in str(e) and "status -6" in str(e), str(e)
    print("planted index caught:", e)
else:
    raise SystemExit("the planted index was not reported")
# the context is still usable and an ordinary call is clean
fast.draw_tables = orig
out = sa.fast_article_causal_attention(q, k, v, degree=2, block_size=bs, scale=None, compressor="random", seed=0)
torch.cuda.synchronize()
assert torch.isfinite(out).all()
"""


@pytest.mark.gpu
def test_planted_bad_index_is_reported_and_skipped():
    r = subprocess.run([sys.executable, "-c", PLANTED], env=_env(), cwd=ROOT, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-3000:]
    assert "planted index caught" in r.stdout
