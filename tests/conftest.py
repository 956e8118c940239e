"""Shared pytest configuration.

Tests marked ``gpu`` need a CUDA device and the built sm_100a library; the
rest run on CPU only (oracle vs. golden fixtures, host logic, the C-ABI symbol
table and the gloo multi-process paths).
"""

import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# every forward in the tests reads back the device status word of its launch
os.environ.setdefault("SA_CHECK_STATUS", "1")
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built CUDA library")


def load_golden(name):
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    d = {key: z[key] for key in z.files}
    d["meta"] = json.loads(bytes(d["meta"]).decode())
    return d


def golden_names():
    return sorted(f[:-4] for f in os.listdir(GOLDEN)
                  if f.endswith(".npz") and f not in ("misc.npz", "selections_full.npz")
                  and not f.startswith(("stream_", "segment_")))


def segment_golden_names():
    """Fixtures of the segment-mean variant (reference reps, exact attention at stride 1)."""
    return sorted(f[:-4] for f in os.listdir(GOLDEN) if f.startswith("segment_") and f.endswith(".npz"))


def stream_golden_names():
    """Fixtures of the streaming class (one update + query per token)."""
    return sorted(f[:-4] for f in os.listdir(GOLDEN) if f.startswith("stream_") and f.endswith(".npz"))
