"""Shared fixtures. `-m "not gpu"` runs on any host; `-m gpu` needs a B200.

The oracle (oracle/) is the checker: tests compare the CUDA path, called
through the C ABI, against it and against the reference's own compiled
sources (oracle/_ref/), and pin the oracle against the golden vectors the
reference produced (tests/golden/).
"""
import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    # build once per session (no-ops when the outputs are newer than the sources)
    from hako_b200 import build as hb
    hb.build_synth()
    hb.build_tok()
    hb.build_cuda()
    from oracle import oracle as orc
    orc.build(ref=True)


def golden_npz(name):
    return np.load(os.path.join(GOLDEN, name))


def golden_json(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


def have_reference():
    from oracle.oracle import REF_SO
    return os.path.exists(REF_SO)


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    if not have_reference():
        pytest.skip("reference build (oracle/_ref) not present")
    from oracle.oracle import Reference
    return Reference()


@pytest.fixture(scope="session")
def cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def first_divergence(ours, ref):
    for i, (a, b) in enumerate(zip(ours, ref)):
        if a != b:
            return i
    return None
