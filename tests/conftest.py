"""Shared test set-up.

* registers the ``gpu`` marker (tests that need a B200; run with ``-m gpu``)
* puts the package (``stablediffusion-cpp_b200/``), ``oracle/`` and the repo root on
  sys.path
* fixtures: ``orc`` (C restatement of the reference CPU path), ``ref`` (the reference
  CPU path compiled from its sources, skipped where it was not built), ``sdb`` (the
  sdb200 binding; GPU tests only)
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "stablediffusion-cpp_b200")
ORACLE = os.path.join(ROOT, "oracle")
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, PKG, ORACLE, GOLDEN):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


@pytest.fixture(scope="session")
def orc():
    from oracle import Oracle

    return Oracle()


@pytest.fixture(scope="session")
def ref():
    from oracle import RefCPU

    if not RefCPU.available():
        pytest.skip("reference CPU library oracle/_ref/libsdref.so not built here")
    return RefCPU()


@pytest.fixture(scope="session")
def sdb():
    import torch

    import sdb200

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but torch sees no CUDA device")
    if not sdb200.available():
        pytest.fail("libsdb200 reports no usable sm_100 device: " + sdb200.lib().sdb200_last_error().decode())
    torch.cuda.init()
    return sdb200


def rel_fro(a, b) -> float:
    """Relative Frobenius error ||a - b|| / ||b|| in float64."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))


def load_golden(name):
    return np.load(os.path.join(GOLDEN, name + ".npz"))
