"""Shared fixtures of the test suite.

Tests marked ``gpu`` need a B200 and the built libdianoia_b200.so; the rest
run on any CPU (oracle against the golden fixtures, the C-ABI's exports,
host-side logic, gloo ranks for the multi-GPU host logic).
"""
from __future__ import annotations

import glob
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA sm_100 device and the built library")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as orc
    return orc.Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle import oracle as orc
    if not os.path.exists(orc.REF_SO):
        pytest.skip("oracle/_ref/libref_lab.so is not built here")
    return orc.Reference()


def golden_names(kind: str = "linear"):
    names = []
    for path in sorted(glob.glob(os.path.join(GOLDEN, "*.npz"))):
        with np.load(path) as z:
            if str(z["kind"]) == kind:
                names.append(os.path.basename(path)[:-4])
    return names


def load_golden(name: str) -> dict:
    with np.load(os.path.join(GOLDEN, name + ".npz")) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def cuda_lib():
    """The built library on a machine with a usable device (gpu tests only)."""
    import dianoia_b200
    from dianoia_b200 import build as b
    if not os.path.exists(dianoia_b200.LIB_PATH):
        b.build()
    L = dianoia_b200.lib()
    assert L.lab_cpu_supported() == 1, "no sm_100 device visible to the library"
    return L
