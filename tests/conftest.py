"""pytest configuration: the ``gpu`` marker and shared fixtures.

Tests marked ``gpu`` need a B200 (sm_100a) and the built CUDA library; every
other test runs on the CPU.
"""

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU and the built akv_b200 library")


def golden(name):
    return np.load(os.path.join(GOLDEN, name + ".npz"))


def golden_cases(z, section="in"):
    names = sorted({k.split("/")[0] for k in z.files})
    return names
