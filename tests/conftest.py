"""pytest configuration: the ``gpu`` marker and shared fixtures.

Tests marked ``gpu`` need a B200 (sm_100a) and the built CUDA library; every
other test runs on the CPU.
"""

import importlib.util
import os
import sys
import types

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


SG = os.path.join(ROOT, "baseline", "_ref", "akv", "system", "sglang")


@pytest.fixture(scope="module")
def reference_backend():
    """The reference's unmodified ``context_backend.py`` (with its
    ``occurrence.py`` and ``request_storage.py``) loaded from the reference
    package installed in baseline/_ref, its kernel modules bound to this
    package; skips when the package is not installed."""
    path = os.path.join(SG, "srt", "layers", "attention", "context_backend.py")
    if not os.path.exists(path):
        pytest.skip("the reference package is not installed in baseline/_ref")
    from akv_b200 import context_page_table, context_reposition

    saved = {k: v for k, v in sys.modules.items() if k == "sglang" or k.startswith("sglang.")}
    for pkg in ("sglang", "sglang.kernels", "sglang.kernels.ops", "sglang.kernels.ops.attention",
                "sglang.srt", "sglang.srt.context_system", "sglang.srt.layers",
                "sglang.srt.layers.attention"):
        sys.modules[pkg] = types.ModuleType(pkg)
    sys.modules["sglang.kernels.ops.attention.context_reposition"] = context_reposition
    sys.modules["sglang.kernels.ops.attention.context_page_table"] = context_page_table

    def load(name, rel):
        spec = importlib.util.spec_from_file_location(name, os.path.join(SG, rel))
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
        return mod

    load("sglang.srt.context_system.request_storage", "srt/context_system/request_storage.py")
    load("sglang.srt.context_system.occurrence", "srt/context_system/occurrence.py")
    mod = load("sglang.srt.layers.attention.context_backend",
               "srt/layers/attention/context_backend.py")
    yield mod
    for k in [k for k in sys.modules if k == "sglang" or k.startswith("sglang.")]:
        del sys.modules[k]
    sys.modules.update(saved)
