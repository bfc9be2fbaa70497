"""Shared fixtures. GPU tests carry @pytest.mark.gpu; everything else runs on CPU.

The library under test is llamini.cpp_b200/lib/libllamini_cuda.so (loaded with
ctypes through the package binding); the checker is the CPU oracle in oracle/
(and, where it was built, the reference's own code in oracle/_ref/).
"""
from __future__ import annotations

import importlib.util
import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, GOLDEN)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


def _load_pkg():
    name = "llamini_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, os.path.join(ROOT, "llamini.cpp_b200", "__init__.py"))
    m = importlib.util.module_from_spec(spec)
    sys.modules[name] = m
    spec.loader.exec_module(m)
    return m


def _ensure_built():
    so = os.path.join(ROOT, "llamini.cpp_b200", "lib", "libllamini_cuda.so")
    if not os.path.exists(so):
        spec = importlib.util.spec_from_file_location("llamini_b200_build", os.path.join(ROOT, "llamini.cpp_b200", "build.py"))
        b = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(b)
        b.build()
    if not os.path.exists(os.path.join(ROOT, "oracle", "liboracle.so")):
        subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), "all"], check=True, capture_output=True)


@pytest.fixture(scope="session")
def lm():
    _ensure_built()
    return _load_pkg()


@pytest.fixture(scope="session")
def orc():
    _ensure_built()
    import oracle
    return oracle


@pytest.fixture(scope="session")
def tiny():
    import tiny as t
    return t


@pytest.fixture(scope="session")
def synth():
    import tiny as t
    return t.synthetic()


@pytest.fixture(scope="session")
def golden():
    import json
    g = {"dequant": np.load(os.path.join(GOLDEN, "dequant.npz")),
         "kat": json.load(open(os.path.join(GOLDEN, "kat.json"))),
         "tokens": json.load(open(os.path.join(GOLDEN, "tokens.json"))),
         "logits": np.load(os.path.join(GOLDEN, "logits.npz"))}
    return g


@pytest.fixture(scope="session")
def gpu(lm):
    """The library, on a machine with a usable device."""
    if lm.lib().llamini_device_count() <= 0:
        pytest.fail("GPU test without a CUDA device")
    return lm


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    d = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (d if d > 0 else 1.0))


def same_bits(a: np.ndarray, b: np.ndarray) -> bool:
    """Bit-identical f32 arrays, except that any NaN matches any NaN (NaN
    payloads are not preserved by arithmetic on either side)."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    na, nb = np.isnan(a), np.isnan(b)
    if not np.array_equal(na, nb):
        return False
    return np.array_equal(a[~na].view(np.uint32), b[~nb].view(np.uint32))
