"""Shared fixtures. GPU tests carry @pytest.mark.gpu; everything else runs on a CPU-only box."""
from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def load_package():
    """Imports ming-tts_b200/ as module ``mingtts_b200``."""
    name = "mingtts_b200"
    if name in sys.modules:
        return sys.modules[name]
    pkg = os.path.join(ROOT, "ming-tts_b200")
    spec = importlib.util.spec_from_file_location(name, os.path.join(pkg, "__init__.py"),
                                                  submodule_search_locations=[pkg])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(scope="session")
def mt():
    return load_package()


@pytest.fixture(scope="session")
def oracle():
    import oracle as orc
    orc.lib()
    return orc


@pytest.fixture(scope="session")
def ctx(mt):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    c = mt.Context(0)
    yield c
    c.close()


def assert_close(got, want, atol, rtol=1e-4, what=""):
    """KernelTests.swift:58-68 style check: |got - want| <= atol + rtol |want| everywhere."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, f"{what}: shape {got.shape} vs {want.shape}"
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    d = np.abs(got - want)
    tol = atol + rtol * np.abs(want)
    bad = d > tol
    if bad.any():
        i = int(np.argmax(d - tol))
        raise AssertionError(f"{what}: {int(bad.sum())} of {d.size} out of tolerance; worst flat index {i} "
                             f"got {got.flat[i]:.7g} want {want.flat[i]:.7g} (atol {atol:.3g})")


def rel_err(got, want):
    """max |got - want| / max |want| (the relative error of the parity bar)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float(np.max(np.abs(got - want)) / max(np.max(np.abs(want)), 1e-30))


def cosine(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / max(np.linalg.norm(a) * np.linalg.norm(b), 1e-300))
