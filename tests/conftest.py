"""Shared fixtures: the product package (loaded from the hyphenated draw-instant_b200/ directory), the CPU
oracle, and a libdi context on cuda:0 for tests marked `gpu`."""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def load_package():
    """Imports draw-instant_b200/ as the package `draw_instant_b200`."""
    name = "draw_instant_b200"
    if name in sys.modules:
        return sys.modules[name]
    pkg_dir = ROOT / "draw-instant_b200"
    spec = importlib.util.spec_from_file_location(name, pkg_dir / "__init__.py",
                                                  submodule_search_locations=[str(pkg_dir)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built libdi.so")


@pytest.fixture(scope="session")
def dib():
    return load_package()


@pytest.fixture(scope="session")
def oracle():
    import oracle as o
    o.build()
    return o


@pytest.fixture(scope="session")
def ctx(dib):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    c = dib.Context(0)
    yield c
    assert c.fault() == 0, "a kernel reported a timed-out wait"
    c.close()


def rel_err(got, ref):
    """max|got - ref| / max|ref| — the per-block tolerance metric (max-relative-error 1e-2)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(got - ref)) / max(np.max(np.abs(ref)), 1e-30))


def cosine(got, ref):
    a = np.asarray(got, np.float64).ravel()
    b = np.asarray(ref, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))


GOLDEN = ROOT / "tests" / "golden"


def golden_cases():
    """The 27 wgsl-ops-test.js known-answer cases: [(name, tol, {array name: array})]."""
    z = np.load(GOLDEN / "wgsl_ops_cases.npz")
    out = []
    for name in z["names"]:
        name = str(name)
        arrays = {k.split("|", 1)[1]: z[k] for k in z.files if k.startswith(name + "|")}
        out.append((name, float(arrays.pop("tol")[0]), arrays))
    return out
