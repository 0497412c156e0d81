"""Pins the oracle's op families to the reference's own kernel self-test (wgsl-ops-test.js:36-435):
every one of its 27 cases, same inputs, same CPU formulas, same gate (max |got - ref| < tol)."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import golden_cases

CASES = golden_cases()
UNARY = {"Sigmoid": 0, "Sqrt": 1, "Neg": 2, "Abs": 3, "SiLU": 8, "GELU": 9, "Erf": 10}
BINARY = {"Add": 0, "Sub": 1, "Mul": 2, "Div": 3, "Max": 5, "Min": 6}


def run_oracle(o, name, a):
    kind = name.split()[0]
    if kind == "unary":
        return o.unary(UNARY[name.split()[1]], a["X"])
    if kind == "binary":
        return o.binary(BINARY[name.split()[1]], a["A"], a["B"])
    if kind == "softmax":
        return o.softmax(a["X"], int(a["cfg"][0]), int(a["cfg"][1]))
    if kind == "instancenorm":
        C, HW, N = (int(v) for v in a["cfg"][:3])
        return o.instance_norm(a["X"], a["gamma"], a["beta"], C, HW, N)
    if kind == "matmul":
        M, N, K, bb = (int(v) for v in a["cfg"])
        return o.matmul(a["A"], a["B"], M, N, K, bb, int(a["batch"][0]))
    if kind == "conv2d":
        Ci, Co, H, W = (int(v) for v in a["cfg"])
        K = int(a["K"][0])
        return o.conv(a["X"], a["W"], a["bias"], 1, Ci, H, W, Co, K, 1, (K - 1) // 2).ravel()
    if kind == "layernorm":
        return o.layer_norm(a["X"], a["gamma"], a["beta"], int(a["cfg"][1]), int(a["cfg"][0]))
    if kind == "gemm":
        M, N, K, tb = (int(v) for v in a["cfg"])
        return o.gemm(a["A"], a["B"], a["C"], M, N, K, tb)
    if kind == "resize":
        return o.resize_nearest(a["X"], a["cfg"])
    if kind == "powScalar":
        return o.pow_scalar(a["X"], float(a["cfg"][0]))
    raise AssertionError(name)


def test_case_count():
    assert len(CASES) == 27


@pytest.mark.parametrize("name,tol,arrays", CASES, ids=[c[0] for c in CASES])
def test_oracle_matches_reference_selftest(oracle, name, tol, arrays):
    got = np.asarray(run_oracle(oracle, name, arrays), np.float64).ravel()
    ref = arrays["ref"].astype(np.float64).ravel()
    assert got.shape == ref.shape
    assert np.max(np.abs(got - ref)) < tol
