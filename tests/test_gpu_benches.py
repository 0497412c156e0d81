"""The runXBench drivers (draw-instant_b200/benches.py): reference result schema, naive and fused paths
agreeing, positive timings.  Naive = fp32 op-family sequence, fused = fp16 fused block."""
from __future__ import annotations

import importlib

import numpy as np
import pytest

from conftest import load_package

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def benches():
    load_package()
    m = importlib.import_module("draw_instant_b200.benches")
    m.REPEATS = 3
    m.WARM_MS = 50.0
    return m


@pytest.mark.parametrize("name,tol", [("conv", 2e-3), ("groupnorm", 1e-2), ("resnet", 5e-2), ("attn", 2e-3),
                                      ("cross-attn", 2e-3), ("tembed", 1e-3)])
def test_bench_schema_and_agreement(ctx, benches, name, tol):
    r = benches.ALL[name](lambda s: None)
    for k in ("naive", "fused", "speedup", "correctness", "dispatchesNaive", "dispatchesFused", "naiveRuns",
              "fusedRuns"):
        assert k in r, k
    assert r["naive"] > 0 and r["fused"] > 0 and abs(r["speedup"] - r["naive"] / r["fused"]) < 1e-9
    assert set(r["correctness"]) == {"maxAbsDiff", "l2"}
    assert np.isfinite(r["correctness"]["maxAbsDiff"]) and r["correctness"]["maxAbsDiff"] < tol, r["correctness"]
    assert len(r["naiveRuns"]) == 3 == len(r["fusedRuns"])
