"""The ONNX-graph executor on libdi: the SD-style test graph (as written and after the executor's graph
rewrites, from protobuf bytes) against the oracle-backed walk and an independent NumPy evaluation, with
pool reuse across runs (the fp32 op families hold the reference self-test's 1e-3 gates)."""
from __future__ import annotations

import copy
import importlib

import numpy as np
import pytest

from executor_cases import OracleBackend, encode_model, sd_graph, sd_graph_numpy

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float(np.abs(a - b).max() / np.abs(b).max())


@pytest.mark.parametrize("rewrite", [False, True])
def test_executor_on_libdi(ctx, dib, oracle, rewrite):
    E = importlib.import_module("draw_instant_b200.executor")
    G = importlib.import_module("draw_instant_b200.graph")
    P = importlib.import_module("draw_instant_b200.onnx_parser")
    graph, T, x = sd_graph(seed=5)
    g = P.parse_onnx_graph(encode_model(graph, T))
    if rewrite:
        G.fuse_silu_pattern(g)
        G.fuse_mul_add_pattern(g)
        assert G.fuse_group_norm_pattern(g)["fused"] == 1
    gpu = E.GpuBackend(ctx)
    ex = E.Executor(gpu, copy.deepcopy(g), E.WeightCache(gpu, g["tensors"]))
    out = ex.run({"x": x})
    host = OracleBackend(oracle, dib.UNARY, dib.BINARY)
    ex_h = E.Executor(host, copy.deepcopy(g), E.WeightCache(host, g["tensors"]))
    out_h = ex_h.run({"x": x})
    ref = sd_graph_numpy(T, x)
    for k in ("y", "z"):
        got = gpu.read(out[k].buf, out[k].numel * 4).reshape(out[k].dims)
        hv = host.read(out_h[k].buf, out_h[k].numel * 4).reshape(out_h[k].dims)
        assert np.all(np.isfinite(got))
        assert _rel(got, ref[k]) < 1e-3, k
        assert _rel(got, hv) < 1e-3, k
    allocs = ex.pool.allocs
    out2 = ex.run({"x": x})
    assert ex.pool.allocs == allocs and ex.pool.live == 0
    assert np.array_equal(gpu.read(out2["y"].buf, out2["y"].numel * 4),
                          gpu.read(out["y"].buf, out["y"].numel * 4))
    assert ctx.fault() == 0
