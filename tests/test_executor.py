"""The ONNX-graph executor's host logic, on the CPU: the walk over an SD-style graph with the oracle as
the device (against an independent NumPy evaluation), the same graph after the executor's rewrites and
after a protobuf round trip, tensor lifetimes and pool reuse across runs, the host shape path, graph-IO
inference and op coverage (wgsl-executor.js:45-94, 129-1114, 1205-1467)."""
from __future__ import annotations

import copy
import importlib

import numpy as np
import pytest

from executor_cases import OracleBackend, encode_model, sd_graph, sd_graph_numpy


@pytest.fixture(scope="module")
def E(dib):
    return importlib.import_module("draw_instant_b200.executor")


@pytest.fixture()
def backend(dib, oracle):
    return OracleBackend(oracle, dib.UNARY, dib.BINARY)


def _run(E, backend, graph, tensors, x):
    ex = E.Executor(backend, copy.deepcopy(graph), E.WeightCache(backend, tensors))
    out = ex.run({"x": x})
    res = {k: backend.read(t.buf, t.numel * 4).reshape(t.dims) for k, t in out.items()}
    return ex, res


def _rel(a, b):
    return float(np.abs(a - b).max() / np.abs(b).max())


def test_sd_graph_matches_numpy(E, backend):
    graph, T, x = sd_graph()
    ex, res = _run(E, backend, graph, T, x)
    ref = sd_graph_numpy(T, x)
    assert res["y"].shape == (1, 8, 8, 8) and res["z"].shape == (1, 10)
    assert _rel(res["y"], ref["y"]) < 1e-4
    assert _rel(res["z"], ref["z"]) < 1e-4
    assert ex.op_hist["Conv"] == 3 and ex.op_hist["Shape"] == 3


def test_rewritten_graph_same_result(E, backend, dib):
    """fuseSiluPattern / fuseMulAddPattern / fuseGroupNormPattern, then the walk: same outputs."""
    G = importlib.import_module("draw_instant_b200.graph")
    graph, T, x = sd_graph()
    g2 = copy.deepcopy(graph)
    g2["tensors"] = T
    G.fuse_silu_pattern(g2)
    G.fuse_mul_add_pattern(g2)
    assert G.fuse_group_norm_pattern(g2)["fused"] == 1
    ops = [n["op_type"] for n in g2["nodes"]]
    assert "Silu" in ops and "Sigmoid" not in ops and "GroupNorm" in ops and "InstanceNormalization" not in ops
    _, a = _run(E, backend, graph, T, x)
    _, b = _run(E, backend, g2, T, x)
    for k in a:
        assert _rel(b[k], a[k]) < 1e-5


def test_protobuf_round_trip(E, backend, dib):
    P = importlib.import_module("draw_instant_b200.onnx_parser")
    graph, T, x = sd_graph()
    g = P.parse_onnx_graph(encode_model(graph, T))
    assert [n["op_type"] for n in g["nodes"]] == [n["op_type"] for n in graph["nodes"]]
    assert set(g["tensors"]) == set(T)
    ex = E.Executor(backend, g, E.WeightCache(backend, g["tensors"]))
    out = ex.run({"x": x})
    ref = sd_graph_numpy(T, x)
    for k in ("y", "z"):
        t = out[k]
        assert _rel(backend.read(t.buf, t.numel * 4).reshape(t.dims), ref[k]) < 1e-4


def test_lifetimes_and_pool_reuse(E, backend):
    """Intermediates go back to the pool after each run; a second run allocates nothing new except the
    output snapshots; outputs of run 1 are not overwritten by run 2."""
    graph, T, x = sd_graph()
    ex = E.Executor(backend, copy.deepcopy(graph), E.WeightCache(backend, T))
    o1 = ex.run({"x": x})
    y1 = backend.read(o1["y"].buf, o1["y"].numel * 4).copy()
    allocs1 = ex.pool.allocs
    live1 = ex.pool.live
    o2 = ex.run({"x": x * 2})
    assert ex.pool.allocs == allocs1          # everything the walk acquired went back to the pool
    assert ex.pool.live == live1 == 0
    assert np.array_equal(backend.read(o1["y"].buf, o1["y"].numel * 4), y1)   # snapshots are stable
    assert o1["y"].buf is not o2["y"].buf
    assert not ex.pool.owns(o1["y"].buf)


def test_buffer_pool_classes(E, backend):
    pool = E.BufferPool(backend)
    a = pool.acquire(10)
    assert backend.nbytes(a) == 4096 and pool.live == 1 and pool.allocs == 1
    pool.release(a)
    b = pool.acquire(4000)
    assert b is a and pool.allocs == 1
    c = pool.acquire(4097)
    assert backend.nbytes(c) == 8192 and pool.peak == 2
    foreign = backend.alloc(4096)
    pool.release(foreign)  # not ours: ignored
    assert pool.live == 2


def test_shape_path_stays_on_host(E, backend):
    """Shape -> Gather -> Unsqueeze -> Concat -> Reshape builds the target shape on the host."""
    from executor_cases import _n, _t
    T = {"i0": _t("i0", np.array(0), "int64"), "m1": _t("m1", np.array([-1]), "int64")}
    nodes = [_n("Shape", ["x"], ["s"]), _n("Gather", ["s", "i0"], ["b"], axis=0),
             _n("Unsqueeze", ["b"], ["bu"], axes=[0]), _n("Concat", ["bu", "m1"], ["tgt"], axis=0),
             _n("Reshape", ["x", "tgt"], ["y"]), _n("Mul", ["bu", "bu"], ["b2"])]
    graph = {"nodes": nodes, "inputs": [{"name": "x"}], "outputs": [{"name": "y"}, {"name": "b2"}]}
    ex = E.Executor(backend, graph, E.WeightCache(backend, T))
    x = np.arange(24, dtype=np.float32).reshape(2, 3, 4)
    out = ex.run({"x": x})
    assert out["y"].dims == [2, 12]
    assert np.array_equal(backend.read(out["y"].buf, 96).reshape(2, 12), x.reshape(2, 12))
    assert out["b2"].buf is None and list(out["b2"].cpu_data) == [4]


def test_infer_io_and_coverage(E):
    nodes = [{"inputs": ["a", "w"], "outputs": ["b"], "op_type": "MatMul", "name": "m", "attributes": []},
             {"inputs": ["b"], "outputs": ["c"], "op_type": "Fancy", "name": "f", "attributes": []}]
    ins, outs = E.infer_graph_io(nodes, {"w"})
    assert ins == [{"name": "a"}] and outs == [{"name": "c"}]
    cov = E.plan_execution({"nodes": nodes})
    assert cov["supportedCount"] == 1 and cov["unsupportedOps"] == [("Fancy", 1)]


def test_unsupported_op_and_missing_tensor(E, backend, dib):
    graph = {"nodes": [{"inputs": ["x"], "outputs": ["y"], "op_type": "Fancy", "name": "f", "attributes": []}],
             "inputs": [{"name": "x"}], "outputs": [{"name": "y"}]}
    ex = E.Executor(backend, graph, E.WeightCache(backend, {}))
    with pytest.raises(dib.DIError, match="unsupported op @0: Fancy"):
        ex.run({"x": np.zeros(4, np.float32)})
    graph = {"nodes": [{"inputs": ["q"], "outputs": ["y"], "op_type": "Sigmoid", "name": "s", "attributes": []}],
             "inputs": [{"name": "x"}], "outputs": [{"name": "y"}]}
    ex = E.Executor(backend, graph, E.WeightCache(backend, {}))
    with pytest.raises(dib.DIError, match="tensor not found"):
        ex.run({"x": np.zeros(4, np.float32)})


def test_timestep_expand_lowering_stays_on_host(E, backend):
    """torch.onnx lowers `timesteps.expand(sample.shape[0])` to Shape -> Gather -> Unsqueeze ->
    ConstantOfShape(int64) -> Mul -> Equal -> Where -> Expand; all of it must stay host metadata
    (wgsl-executor.js:249-287, 542-573), and the float timestep then promotes into a device op."""
    from executor_cases import _n, _t
    one = _t("one", np.array([1]), "int64")
    T = {"i0": _t("i0", np.array(0), "int64"), "neg1": _t("neg1", np.array([-1]), "int64"),
         "w": _t("w", np.ones((1, 3), np.float32))}
    nodes = [_n("Shape", ["sample"], ["s"]), _n("Gather", ["s", "i0"], ["b"], axis=0),
             _n("Unsqueeze", ["b"], ["bu"], axes=[0]),
             _n("ConstantOfShape", ["bu"], ["c"], value=one),
             _n("Mul", ["c", "neg1"], ["m"]), _n("Equal", ["bu", "m"], ["e"]),
             _n("Where", ["e", "c", "bu"], ["shape"]), _n("Expand", ["t", "shape"], ["te"]),
             _n("Cast", ["te"], ["tf"], to=1), _n("Unsqueeze", ["tf"], ["tf2"], axes=[1]),
             _n("MatMul", ["tf2", "w"], ["y"])]
    graph = {"nodes": nodes, "inputs": [{"name": "sample"}, {"name": "t"}], "outputs": [{"name": "y"}]}
    ex = E.Executor(backend, graph, E.WeightCache(backend, T))
    t = E.Tensor(None, [1], "int64", np.array([999], np.int64), True)
    out = ex.run({"sample": np.zeros((1, 4, 8, 8), np.float32), "t": t})
    y = backend.read(out["y"].buf, 12)
    assert out["y"].dims == [1, 3] and np.allclose(y, 999.0)
