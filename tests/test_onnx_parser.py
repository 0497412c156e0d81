"""ONNX reader (draw-instant_b200/onnx_parser.py) against the reference's synthetic protobuf fixture
(onnx-parser-test.mjs: ModelProto with one MatMul node, one [2,3] float initializer, graph input/output,
opset import) plus the wire-format cases the parser handles (packed fields, attributes, value-info dims,
fp16 initializers, desync recovery)."""
from __future__ import annotations

import importlib
import struct

import numpy as np
import pytest

from conftest import load_package


@pytest.fixture(scope="module")
def P():
    load_package()
    return importlib.import_module("draw_instant_b200.onnx_parser")


# protobuf encoders restated from onnx-parser-test.mjs:7-26
def varint(n):
    out = bytearray()
    n &= (1 << 64) - 1
    while n > 0x7F:
        out.append((n & 0x7F) | 0x80)
        n >>= 7
    out.append(n)
    return bytes(out)


def tag(field, wire):
    return varint((field << 3) | wire)


def ld(field, payload):
    return tag(field, 2) + varint(len(payload)) + payload


def s(field, text):
    return ld(field, text.encode())


def vint(field, n):
    return tag(field, 0) + varint(n)


def tensor(name, dims, dtype, raw, packed=False):
    out = ld(1, b"".join(varint(d) for d in dims)) if packed else b"".join(vint(1, d) for d in dims)
    return out + vint(2, dtype) + s(8, name) + ld(9, raw)


def node(inputs, outputs, op, attrs=b"", name=""):
    return b"".join(s(1, i) for i in inputs) + b"".join(s(2, o) for o in outputs) + (s(3, name) if name else b"") + \
        s(4, op) + attrs


def reference_fixture():
    raw = bytearray(24)
    struct.pack_into("<ff", raw, 0, 1.5, -2.25)
    graph = ld(1, node(["a", "w1"], ["y"], "MatMul")) + ld(5, tensor("w1", [2, 3], 1, bytes(raw))) + \
        ld(11, s(1, "a")) + ld(12, s(1, "y"))
    return vint(1, 8) + s(2, "draw.instant.test") + ld(7, graph) + ld(8, vint(2, 17))


def test_reference_fixture(P):
    buf = reference_fixture()
    g = P.parse_onnx_graph(buf)
    assert len(g["tensors"]) == 1 and len(g["nodes"]) == 1
    assert g["nodes"][0]["op_type"] == "MatMul" and g["nodes"][0]["inputs"] == ["a", "w1"]
    assert g["tensors"]["w1"]["dims"] == [2, 3] and g["tensors"]["w1"]["dtype"] == "float32"
    assert struct.unpack_from("<ff", g["tensors"]["w1"]["data"]) == (1.5, -2.25)
    assert [v["name"] for v in g["inputs"]] == ["a"] and [v["name"] for v in g["outputs"]] == ["y"]
    assert g["opHist"] == {"MatMul": 1} and g["bytes"] == 24
    w = P.parse_onnx_weights(buf)
    assert w["count"] == 1 and w["bytes"] == 24


def test_attributes_value_info_and_packed(P):
    attrs = ld(5, s(1, "axes") + ld(8, varint(1) + varint(-1)) + vint(20, 7)) + \
        ld(5, s(1, "epsilon") + tag(2, 5) + struct.pack("<f", 1e-5)) + \
        ld(5, s(1, "value") + ld(5, tensor("c", [3], 7, struct.pack("<qqq", 1, 16, -1))))
    vi = s(1, "x") + ld(2, ld(1, vint(1, 10) + ld(2, ld(1, vint(1, 2)) + ld(1, s(2, "N")) + ld(1, vint(1, 64)))))
    half = np.array([1.0, -0.5, 65504.0, 2.0 ** -24], np.float16).tobytes()
    graph = ld(1, node(["x"], ["y"], "Constant", attrs, name="/c")) + \
        ld(5, tensor("h", [2, 2], 10, half, packed=True)) + ld(11, vi)
    g = P.parse_onnx_graph(vint(1, 8) + ld(7, graph))
    n = g["nodes"][0]
    a = {x["name"]: x for x in n["attributes"]}
    assert n["name"] == "/c" and a["axes"]["ints"] == [1, -1] and a["axes"]["type"] == 7
    assert abs(a["epsilon"]["f"] - 1e-5) < 1e-12
    assert a["value"]["t"]["dtype"] == "int64" and struct.unpack("<qqq", a["value"]["t"]["data"]) == (1, 16, -1)
    assert g["inputs"][0] == {"name": "x", "dtype": 10, "dims": [2, -1, 64]}
    t = g["tensors"]["h"]
    assert t["dims"] == [2, 2] and t["dtype"] == "float16"
    fn = P.weight_fn(g)
    np.testing.assert_array_equal(fn("h", 4), np.array([1.0, -0.5, 65504.0, 2.0 ** -24], np.float32))
    assert fn("h", 5) is None and fn("missing", 4) is None


def test_float_data_field(P):
    t = P.parse_tensor(b := (vint(1, 2) + vint(2, 1) + s(8, "f") + ld(4, struct.pack("<ff", 3.0, 4.0))), 0, len(b))
    assert t["data"] == struct.pack("<ff", 3.0, 4.0)


def test_recovers_graph_after_top_level_desync(P):
    # a corrupt top-level field (wire type 7) before the graph: the reader falls back to the 0x3a scan
    buf = tag(3, 7) + reference_fixture()
    g = P.parse_onnx_graph(buf)
    assert "w1" in g["tensors"] and g["nodes"] and g["nodes"][0]["op_type"] == "MatMul"


def test_initializer_scan_finds_tensors_after_graph_desync(P):
    raw = np.arange(6, dtype=np.float32).tobytes()
    graph = ld(5, tensor("good", [2, 3], 1, raw)) + tag(2, 6) + ld(5, tensor("later", [6], 1, raw))
    g = P.parse_onnx_graph(ld(7, graph))
    assert set(g["tensors"]) == {"good", "later"}  # the walk stops at wire 6; the 0x2a scan finds 'later'
