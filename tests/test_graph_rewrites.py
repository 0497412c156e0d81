"""Graph rewrites (draw-instant_b200/graph.py) against the reference's fusion regression fixture
(fusion-test.mjs: the GroupNorm pattern must fuse exactly once with constants as Constant nodes AND as
initializers) and the node lists wgsl-executor.js:795-1006 produce (bit-exact: names, order, attrs)."""
from __future__ import annotations

import importlib
import struct

import numpy as np
import pytest

from conftest import load_package


@pytest.fixture(scope="module")
def G():
    load_package()
    return importlib.import_module("draw_instant_b200.graph")


def f32(vals):
    return {"dtype": "float32", "dims": [len(vals)], "data": np.asarray(vals, "<f4").tobytes()}


def mk(op, name, inputs, outputs, attributes=None):
    return {"op_type": op, "name": name, "inputs": inputs, "outputs": outputs, "attributes": attributes or []}


def gn_fixture(const_as_initializer: bool):
    # fusion-test.mjs:20-40
    tensors = {"shape0": {"dtype": "int64", "dims": [3], "data": bytes(24)},
               "shape1": {"dtype": "int64", "dims": [4], "data": bytes(32)},
               "gamma": f32([1, 1]), "beta": f32([0, 0])}
    nodes = [mk("Reshape", "/r0", ["X", "shape0"], ["r0"]),
             mk("InstanceNormalization", "/in", ["r0", "sc", "bi"], ["inout"], [{"name": "epsilon", "f": 1e-5}]),
             mk("Reshape", "/r1", ["inout", "shape1"], ["r1"]),
             mk("AffineBcast", "/aff", ["r1", "gamma", "beta"], ["Y"])]
    if const_as_initializer:
        tensors["sc"] = f32([1, 1])
        tensors["bi"] = f32([0, 0])
    else:
        nodes = [mk("Constant", "/c_sc", [], ["sc"], [{"name": "value", "t": f32([1, 1])}]),
                 mk("Constant", "/c_bi", [], ["bi"], [{"name": "value", "t": f32([0, 0])}])] + nodes
    return {"nodes": nodes, "tensors": tensors, "outputs": [{"name": "Y"}]}


@pytest.mark.parametrize("as_init", [False, True], ids=["constant-nodes", "initializers"])
def test_group_norm_fixture_fuses_once(G, as_init):
    g = gn_fixture(as_init)
    before = len(g["nodes"])
    assert G.fuse_group_norm_pattern(g) == {"fused": 1}
    assert len(g["nodes"]) == before - 3
    gn = g["nodes"][-1]
    assert gn == {"op_type": "GroupNorm", "name": "/aff_gn", "inputs": ["X", "gamma", "beta"], "outputs": ["Y"],
                  "attributes": [{"name": "num_groups", "i": 32}, {"name": "epsilon", "f": 1e-5}]}


def test_group_norm_reads_groups_from_constant_and_rejects_non_identity(G):
    g = gn_fixture(False)
    g["tensors"].pop("shape0")
    g["nodes"].insert(0, mk("Constant", "/c_shape", [], ["shape0"],
                            [{"name": "value", "t": {"dtype": "int64", "dims": [3],
                                                     "data": struct.pack("<qqq", 1, 16, -1)}}]))
    assert G.fuse_group_norm_pattern(g)["fused"] == 1
    assert g["nodes"][-1]["attributes"][0] == {"name": "num_groups", "i": 16}
    g2 = gn_fixture(True)
    g2["tensors"]["sc"] = f32([1, 2])  # not all ones -> untouched
    assert G.fuse_group_norm_pattern(g2)["fused"] == 0 and len(g2["nodes"]) == 4
    g3 = gn_fixture(True)
    g3["nodes"].append(mk("Relu", "/tap", ["inout"], ["t"]))  # IN output has a second consumer
    assert G.fuse_group_norm_pattern(g3)["fused"] == 0


def test_f16_initializers_resolve(G):
    g = gn_fixture(True)
    g["tensors"]["sc"] = {"dtype": "float16", "dims": [2], "data": np.array([1, 1], "<f2").tobytes()}
    g["tensors"]["bi"] = {"dtype": "float16", "dims": [2], "data": np.array([0, -0.0], "<f2").tobytes()}
    assert G.fuse_group_norm_pattern(g)["fused"] == 1


def test_silu_pattern(G):
    g = {"nodes": [mk("Conv", "c", ["x", "w"], ["h"]), mk("Sigmoid", "s", ["h"], ["sg"]),
                   mk("Mul", "m", ["sg", "h"], ["y"]), mk("Sigmoid", "s2", ["h"], ["sg2"]),
                   mk("Mul", "m2", ["h", "sg2"], ["y2"]), mk("Add", "a", ["sg2", "y2"], ["z"])],
         "outputs": [{"name": "y"}, {"name": "z"}]}
    assert G.fuse_silu_pattern(g) == {"fused": 1}  # sg2 has two consumers -> second pair stays
    assert [n["op_type"] for n in g["nodes"]] == ["Conv", "Silu", "Sigmoid", "Mul", "Add"]
    assert g["nodes"][1] == {"op_type": "Silu", "name": "m_fused", "inputs": ["h"], "outputs": ["y"], "attributes": []}


def test_mul_add_pattern_then_group_norm(G):
    # Reshape -> IN -> Reshape -> Mul(gamma) -> Add(beta): mul-add first, then the GroupNorm pass
    g = gn_fixture(True)
    g["nodes"][-1] = mk("Mul", "/mul", ["r1", "gamma"], ["mo"])
    g["nodes"].append(mk("Add", "/add", ["mo", "beta"], ["Y"]))
    assert G.fuse_group_norm_pattern(g)["fused"] == 0
    assert G.fuse_mul_add_pattern(g) == {"fused": 1}
    assert g["nodes"][-1] == {"op_type": "AffineBcast", "name": "/mul_affinefused", "inputs": ["r1", "gamma", "beta"],
                              "outputs": ["Y"], "attributes": []}
    assert G.fuse_group_norm_pattern(g)["fused"] == 1
    assert [n["op_type"] for n in g["nodes"]] == ["GroupNorm"]


def test_mul_add_needs_matching_shapes(G):
    g = {"nodes": [mk("Mul", "m", ["x", "g"], ["t"]), mk("Add", "a", ["t", "b"], ["y"])],
         "tensors": {"g": f32([1, 2, 3]), "b": f32([1, 2])}, "outputs": [{"name": "y"}]}
    assert G.fuse_mul_add_pattern(g)["fused"] == 0
    assert G.fuse_mul_add_pattern(g, {"x": [2], "g": [5], "b": [2]})["fused"] == 1
    assert g["nodes"][0]["inputs"] == ["g", "x", "b"]  # shape of x matches beta -> x is gamma by the rule


def test_f16_bytes_to_f32_matches_oracle(G, oracle):
    h = np.arange(65536, dtype=np.uint16)
    got = G.f16_bytes_to_f32(h.astype("<u2").tobytes()).view(np.uint32)
    np.testing.assert_array_equal(got, oracle.f16_to_f32(h).view(np.uint32))
