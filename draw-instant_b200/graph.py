"""ONNX-graph rewrites of the executor (wgsl-executor.js:795-1008), host side.

A graph is the reference's plain structure: ``{"nodes": [node...], "tensors": {name: tensor},
"outputs": [{"name": ...}]}`` with ``node = {"op_type", "name", "inputs", "outputs", "attributes"}`` and
``tensor = {"dtype": "float32" | "float16" | "int64" ..., "dims": [...], "data": bytes}`` (initializers).
Each pass rewrites ``graph["nodes"]`` in place and returns ``{"fused": k}``; the node lists it produces
(order, names, inputs, outputs, attributes) are the ones the reference's passes produce, so the executor
walks the same graph.

  fuse_silu_pattern        Sigmoid(X) -> Mul(X, sig)                    => Silu(X)
  fuse_mul_add_pattern     Mul(X, gamma) -> Add(., beta), same shapes   => AffineBcast(X, gamma, beta)
  fuse_group_norm_pattern  Reshape(X, [N, G, -1]) -> InstanceNormalization(., ones, zeros) -> Reshape
                           -> AffineBcast(., gamma, beta)               => GroupNorm(X, gamma, beta)
                           (run after fuse_mul_add_pattern; G from the Reshape shape Constant, else 32)

The fused GroupNorm / Silu / AffineBcast nodes are what libdi's di_group_norm (fuse_silu), di_unary
(SiLU) and di_affine_bcast entry points execute.
"""
from __future__ import annotations

import struct

import numpy as np

__all__ = ["fuse_silu_pattern", "fuse_mul_add_pattern", "fuse_group_norm_pattern", "f16_bytes_to_f32",
           "fuseSiluPattern", "fuseMulAddPattern", "fuseGroupNormPattern"]


def _consumers(graph) -> dict:
    cnt: dict = {}
    for n in graph["nodes"]:
        for i in n["inputs"]:
            if i:
                cnt[i] = cnt.get(i, 0) + 1
    for o in graph.get("outputs") or []:
        cnt[o["name"]] = cnt.get(o["name"], 0) + 1
    return cnt


def _producers(nodes) -> dict:
    prod = {}
    for idx, n in enumerate(nodes):
        for o in n["outputs"]:
            prod[o] = idx
    return prod


def _drop(graph, nodes, drop) -> None:
    graph["nodes"] = [n for i, n in enumerate(nodes) if i not in drop]


def fuse_silu_pattern(graph) -> dict:
    """wgsl-executor.js:795-836: a Mul whose one input is a Sigmoid of its other input, the Sigmoid having
    no other consumer, becomes Silu(x) named '<mul>_fused'; the Sigmoid is dropped."""
    nodes = graph["nodes"]
    consumers, producer = _consumers(graph), _producers(nodes)
    drop, fused = set(), 0
    for i, mul in enumerate(nodes):
        if mul["op_type"] != "Mul":
            continue
        a, b = (list(mul["inputs"]) + [None, None])[:2]

        def try_fuse(sig_out, other_in):
            if not sig_out or not other_in or consumers.get(sig_out, 0) != 1:
                return False
            pi = producer.get(sig_out)
            if pi is None:
                return False
            sig = nodes[pi]
            if sig["op_type"] != "Sigmoid" or sig["inputs"][0] != other_in:
                return False
            nodes[i] = {"op_type": "Silu", "name": (mul.get("name") or "") + "_fused", "inputs": [other_in],
                        "outputs": list(mul["outputs"]), "attributes": []}
            drop.add(pi)
            return True

        if try_fuse(a, b) or try_fuse(b, a):
            fused += 1
    if fused:
        _drop(graph, nodes, drop)
    return {"fused": fused}


def fuse_mul_add_pattern(graph, tensor_shapes: dict | None = None) -> dict:
    """wgsl-executor.js:838-893: Add(Mul(x, gamma), beta) with gamma and beta of identical shape and the
    Mul consumed once becomes AffineBcast(x, gamma, beta) named '<mul>_affinefused'."""
    nodes = graph["nodes"]
    consumers, producer = _consumers(graph), _producers(nodes)
    tensors = graph.get("tensors") or {}

    def shape_of(name):
        if tensor_shapes and name in tensor_shapes:
            return list(tensor_shapes[name])
        t = tensors.get(name)
        return list(t["dims"]) if t is not None and "dims" in t else None

    drop, fused = set(), 0
    for i, add in enumerate(nodes):
        if add["op_type"] != "Add":
            continue
        add_a, add_b = (list(add["inputs"]) + [None, None])[:2]

        def try_fuse(mul_out, beta):
            if consumers.get(mul_out, 0) != 1:
                return False
            pi = producer.get(mul_out)
            if pi is None or nodes[pi]["op_type"] != "Mul":
                return False
            mul = nodes[pi]
            mul_a, mul_b = mul["inputs"][:2]
            s_a, s_b, s_beta = shape_of(mul_a), shape_of(mul_b), shape_of(beta)
            if not s_beta:
                return False
            if s_a is not None and s_a == s_beta:
                x, gamma = mul_b, mul_a
            elif s_b is not None and s_b == s_beta:
                x, gamma = mul_a, mul_b
            else:
                return False
            nodes[i] = {"op_type": "AffineBcast", "name": (mul.get("name") or "") + "_affinefused",
                        "inputs": [x, gamma, beta], "outputs": list(add["outputs"]), "attributes": []}
            drop.add(pi)
            return True

        if try_fuse(add_a, add_b) or try_fuse(add_b, add_a):
            fused += 1
    if fused:
        _drop(graph, nodes, drop)
    return {"fused": fused}


def f16_bytes_to_f32(raw: bytes) -> np.ndarray:
    """wgsl-unet.js:23-47 on the host (integer bit manipulation; subnormals, Inf and NaN payloads exact)."""
    h = np.frombuffer(raw, dtype="<u2").astype(np.uint32)
    sign = (h & 0x8000) << 16
    exp = (h >> 10) & 0x1F
    mant = h & 0x3FF
    bits = sign | ((exp + 112) << 23) | (mant << 13)
    bits = np.where(exp == 31, sign | 0x7F800000 | (mant << 13), bits)
    sub = (exp == 0) & (mant != 0)
    if np.any(sub):
        m = mant[sub].astype(np.int64)
        lz = np.zeros_like(m)
        for _ in range(10):  # shift until bit 10 is set (at most 10 shifts for a nonzero 10-bit mantissa)
            need = (m & 0x400) == 0
            m = np.where(need, m << 1, m)
            lz += need
        e = 1 - lz
        bits[sub] = sign[sub] | ((e + 112) << 23).astype(np.uint32) | ((m & 0x3FF) << 13).astype(np.uint32)
    bits = np.where((exp == 0) & (mant == 0), sign, bits)
    return bits.astype(np.uint32).view(np.float32)


def _uniform_of(t):
    """A tensor's single value if all its elements are equal (float32 / float16), else None."""
    if not t or not t.get("data"):
        return None
    if t["dtype"] == "float32":
        f = np.frombuffer(t["data"], dtype="<f4")
    elif t["dtype"] == "float16":
        f = f16_bytes_to_f32(t["data"])
    else:
        return None
    if f.size == 0:
        return None
    return float(f[0]) if np.all(f == f[0]) else None


def fuse_group_norm_pattern(graph) -> dict:
    """wgsl-executor.js:895-1006: Reshape -> InstanceNormalization(scale all ones, bias all zeros) ->
    Reshape -> AffineBcast, each intermediate consumed once, becomes GroupNorm(x, gamma, beta) named
    '<aff>_gn' with attributes num_groups (from a Constant int64 [N, G, -1] shape, else 32) and epsilon.
    Constants resolve from initializers as well as Constant nodes (the U-Net has only initializers)."""
    nodes = graph["nodes"]
    consumers, producer = _consumers(graph), _producers(nodes)
    tensors = graph.get("tensors") or {}

    def const_val(name):
        if name in tensors and tensors[name].get("data"):
            return _uniform_of(tensors[name])
        pi = producer.get(name)
        if pi is None or nodes[pi]["op_type"] != "Constant":
            return None
        a = next((x for x in nodes[pi]["attributes"] if x.get("name") == "value"), None)
        return _uniform_of(a.get("t")) if a else None

    drop, fused = set(), 0
    for i, aff in enumerate(nodes):
        if aff["op_type"] != "AffineBcast":
            continue
        aff_x, gamma, beta = aff["inputs"][:3]
        if consumers.get(aff_x, 0) != 1:
            continue
        rs1i = producer.get(aff_x)
        if rs1i is None or nodes[rs1i]["op_type"] != "Reshape":
            continue
        in_out = nodes[rs1i]["inputs"][0]
        if consumers.get(in_out, 0) != 1:
            continue
        ini = producer.get(in_out)
        if ini is None or nodes[ini]["op_type"] != "InstanceNormalization":
            continue
        in_node = nodes[ini]
        resh_out, scale, bias = in_node["inputs"][:3]
        if const_val(scale) != 1 or const_val(bias) != 0:
            continue
        if consumers.get(resh_out, 0) != 1:
            continue
        rs0i = producer.get(resh_out)
        if rs0i is None or nodes[rs0i]["op_type"] != "Reshape":
            continue
        x, shape0 = nodes[rs0i]["inputs"][:2]
        G = 32
        spi = producer.get(shape0)
        if spi is not None and nodes[spi]["op_type"] == "Constant":
            a = next((y for y in nodes[spi]["attributes"] if y.get("name") == "value"), None)
            t = a.get("t") if a else None
            if t and t.get("dtype") == "int64" and t.get("data") and len(t["data"]) >= 16:
                G = struct.unpack_from("<q", t["data"], 8)[0]
        eps_a = next((y for y in in_node["attributes"] if y.get("name") == "epsilon"), None)
        eps = float(eps_a["f"]) if eps_a else 1e-5
        nodes[i] = {"op_type": "GroupNorm", "name": (aff.get("name") or "") + "_gn", "inputs": [x, gamma, beta],
                    "outputs": list(aff["outputs"]),
                    "attributes": [{"name": "num_groups", "i": G}, {"name": "epsilon", "f": eps}]}
        drop.update((rs1i, ini, rs0i))
        fused += 1
    if fused:
        _drop(graph, nodes, drop)
    return {"fused": fused}


# reference spellings
fuseSiluPattern = fuse_silu_pattern
fuseMulAddPattern = fuse_mul_add_pattern
fuseGroupNormPattern = fuse_group_norm_pattern
