"""Minimal ONNX protobuf reader: the host-side mirror of onnx-parser.js.

parse_onnx_graph(bytes) returns the structure the executor and the weight loaders consume,
``{"tensors": {name: {"name", "dims", "dtype", "data"}}, "nodes": [...], "inputs": [...], "outputs": [...],
"opHist": {op_type: count}, "bytes": total initializer bytes}``, with the reference's walk:

  * a structured walk of ModelProto field 7 (graph) -> GraphProto fields 1 (node), 5 (initializer),
    11 / 12 (input / output value infos) (onnx-parser.js:358-392, :417-463);
  * when nothing was found, a byte scan for the graph tag 0x3a, keeping the best candidate and stopping at
    the first one with more than 50 tensors or nodes (:464-509);
  * unless the walk looks healthy (more than 500 tensors and nodes), a byte scan of the graph body for
    initializer tags 0x2a accepting only well-formed tensors (printable name, known dtype, data length =
    product(dims) x element size) (:300-356, :510-528).

Tensor data stays raw little-endian bytes (``bytes``); ``f16_bytes_to_f32`` (graph.py) widens fp16.
"""
from __future__ import annotations

import struct

DTYPE = {1: "float32", 2: "uint8", 3: "int8", 4: "uint16", 5: "int16", 6: "int32", 7: "int64", 9: "bool",
         10: "float16", 11: "float64"}
ELEM_SIZE = {1: 4, 6: 4, 7: 8, 9: 1, 10: 2, 11: 8}  # dtypes the initializer scan accepts


class ProtoError(ValueError):
    pass


class PBReader:
    """Protobuf wire-format cursor over bytes[p:end] (onnx-parser.js:41-102)."""

    def __init__(self, b: bytes, p: int = 0, end: int | None = None):
        self.b, self.p = b, p
        self.end = len(b) if end is None else end

    def eof(self) -> bool:
        return self.p >= self.end

    def varint(self) -> int:
        result, shift = 0, 0
        while True:
            if self.p >= len(self.b):
                raise ProtoError("varint past end of buffer")
            byte = self.b[self.p]
            self.p += 1
            result |= (byte & 0x7F) << shift
            if not byte & 0x80:
                return result
            shift += 7

    def tag(self):
        v = self.varint()
        return v >> 3, v & 7

    def len_delimited(self):
        n = self.varint()
        start = self.p
        self.p += n
        return start, start + n

    def skip(self, wire: int) -> None:
        if wire == 0:
            self.varint()
        elif wire == 1:
            self.p += 8
        elif wire == 2:
            n = self.varint()
            self.p += n
        elif wire == 5:
            self.p += 4
        elif wire in (3, 4):  # deprecated group markers: no payload
            pass
        else:
            raise ProtoError(f"unknown wire type {wire} at byte {self.p - 1} (end={self.end})")

    def seek_tag(self, tag_byte: int) -> bool:
        while self.p < self.end:
            hit = self.b[self.p] == tag_byte
            self.p += 1
            if hit:
                return True
        return False


def _signed64(v: int) -> int:
    return v - (1 << 64) if v >= 1 << 63 else v


def _text(b: bytes, s: int, e: int) -> str:
    return bytes(b[s:e]).decode("utf-8", errors="replace")


def parse_tensor(b: bytes, start: int, end: int) -> dict:
    """TensorProto: dims (1, packed or not), data_type (2), float_data (4), name (8), raw_data (9)."""
    r = PBReader(b, start, end)
    dims, data_type, name, float_data, raw = [], 0, "", None, None
    while not r.eof():
        field, wire = r.tag()
        if field == 1:
            if wire == 0:
                dims.append(r.varint())
            elif wire == 2:  # packed
                s2, e2 = r.len_delimited()
                r.p = s2
                while r.p < e2:
                    dims.append(r.varint())
            else:
                r.skip(wire)
        elif field == 2 and wire == 0:
            data_type = r.varint()
        elif field == 4 and wire == 2:
            s2, e2 = r.len_delimited()
            float_data = bytes(b[s2:e2 - (e2 - s2) % 4])
        elif field == 4 and wire == 5:
            float_data = (float_data or b"") + bytes(b[r.p:r.p + 4])
            r.p += 4
        elif field == 8 and wire == 2:
            s2, e2 = r.len_delimited()
            name = _text(b, s2, e2)
        elif field == 9 and wire == 2:
            s2, e2 = r.len_delimited()
            raw = bytes(b[s2:e2])
        else:
            r.skip(wire)
    data = raw if raw is not None else float_data
    return {"name": name, "dims": dims, "dtype": DTYPE.get(data_type, f"unknown({data_type})"), "data": data}


def parse_attribute(b: bytes, start: int, end: int) -> dict:
    """AttributeProto: name 1, f 2, i 3 (signed), s 4, t 5, floats 7, ints 8, strings 9, type 20."""
    r = PBReader(b, start, end)
    a = {"name": "", "type": 0, "f": None, "i": None, "s": None, "t": None, "floats": None, "ints": None,
         "strings": None}
    while not r.eof():
        try:
            field, wire = r.tag()
            if field == 1 and wire == 2:
                s2, e2 = r.len_delimited()
                a["name"] = _text(b, s2, e2)
            elif field == 20 and wire == 0:
                a["type"] = r.varint()
            elif field == 2 and wire == 5:
                a["f"] = struct.unpack_from("<f", b, r.p)[0]
                r.p += 4
            elif field == 3 and wire == 0:
                a["i"] = _signed64(r.varint())
            elif field == 4 and wire == 2:
                s2, e2 = r.len_delimited()
                a["s"] = bytes(b[s2:e2])
            elif field == 5 and wire == 2:
                s2, e2 = r.len_delimited()
                try:
                    a["t"] = parse_tensor(b, s2, e2)
                except Exception:
                    a["t"] = None
            elif field == 7 and wire == 2:
                s2, e2 = r.len_delimited()
                n = (e2 - s2) // 4
                a["floats"] = list(struct.unpack_from(f"<{n}f", b, s2))
            elif field == 8:
                if a["ints"] is None:
                    a["ints"] = []
                if wire == 0:
                    a["ints"].append(_signed64(r.varint()))
                elif wire == 2:  # packed
                    s2, e2 = r.len_delimited()
                    r.p = s2
                    while r.p < e2:
                        a["ints"].append(_signed64(r.varint()))
                else:
                    r.skip(wire)
            elif field == 9 and wire == 2:
                s2, e2 = r.len_delimited()
                a["strings"] = (a["strings"] or []) + [_text(b, s2, e2)]
            else:
                r.skip(wire)
        except Exception:
            break
    return a


def parse_node(b: bytes, start: int, end: int) -> dict:
    """NodeProto: input 1, output 2, name 3, op_type 4, attribute 5, domain 7."""
    r = PBReader(b, start, end)
    n = {"name": "", "op_type": "", "domain": "", "inputs": [], "outputs": [], "attributes": []}
    while not r.eof():
        try:
            field, wire = r.tag()
            if wire == 2 and field in (1, 2, 3, 4, 7):
                s2, e2 = r.len_delimited()
                t = _text(b, s2, e2)
                if field == 1:
                    n["inputs"].append(t)
                elif field == 2:
                    n["outputs"].append(t)
                elif field == 3:
                    n["name"] = t
                elif field == 4:
                    n["op_type"] = t
                else:
                    n["domain"] = t
            elif field == 5 and wire == 2:
                s2, e2 = r.len_delimited()
                n["attributes"].append(parse_attribute(b, s2, e2))
            else:
                r.skip(wire)
        except Exception:
            break
    return n


def parse_value_info(b: bytes, start: int, end: int) -> dict:
    """ValueInfoProto: name 1, type 2 -> tensor_type 1 -> elem_type 1, shape 2 -> dim 1 -> dim_value 1
    (signed; -1 where a dim has no value)."""
    r = PBReader(b, start, end)
    vi = {"name": "", "dtype": 0, "dims": []}
    while not r.eof():
        try:
            field, wire = r.tag()
            if field == 1 and wire == 2:
                s2, e2 = r.len_delimited()
                vi["name"] = _text(b, s2, e2)
            elif field == 2 and wire == 2:
                ts, te = r.len_delimited()
                tr = PBReader(b, ts, te)
                while not tr.eof():
                    f2, w2 = tr.tag()
                    if f2 == 1 and w2 == 2:
                        tts, tte = tr.len_delimited()
                        ttr = PBReader(b, tts, tte)
                        while not ttr.eof():
                            f3, w3 = ttr.tag()
                            if f3 == 1 and w3 == 0:
                                vi["dtype"] = ttr.varint()
                            elif f3 == 2 and w3 == 2:
                                shs, she = ttr.len_delimited()
                                shr = PBReader(b, shs, she)
                                while not shr.eof():
                                    f4, w4 = shr.tag()
                                    if f4 == 1 and w4 == 2:
                                        ds, de = shr.len_delimited()
                                        dr = PBReader(b, ds, de)
                                        dim = -1
                                        while not dr.eof():
                                            f5, w5 = dr.tag()
                                            if f5 == 1 and w5 == 0:
                                                dim = _signed64(dr.varint())
                                            else:
                                                dr.skip(w5)
                                        vi["dims"].append(dim)
                                    else:
                                        shr.skip(w4)
                            else:
                                ttr.skip(w3)
                    else:
                        tr.skip(w2)
            else:
                r.skip(wire)
        except Exception:
            break
    return vi


def _printable(s: str) -> bool:
    return 0 < len(s) <= 512 and all(0x20 <= ord(ch) <= 0x7E for ch in s)


def scan_initializers(b: bytes, start: int, end: int, on_tensor) -> None:
    """Byte scan for 0x2a-tagged TensorProtos that validate (onnx-parser.js:320-356)."""
    codes = {v: k for k, v in DTYPE.items()}
    p = start
    while p < end:
        if b[p] != 0x2A:
            p += 1
            continue
        r = PBReader(b, p + 1, end)
        try:
            n = r.varint()
        except Exception:
            p += 1
            continue
        if n < 8 or n > 512 * 1024 * 1024 or r.p + n > end:
            p += 1
            continue
        s2, e2 = r.p, r.p + n
        try:
            t = parse_tensor(b, s2, e2)
            code = codes.get(t["dtype"])
            elem = ELEM_SIZE.get(code) if code is not None else None
            expected = elem
            if elem is not None:
                for d in t["dims"]:
                    expected *= d
            if elem and _printable(t["name"]) and t["data"] is not None and len(t["data"]) == expected:
                on_tensor(t)
                p = e2
                continue
        except Exception:
            pass
        p += 1


def parse_graph(b: bytes, start: int, end: int, cb: dict, on_warn=lambda w: None) -> None:
    """GraphProto walk: node 1, initializer 5, input 11, output 12; stops at the first desync."""
    r = PBReader(b, start, end)
    while not r.eof():
        try:
            field, wire = r.tag()
            if wire == 2 and field in (1, 5, 11, 12):
                s2, e2 = r.len_delimited()
                fn = {1: ("onNode", parse_node), 5: ("onTensor", parse_tensor), 11: ("onInput", parse_value_info),
                      12: ("onOutput", parse_value_info)}[field]
                try:
                    cb.get(fn[0], lambda x: None)(fn[1](b, s2, e2))
                except Exception as e:
                    on_warn(f"{fn[0]} parse failed at byte {s2}: {e}")
            else:
                r.skip(wire)
        except Exception as e:
            on_warn(f"graph-tag read halted at byte {r.p}: {e}")
            break


def parse_onnx_graph(b: bytes, on_progress=lambda s: None) -> dict:
    """onnx-parser.js:417-540."""
    b = bytes(b)
    tensors, nodes, inputs, outputs = {}, [], [], []
    total = [0]

    def on_tensor(t):
        tensors[t["name"]] = t
        total[0] += len(t["data"] or b"")

    cb = {"onTensor": on_tensor, "onNode": nodes.append, "onInput": inputs.append, "onOutput": outputs.append}
    parsed, g0, g1 = False, 0, len(b)
    r = PBReader(b, 0, len(b))
    while not r.eof():
        tag_start = r.p
        try:
            field, wire = r.tag()
            if field == 7 and wire == 2:
                s2, e2 = r.len_delimited()
                g0, g1 = s2, e2
                parse_graph(b, s2, e2, cb)
                parsed = True
            else:
                r.skip(wire)
        except Exception:
            p = tag_start + 1
            while p < len(b) and b[p] != 0x3A:
                p += 1
            if p >= len(b):
                break
            r.p = p
    if not tensors and not nodes:
        best = 0
        r2 = PBReader(b, 0, len(b))
        while r2.seek_tag(0x3A):
            tag_pos = r2.p - 1
            try:
                saved = r2.p
                n = r2.varint()
                if 0 < n < len(b) and r2.p + n <= len(b):
                    s2, e2 = r2.p, r2.p + n
                    tt, tn, ti, to = {}, [], [], []
                    parse_graph(b, s2, e2, {"onTensor": lambda t: tt.__setitem__(t["name"], t), "onNode": tn.append,
                                            "onInput": ti.append, "onOutput": to.append})
                    if len(tt) + len(tn) > best:
                        tensors.clear()
                        tensors.update(tt)
                        nodes[:], inputs[:], outputs[:] = tn, ti, to
                        total[0] = sum(len(t["data"] or b"") for t in tt.values())
                        best = len(tt) + len(tn)
                        g0, g1 = s2, e2
                        if len(tt) > 50 or len(tn) > 50:
                            break
                r2.p = saved + 1
            except Exception:
                r2.p = tag_pos + 1
    if not (len(tensors) > 500 and len(nodes) > 500):
        def add(t):
            if t["name"] not in tensors:
                on_tensor(t)
        scan_initializers(b, g0, g1, add)
    op_hist: dict = {}
    for n in nodes:
        op_hist[n["op_type"]] = op_hist.get(n["op_type"], 0) + 1
    return {"tensors": tensors, "nodes": nodes, "inputs": inputs, "outputs": outputs, "opHist": op_hist,
            "bytes": total[0]}


def parse_onnx_weights(b: bytes, on_progress=lambda s: None) -> dict:
    """onnx-parser.js:401-415: the initializers only."""
    g = parse_onnx_graph(b, on_progress)
    return {"tensors": g["tensors"], "count": len(g["tensors"]), "bytes": g["bytes"]}


def weight_fn(graph: dict):
    """A `weights(name, n)` callback for UNet / VAEDecoder / blocks: initializer `name` as float32 when it
    exists with n elements (fp16 data widened bit-exactly, as WeightCache does)."""
    import numpy as np
    from .graph import f16_bytes_to_f32

    def fn(name, n):
        t = graph["tensors"].get(name)
        if t is None or t["data"] is None:
            return None
        if t["dtype"] == "float16":
            a = f16_bytes_to_f32(t["data"])
        elif t["dtype"] == "float32":
            a = np.frombuffer(t["data"], "<f4")
        else:
            return None
        return a if a.size == n else None
    return fn


# reference spellings
parseONNXGraph = parse_onnx_graph
parseONNXWeights = parse_onnx_weights
parseTensor = parse_tensor
