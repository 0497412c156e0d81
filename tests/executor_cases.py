"""Test infrastructure for the ONNX-graph executor: a host "device" whose op families are the CPU oracle's
restatements of wgsl-ops.js (same cfg blocks as the libdi closures), a small SD-style graph that exercises
the op set and the host shape path, its protobuf encoding, and an independent NumPy evaluation."""
from __future__ import annotations

import struct

import numpy as np


class HostBuf:
    """A flat fp32 host buffer standing in for a device buffer."""

    def __init__(self, nbytes: int):
        self.a = np.zeros((nbytes + 3) // 4, np.float32)


class OracleBackend:
    def __init__(self, oracle, unary_codes, binary_codes):
        self.o = oracle
        d = {"unary": {}, "binary": {}, "binaryBcast": {}}
        o = oracle

        def put(Y, v):
            v = np.asarray(v, np.float32).ravel()
            Y.a[: v.size] = v

        for name, code in unary_codes.items():
            d["unary"][name] = lambda enc, X, Y, N, c=code: put(Y, o.unary(c, X.a[:N]))
        for name, code in binary_codes.items():
            d["binary"][name] = lambda enc, A, B, Y, N, c=code: put(Y, o.binary(c, A.a[:N], B.a[:N], N))
            d["binaryBcast"][name] = lambda enc, A, B, Y, cfg, n, c=code: put(Y, o.binary_bcast(c, A.a, B.a, cfg))
        d["affineBcast"] = lambda enc, A, G, Bt, Y, cfg, n: put(Y, o.affine_bcast(A.a, G.a, Bt.a, cfg))
        d["softmax"] = lambda enc, X, Y, cfg, rows: put(Y, o.softmax(X.a[: cfg[0] * rows], int(cfg[0]), rows))
        d["instanceNorm"] = lambda enc, X, g, b, Y, cfg, C, N: put(
            Y, o.instance_norm(X.a[: int(cfg[0] * cfg[1] * cfg[2])], g.a[:C], b.a[:C], int(cfg[0]), int(cfg[1]),
                               int(cfg[2])))

        def gn(enc, X, g, b, Y, cfg, G, N):
            n_, g_, cpg, hw = (int(v) for v in cfg[:4])
            eps = float(np.asarray(cfg[4:5], np.uint32).view(np.float32)[0])
            C = g_ * cpg
            put(Y, o.group_norm(X.a[: n_ * C * hw], g.a[:C], b.a[:C], n_, C, hw, g_, eps))
        d["groupNorm"] = gn
        d["matmul"] = lambda enc, A, B, Y, cfg, M, N, batch=1: put(
            Y, o.matmul(A.a, B.a, int(cfg[0]), int(cfg[1]), int(cfg[2]), int(cfg[3]), batch))
        d["gemm"] = lambda enc, A, B, C, Y, cfg, M, N: put(
            Y, o.gemm(A.a, B.a, C.a, int(cfg[0]), int(cfg[1]), int(cfg[2]), int(cfg[3])))

        def conv(enc, X, W, bias, Y, cfg, Co, HW):
            ci, co, k, _, h, w, pad, s = (int(v) for v in cfg[:8])
            put(Y, o.conv(X.a[: ci * h * w], W.a[: co * ci * k * k], bias.a[:co], 1, ci, h, w, co, k, s, pad))
        d["convMM"] = conv
        d["resizeNearest"] = lambda enc, X, Y, cfg, n: put(Y, o.resize_nearest(X.a, cfg))
        d["reduceMean"] = lambda enc, X, Y, cfg, rows: put(Y, o.reduce_mean(X.a, int(cfg[0]), rows))
        d["transpose"] = lambda enc, X, Y, cfg, n: put(Y, o.transpose(X.a, cfg))
        d["powScalar"] = lambda enc, X, Y, cfg, N: put(Y, o.pow_scalar(X.a[:N], float(cfg.view(np.float32)[0])))
        d["slice"] = lambda enc, X, Y, cfg, n: put(Y, o.slice_(X.a, cfg))

        def concat(enc, X, Y, cfg, n):
            Y.a[:] = o.concat_copy(X.a, Y.a, cfg)[: Y.a.size]
        d["concatCopy"] = concat
        self.dispatchers = d

    def alloc(self, nbytes):
        return HostBuf(nbytes)

    @staticmethod
    def nbytes(buf):
        return buf.a.size * 4

    def write(self, buf, arr):
        a = np.asarray(arr, np.float32).ravel()
        buf.a[: a.size] = a

    def copy(self, src, dst, nbytes):
        dst.a[: nbytes // 4] = src.a[: nbytes // 4]

    def read(self, buf, nbytes):
        return buf.a[: nbytes // 4].copy()

    def encoder(self):
        return None

    def uniform(self, arr):
        return np.ascontiguousarray(arr).view(np.uint32) if np.asarray(arr).dtype == np.float32 else \
            np.ascontiguousarray(arr, np.uint32)

    def sync(self):
        pass


# ---- the test graph --------------------------------------------------------------------------------
def _n(op, ins, outs, name="", **attrs):
    al = []
    for k, v in attrs.items():
        a = {"name": k, "type": 0, "f": None, "i": None, "s": None, "t": None, "floats": None, "ints": None,
             "strings": None}
        if isinstance(v, float):
            a["f"] = v
        elif isinstance(v, int):
            a["i"] = v
        elif isinstance(v, str):
            a["s"] = v.encode()
        elif isinstance(v, list):
            a["ints"] = list(v)
        elif isinstance(v, dict):
            a["t"] = v
        al.append(a)
    return {"name": name or outs[0], "op_type": op, "domain": "", "inputs": list(ins), "outputs": list(outs),
            "attributes": al}


def _t(name, arr, dtype="float32"):
    a = np.asarray(arr)
    raw = a.astype({"float32": "<f4", "float16": "<f2", "int64": "<i8"}[dtype]).tobytes()
    return {"name": name, "dims": list(a.shape), "dtype": dtype, "data": raw}


def sd_graph(seed=0):
    """An SD-style subgraph (NCHW fp32, batch 1): conv -> GroupNorm pattern (Reshape / InstanceNorm /
    Reshape / Mul / Add) -> Sigmoid * x -> strided conv -> single-head attention over the 16 pixels with the
    1/sqrt(d) scale from the shape path -> LayerNorm pattern -> nearest x2 -> channel concat -> Slice ->
    1x1 conv; and a Gemm head on the flattened result.  Returns (graph, tensors, x)."""
    rng = np.random.default_rng(seed)
    w = lambda *s, k=1.0: (rng.standard_normal(s) * k).astype(np.float32)
    T = {}
    for t in [_t("W1", w(64, 4, 3, 3, k=0.3)), _t("b1", w(64, k=0.1)),
              _t("gn_scale", np.ones(32, np.float32)), _t("gn_bias", np.zeros(32, np.float32)),
              _t("shape3", np.array([0, 32, -1]), "int64"),
              _t("gamma", (1 + w(64, 1, 1, k=0.1)).astype(np.float16), "float16"), _t("beta", w(64, 1, 1, k=0.1)),
              _t("W2", w(64, 64, 3, 3, k=0.05)), _t("b2", w(64, k=0.1)),
              _t("Wq", w(64, 64, k=0.12)), _t("idx2", np.array(2), "int64"),
              _t("two", np.array([2.0], np.float32)), _t("eps", np.array([1e-5], np.float32)),
              _t("ln_g", w(64, k=0.1) + 1), _t("ln_b", w(64, k=0.1)),
              _t("scales", np.array([1, 1, 2, 2], np.float32)),
              _t("st", np.array([0]), "int64"), _t("en", np.array([96]), "int64"), _t("ax", np.array([1]), "int64"),
              _t("W3", w(8, 96, 1, 1, k=0.1)), _t("b3", w(8, k=0.1)),
              _t("Wg", w(10, 512, k=0.05)), _t("bg", w(10, k=0.1))]:
        T[t["name"]] = t
    N = []
    N.append(_n("Conv", ["x", "W1", "b1"], ["h"], kernel_shape=[3, 3], pads=[1, 1, 1, 1]))
    N.append(_n("Reshape", ["h", "shape3"], ["h3"]))
    N.append(_n("InstanceNormalization", ["h3", "gn_scale", "gn_bias"], ["hn3"], epsilon=1e-5))
    N.append(_n("Shape", ["h"], ["hshape"]))
    N.append(_n("Reshape", ["hn3", "hshape"], ["hn"]))
    N.append(_n("Mul", ["hn", "gamma"], ["hm"]))
    N.append(_n("Add", ["hm", "beta"], ["ha"]))
    N.append(_n("Sigmoid", ["ha"], ["hsig"]))
    N.append(_n("Mul", ["ha", "hsig"], ["hs"]))
    N.append(_n("Conv", ["hs", "W2", "b2"], ["t"], kernel_shape=[3, 3], pads=[1, 1, 1, 1], strides=[2, 2]))
    N.append(_n("Constant", [], ["c_tok"], value_ints=[1, 64, -1]))
    N.append(_n("Reshape", ["t", "c_tok"], ["t3"]))
    N.append(_n("Transpose", ["t3"], ["q"], perm=[0, 2, 1]))                   # [1, 16, 64]
    N.append(_n("MatMul", ["q", "Wq"], ["qp"]))
    N.append(_n("Transpose", ["q"], ["kT"], perm=[0, 2, 1]))                   # [1, 64, 16]
    N.append(_n("MatMul", ["qp", "kT"], ["s"]))                                # [1, 16, 16]
    N.append(_n("Shape", ["q"], ["qshape"]))
    N.append(_n("Gather", ["qshape", "idx2"], ["dq"], axis=0))                  # 64 (host)
    N.append(_n("Cast", ["dq"], ["dqf"], to=1))
    N.append(_n("Sqrt", ["dqf"], ["sq"]))                                      # host scalar 8
    N.append(_n("Div", ["s", "sq"], ["ss"]))
    N.append(_n("Softmax", ["ss"], ["p"], axis=-1))
    N.append(_n("MatMul", ["p", "q"], ["o"]))                                  # [1, 16, 64]
    N.append(_n("Add", ["o", "q"], ["r"]))
    N.append(_n("ReduceMean", ["r"], ["mu"], axes=[-1], keepdims=1))
    N.append(_n("Sub", ["r", "mu"], ["xc"]))
    N.append(_n("Pow", ["xc", "two"], ["xc2"]))
    N.append(_n("ReduceMean", ["xc2"], ["var"], axes=[-1], keepdims=1))
    N.append(_n("Add", ["var", "eps"], ["ve"]))
    N.append(_n("Sqrt", ["ve"], ["sd"]))
    N.append(_n("Div", ["xc", "sd"], ["ln0"]))
    N.append(_n("Mul", ["ln0", "ln_g"], ["ln1"]))
    N.append(_n("Add", ["ln1", "ln_b"], ["ln"]))
    N.append(_n("Transpose", ["ln"], ["lnT"], perm=[0, 2, 1]))                 # [1, 64, 16]
    N.append(_n("Shape", ["t"], ["tshape"]))
    N.append(_n("Reshape", ["lnT", "tshape"], ["u"]))                          # [1, 64, 4, 4]
    N.append(_n("Resize", ["u", "", "scales"], ["up"], mode="nearest"))         # [1, 64, 8, 8]
    N.append(_n("Concat", ["up", "h"], ["cat"], axis=1))                       # [1, 128, 8, 8]
    N.append(_n("Slice", ["cat", "st", "en", "ax"], ["sl"]))                   # [1, 96, 8, 8]
    N.append(_n("Conv", ["sl", "W3", "b3"], ["y"], kernel_shape=[1, 1], pads=[0, 0, 0, 0]))
    N.append(_n("Constant", [], ["c_flat"], value_ints=[1, -1]))
    N.append(_n("Reshape", ["y", "c_flat"], ["yf"]))                           # [1, 512]
    N.append(_n("Gemm", ["yf", "Wg", "bg"], ["z"], transB=1))                  # [1, 10]
    graph = {"nodes": N, "inputs": [{"name": "x"}], "outputs": [{"name": "y"}, {"name": "z"}]}
    x = (rng.standard_normal((1, 4, 8, 8))).astype(np.float32)
    return graph, T, x


def sd_graph_numpy(T, x):
    """The same graph in float64 NumPy (independent of both op libraries)."""
    g = lambda n: np.frombuffer(T[n]["data"], {"float32": "<f4", "float16": "<f2", "int64": "<i8"}[T[n]["dtype"]]) \
        .astype(np.float64).reshape(T[n]["dims"])

    def conv(a, W, b, s=1, p=1):
        n_, ci, h, w_ = a.shape
        co, _, k, _ = W.shape
        ap = np.pad(a, ((0, 0), (0, 0), (p, p), (p, p)))
        ho, wo = (h + 2 * p - k) // s + 1, (w_ + 2 * p - k) // s + 1
        out = np.zeros((n_, co, ho, wo))
        for ky in range(k):
            for kx in range(k):
                patch = ap[:, :, ky:ky + s * ho:s, kx:kx + s * wo:s]
                out += np.einsum("nchw,oc->nohw", patch, W[:, :, ky, kx])
        return out + b[None, :, None, None]

    x = x.astype(np.float64)
    h = conv(x, g("W1"), g("b1"))
    h3 = h.reshape(1, 32, -1)
    m = h3.mean(-1, keepdims=True)
    v = np.maximum((h3 * h3).mean(-1, keepdims=True) - m * m, 0)
    hn = ((h3 - m) / np.sqrt(v + 1e-5)).reshape(h.shape)
    ha = hn * g("gamma") + g("beta")
    hs = ha / (1 + np.exp(-ha))
    t = conv(hs, g("W2"), g("b2"), s=2)
    q = t.reshape(1, 64, -1).transpose(0, 2, 1)
    s = (q @ g("Wq")) @ q.transpose(0, 2, 1) / 8.0
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    r = p @ q + q
    mu = r.mean(-1, keepdims=True)
    xc = r - mu
    ln = xc / np.sqrt((xc ** 2).mean(-1, keepdims=True) + 1e-5) * g("ln_g") + g("ln_b")
    u = ln.transpose(0, 2, 1).reshape(t.shape)
    up = u.repeat(2, 2).repeat(2, 3)
    cat = np.concatenate([up, h], 1)[:, :96]
    y = conv(cat, g("W3"), g("b3"), p=0)
    z = y.reshape(1, -1) @ g("Wg").T + g("bg")
    return {"y": y.astype(np.float32), "z": z.astype(np.float32)}


# ---- protobuf encoding (ModelProto with one GraphProto) -----------------------------------------------
def _varint(n):
    out = bytearray()
    n &= (1 << 64) - 1
    while n > 0x7F:
        out.append((n & 0x7F) | 0x80)
        n >>= 7
    out.append(n)
    return bytes(out)


def _ld(field, payload):
    return _varint((field << 3) | 2) + _varint(len(payload)) + payload


def _vi(field, n):
    return _varint(field << 3) + _varint(n)


def _s(field, text):
    return _ld(field, text.encode())


DT_CODE = {"float32": 1, "int64": 7, "float16": 10}


def _tensor_pb(t):
    return b"".join(_vi(1, d) for d in t["dims"]) + _vi(2, DT_CODE[t["dtype"]]) + _s(8, t["name"]) + \
        _ld(9, t["data"])


def _attr_pb(a):
    out = _s(1, a["name"])
    if a["f"] is not None:
        out += _varint((2 << 3) | 5) + struct.pack("<f", a["f"])
    if a["i"] is not None:
        out += _vi(3, a["i"])
    if a["s"] is not None:
        out += _ld(4, a["s"])
    if a["t"] is not None:
        out += _ld(5, _tensor_pb(a["t"]))
    if a["ints"] is not None:
        out += b"".join(_vi(8, v) for v in a["ints"])
    return out


def encode_model(graph, tensors) -> bytes:
    g = b""
    for n in graph["nodes"]:
        body = b"".join(_s(1, i) for i in n["inputs"]) + b"".join(_s(2, o) for o in n["outputs"]) + \
            _s(3, n["name"]) + _s(4, n["op_type"]) + b"".join(_ld(5, _attr_pb(a)) for a in n["attributes"])
        g += _ld(1, body)
    for t in tensors.values():
        g += _ld(5, _tensor_pb(t))
    for i in graph["inputs"]:
        g += _ld(11, _s(1, i["name"]))
    for o in graph["outputs"]:
        g += _ld(12, _s(1, o["name"]))
    return _vi(1, 8) + _s(2, "draw-instant-b200 executor test") + _ld(7, g) + _ld(8, _vi(2, 17))
