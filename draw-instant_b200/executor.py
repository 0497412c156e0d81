"""The ONNX-graph executor: walks a parsed graph node by node and dispatches each op to the op-family
closures, with the reference's tensor lifetimes.  It is the libdi counterpart of wgsl-executor.js
(Tensor / BufferPool :45-94, OPS :129-1114, inferGraphIO :1205-1221, Executor.run :1223-1467).

    ex = Executor(GpuBackend(ctx), graph, WeightCache(backend, graph["tensors"]))
    out = ex.run({"sample": Tensor(buf, [1, 4, 64, 64])})   # {output name: Tensor}

What it keeps from the reference, because callers and graphs depend on it:
- the same op set and attribute semantics, the CPU "shape path" (Shape -> Gather -> Concat -> Reshape
  and friends stay host arrays; GPU ops promote them on first use);
- consumer counting per tensor name, releases deferred until the walk has been submitted, graph outputs
  snapshotted into fresh buffers, alias-held intermediates swept back to the pool (and, past the
  reference, the outputs' original buffers and promoted host tensors, which it leaks every run);
- the pool's 4 KB size classes and its owned-buffer rule.

The device is a small backend object (`GpuBackend` drives libdi through `ops.py`): buffer allocation,
upload, copy, read-back, a fence, and the dispatcher table of `createDispatchers`.  Tensors hold fp32
data as the reference's do.  The plans (`unet.UNet`, `vae.VAEDecoder`) are the fast path for the
known models; this walk runs any graph the op set covers.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

from . import DIError

ONNX_CAST = {1: "float32", 6: "int32", 7: "int64"}


# ---------------------------------------------------------------------------------------------------
# Tensor and pool (wgsl-executor.js:45-94)
# ---------------------------------------------------------------------------------------------------
@dataclass
class Tensor:
    """A device buffer with dims (fp32 data), or a host-only tensor (buf None, cpu_data set)."""
    buf: object = None
    dims: list = field(default_factory=list)
    dtype: str = "float32"
    cpu_data: np.ndarray | None = None
    is_shape: bool | None = None

    @property
    def numel(self) -> int:
        return int(np.prod(self.dims)) if self.dims else 1

    @property
    def byte_length(self) -> int:
        return self.numel * 4

    @property
    def on_cpu(self) -> bool:
        return self.buf is None and self.cpu_data is not None


class BufferPool:
    """Free lists keyed by size rounded up to 4 KB; only buffers it allocated are recycled."""

    def __init__(self, backend):
        self.backend = backend
        self.free: dict[int, list] = {}
        self.owned: set[int] = set()
        self.live = 0
        self.peak = 0
        self.allocs = 0

    @staticmethod
    def key(nbytes: int) -> int:
        return max(1, math.ceil(nbytes / 4096)) * 4096

    def acquire(self, nbytes: int):
        k = self.key(nbytes)
        self.live += 1
        self.peak = max(self.peak, self.live)
        lst = self.free.get(k)
        if lst:
            return lst.pop()
        self.allocs += 1
        buf = self.backend.alloc(k)
        self.owned.add(id(buf))
        return buf

    def release(self, buf) -> None:
        if id(buf) not in self.owned:
            return
        self.free.setdefault(self.backend.nbytes(buf), []).append(buf)
        self.live -= 1

    def owns(self, buf) -> bool:
        return id(buf) in self.owned


class WeightCache:
    """Initializers by name, uploaded on first use (wgsl-unet.js:48-104): int64 / int32 / bool stay host
    shape tensors; fp16 is widened bit-exactly to fp32; scalar floats also keep their host value."""

    def __init__(self, backend, tensors: dict):
        from .graph import f16_bytes_to_f32
        self.backend = backend
        self.tensors = tensors
        self.cache: dict[str, Tensor] = {}
        self._f16 = f16_bytes_to_f32

    def has(self, name: str) -> bool:
        return name in self.tensors

    def names(self, prefix: str = ""):
        return [k for k in self.tensors if k.startswith(prefix)]

    def get(self, name: str) -> Tensor:
        if name in self.cache:
            return self.cache[name]
        t = self.tensors.get(name)
        if t is None:
            raise DIError(f"weight not found: {name}")
        dims = list(t["dims"])
        dt = t["dtype"]
        raw = t["data"] or b""
        if dt in ("int64", "int32", "bool"):
            npdt = {"int64": "<i8", "int32": "<i4", "bool": "u1"}[dt]
            out = Tensor(None, dims, dt, np.frombuffer(raw, npdt).copy(), dt != "bool")
        else:
            data = self._f16(raw) if dt == "float16" else np.frombuffer(raw, "<f4").copy()
            buf = self.backend.alloc(max(4, data.nbytes))
            self.backend.write(buf, data)
            out = Tensor(buf, dims, "float32", data if data.size == 1 else None)
        self.cache[name] = out
        return out


def infer_graph_io(nodes, weight_names) -> tuple[list, list]:
    """wgsl-executor.js:1205-1221: inputs = consumed, not produced, not weights; outputs = produced,
    never consumed."""
    produced, consumed = [], []
    ps, cs = set(), set()
    for n in nodes:
        for i in n["inputs"]:
            if i not in cs:
                cs.add(i)
                consumed.append(i)
        for o in n["outputs"]:
            if o not in ps:
                ps.add(o)
                produced.append(o)
    inputs = [{"name": c} for c in consumed if c not in ps and c not in weight_names]
    outputs = [{"name": p} for p in produced if p not in cs]
    return inputs, outputs


# ---------------------------------------------------------------------------------------------------
# Op registry (wgsl-executor.js:129-1114)
# ---------------------------------------------------------------------------------------------------
def _attr(node, name):
    """The attribute dict (parser fields name / i / f / s / t / ints / floats; missing keys are None)."""
    for a in node.get("attributes") or []:
        if a.get("name") == name:
            return {k: a.get(k) for k in ("name", "i", "f", "s", "t", "ints", "floats")}
    return None


def _attr_int(node, name, default):
    a = _attr(node, name)
    return a["i"] if a is not None and a["i"] is not None else default


def _attr_ints(node, name, default):
    a = _attr(node, name)
    return list(a["ints"]) if a is not None and a["ints"] is not None else default


def _attr_str(node, name, default):
    a = _attr(node, name)
    if a is None or not a["s"]:
        return default
    return a["s"].decode() if isinstance(a["s"], (bytes, bytearray)) else a["s"]


def _row_major_strides(dims):
    s = [1] * len(dims)
    for i in range(len(dims) - 2, -1, -1):
        s[i] = s[i + 1] * dims[i + 1]
    return s


def broadcast_shape(a, b):
    n = max(len(a), len(b))
    out = [0] * n
    for i in range(n):
        x = a[len(a) - 1 - i] if i < len(a) else 1
        y = b[len(b) - 1 - i] if i < len(b) else 1
        if x == y or y == 1:
            out[n - 1 - i] = x
        elif x == 1:
            out[n - 1 - i] = y
        else:
            raise DIError(f"cannot broadcast {a} vs {b}")
    return out


def _pad4(v, fill=0):
    return list(v) + [fill] * (4 - len(v))


def _ints(t) -> list[int]:
    return [int(v) for v in np.asarray(t.cpu_data).ravel()]


def _passthrough(x: Tensor, dims) -> Tensor:
    """Reshape-like relabel: host tensors stay host tensors when their element count matches."""
    if x.on_cpu and int(np.asarray(x.cpu_data).size) == (int(np.prod(dims)) if dims else 1):
        dt = x.dtype or ("int64" if x.cpu_data.dtype == np.int64 else "float32")
        shape = x.is_shape if x.is_shape is not None else dt in ("int64", "int32")
        return Tensor(None, list(dims), dt, x.cpu_data, shape)
    return Tensor(x.buf, list(dims))


def _upload_f32(ctx, arr, dims) -> Tensor:
    f = np.ascontiguousarray(arr, np.float32).ravel()
    buf = ctx.pool.acquire(max(4, f.nbytes))
    ctx.backend.write(buf, f)
    return Tensor(buf, list(dims), "float32", f)


def op_identity(ctx, node, ins):
    return _passthrough(ins[0], list(ins[0].dims))


def op_reshape(ctx, node, ins):
    x, shape = ins[0], ins[1] if len(ins) > 1 else None
    new = _ints(shape) if shape is not None and shape.cpu_data is not None else list(x.dims)
    xn = int(np.prod(x.dims)) if x.dims else 1
    for i, d in enumerate(new):
        if d == 0:
            new[i] = x.dims[i]  # allowzero = 0
    known = int(np.prod([d for d in new if d > 0])) if new else 1
    new = [xn // known if d == -1 else d for d in new]
    return _passthrough(x, new)


def op_shape(ctx, node, ins):
    d = list(ins[0].dims)
    return Tensor(None, [len(d)], "int64", np.array(d, np.int64), True)


def op_unsqueeze(ctx, node, ins):
    x, axes = ins[0], ins[1] if len(ins) > 1 else None
    ax = _ints(axes) if axes is not None and axes.cpu_data is not None else _attr_ints(node, "axes", [0])
    dims = list(x.dims) if x.dims is not None else [int(np.asarray(x.cpu_data).size)]
    for a in ax:
        dims.insert(a if a >= 0 else len(dims) + 1 + a, 1)
    if x.on_cpu:
        return Tensor(None, dims, x.dtype or "int64", x.cpu_data, x.is_shape is not False)
    return Tensor(x.buf, dims)


def op_squeeze(ctx, node, ins):
    x, axes = ins[0], ins[1] if len(ins) > 1 else None
    ax = _ints(axes) if axes is not None and axes.cpu_data is not None else _attr_ints(node, "axes", None)
    dims = list(x.dims)
    drop = {a if a >= 0 else len(dims) + a for a in ax} if ax else {i for i, d in enumerate(dims) if d == 1}
    return _passthrough(x, [d for i, d in enumerate(dims) if i not in drop])


def op_constant(ctx, node, ins):
    a = _attr(node, "value")
    if a is not None and a["t"] is not None:
        t = a["t"]
        raw = t["data"] or b""
        if t["dtype"] in ("int64", "int32"):
            data = np.frombuffer(raw, "<i8" if t["dtype"] == "int64" else "<i4").copy()
            return Tensor(None, list(t["dims"]), t["dtype"], data, True)
        if t["dtype"] in ("float32", "float16"):
            f = ctx.f16_to_f32(raw) if t["dtype"] == "float16" else np.frombuffer(raw, "<f4").copy()
            return _upload_f32(ctx, f, t["dims"])
        return Tensor(None, list(t["dims"]), t["dtype"], np.frombuffer(raw, "u1").copy(), True)
    a = _attr(node, "value_ints")
    if a is not None and a["ints"] is not None:
        return Tensor(None, [len(a["ints"])], "int64", np.array(a["ints"], np.int64), True)
    a = _attr(node, "value_int")
    if a is not None and a["i"] is not None:
        return Tensor(None, [], "int64", np.array([a["i"]], np.int64), True)
    a = _attr(node, "value_floats")
    if a is not None and a["floats"] is not None:
        return _upload_f32(ctx, a["floats"], [len(a["floats"])])
    a = _attr(node, "value_float")
    if a is not None and a["f"] is not None:
        return _upload_f32(ctx, [a["f"]], [])
    raise DIError(f"Constant {node['name']}: no recognised value attribute")


def op_constant_of_shape(ctx, node, ins):
    dims = _ints(ins[0])
    n = int(np.prod(dims)) if dims else 1
    a = _attr(node, "value")
    fill, vdt = 0.0, None
    if a is not None and a["t"] is not None and a["t"]["data"]:
        t = a["t"]
        vdt = t["dtype"]
        raw = t["data"]
        fill = {"float32": lambda: float(np.frombuffer(raw[:4], "<f4")[0]),
                "int64": lambda: int(np.frombuffer(raw[:8], "<i8")[0]),
                "int32": lambda: int(np.frombuffer(raw[:4], "<i4")[0]),
                "float16": lambda: float(ctx.f16_to_f32(raw[:2])[0])}.get(vdt, lambda: 0.0)()
    if vdt in ("int64", "int32"):  # shape metadata stays on the host (wgsl-executor.js:270-283)
        return Tensor(None, dims, vdt, np.full(max(n, 0), fill, np.int64 if vdt == "int64" else np.int32), True)
    return _upload_f32(ctx, np.full(max(n, 1), fill, np.float32), dims)


def op_cast(ctx, node, ins):
    x = ins[0]
    to = _attr_int(node, "to", 1)
    if x.on_cpu:
        d = np.asarray(x.cpu_data)
        if to == 7 and d.dtype != np.int64:
            return Tensor(None, list(x.dims), "int64", np.trunc(d.astype(np.float64)).astype(np.int64), x.is_shape is not False)
        if to == 6 and d.dtype != np.int32:
            return Tensor(None, list(x.dims), "int32", np.trunc(d.astype(np.float64)).astype(np.int32), x.is_shape is not False)
        if to == 1 and d.dtype != np.float32:
            return Tensor(None, list(x.dims), "float32", d.astype(np.float32), False)
        return Tensor(None, list(x.dims), x.dtype, d, x.is_shape is not False)
    return Tensor(x.buf, list(x.dims))  # device data is always fp32


def op_slice(ctx, node, ins):
    x = ins[0]
    get = lambda i: _ints(ins[i]) if len(ins) > i and ins[i] is not None and ins[i].cpu_data is not None else None
    starts, ends, axes, steps = get(1), get(2), get(3), get(4)
    if x.on_cpu:  # 1-D slice of a shape vector
        d = np.asarray(x.cpu_data).ravel()
        n = d.size
        s = (starts or [0])[0]
        e = (ends or [n])[0]
        st = (steps or [1])[0] or 1
        s = s + n if s < 0 else s
        e = e + n if e < 0 else e
        s, e = max(0, min(n, s)), max(0, min(n, e))
        out = d[s:e:st] if st > 0 else d[s:e:st]
        return Tensor(None, [int(out.size)], x.dtype or "int64", out.copy(), x.is_shape is not False)
    rank = len(x.dims)
    if rank > 4:
        raise DIError(f"Slice: rank {rank} > 4 not supported")
    starts = starts or []
    axes = axes if axes is not None else list(range(len(starts)))
    steps = steps if steps is not None else [1] * len(starts)
    if any(v != 1 for v in steps):
        raise DIError("Slice: step != 1 not supported")
    out_dim = list(x.dims)
    start = [0] * rank
    for i, ax in enumerate(axes):
        ax = ax + rank if ax < 0 else ax
        s, e = starts[i], ends[i]
        s = s + x.dims[ax] if s < 0 else s
        e = e + x.dims[ax] if e < 0 else e
        s, e = max(0, min(x.dims[ax], s)), max(0, min(x.dims[ax], e))
        start[ax] = s
        out_dim[ax] = max(0, e - s)
    numel = int(np.prod(out_dim))
    cfg = np.zeros(20, np.uint32)
    cfg[0] = rank
    cfg[4:8] = _pad4(out_dim)
    cfg[8:12] = _pad4(_row_major_strides(x.dims))
    cfg[12:16] = _pad4(start)
    cfg[16] = numel
    out = ctx.pool.acquire(max(4, numel * 4))
    ctx.d["slice"](ctx.enc, x.buf, out, ctx.uniform(cfg), numel)
    return Tensor(out, out_dim)


def op_gather(ctx, node, ins):
    data, idx = ins
    if data.is_shape:
        d = np.asarray(data.cpu_data).ravel()
        ii = [i + d.size if i < 0 else i for i in (_ints(idx) if idx.cpu_data is not None else [0])]
        out = np.array([int(d[i]) if 0 <= i < d.size else 0 for i in ii], np.int64)
        return Tensor(None, list(idx.dims or []), "int64", out, True)
    raise DIError(f"Gather {node['name']}: device-tensor path not implemented")


def op_transpose(ctx, node, ins):
    x = ins[0]
    dims = list(x.dims)
    perm = _attr_ints(node, "perm", list(range(len(dims) - 1, -1, -1)))
    new = [dims[i] for i in perm]
    if x.on_cpu:
        return _passthrough(x, new)
    if len(dims) > 4:
        raise DIError(f"Transpose: rank {len(dims)} > 4 not supported")
    numel = int(np.prod(new)) if new else 1
    cfg = np.zeros(20, np.uint32)
    cfg[0] = len(dims)
    cfg[4:8] = _pad4(new, 1)
    cfg[8:12] = _pad4(_row_major_strides(dims))
    cfg[12:16] = _pad4(perm)
    cfg[16] = numel
    out = ctx.pool.acquire(numel * 4)
    ctx.d["transpose"](ctx.enc, x.buf, out, ctx.uniform(cfg), numel)
    return Tensor(out, new)


def op_concat(ctx, node, ins):
    axis = _attr_int(node, "axis", 0)
    first = next((t for t in ins if t is not None), None)
    if axis < 0:
        axis += len(first.dims or [])
    if all(t.on_cpu for t in ins):
        big = any(np.asarray(t.cpu_data).dtype == np.int64 for t in ins)
        out = np.concatenate([np.asarray(t.cpu_data).ravel() for t in ins]).astype(np.int64 if big else np.float32)
        return Tensor(None, [int(out.size)], first.dtype or "int64", out, first.is_shape is not False)
    ins = [ctx.promote(t) if t.on_cpu else t for t in ins]
    dims = list(ins[0].dims)
    dims[axis] = sum(t.dims[axis] for t in ins)
    numel = int(np.prod(dims))
    out = ctx.pool.acquire(numel * 4)
    stripe_out = int(np.prod(dims[axis:]))
    off = 0
    for t in ins:
        stripe_in = int(np.prod(t.dims[axis:]))
        ctx.d["concatCopy"](ctx.enc, t.buf, out, ctx.uniform(np.array([stripe_in, stripe_out, off, t.numel], np.uint32)),
                            t.numel)
        off += stripe_in
    return Tensor(out, dims)


def op_reduce_mean(ctx, node, ins):
    x = ins[0]
    axes = _attr_ints(node, "axes", [len(x.dims) - 1])
    keep = _attr_int(node, "keepdims", 1)
    if len(axes) != 1 or axes[0] not in (-1, len(x.dims) - 1):
        raise DIError(f"ReduceMean: only last-dim reduction supported, got axes {axes}")
    inner = x.dims[-1]
    rows = x.numel // inner
    out = ctx.pool.acquire(rows * 4)
    ctx.d["reduceMean"](ctx.enc, x.buf, out, ctx.uniform(np.array([inner, rows], np.uint32)), rows)
    return Tensor(out, list(x.dims[:-1]) + ([1] if keep else []))


def op_pow(ctx, node, ins):
    a, b = ins
    if b is not None and b.cpu_data is not None and np.asarray(b.cpu_data).size >= 1 and \
            (np.asarray(b.cpu_data).size == 1 or all(d == 1 for d in b.dims)):
        e = float(np.asarray(b.cpu_data).ravel()[0])
        a = ctx.promote(a) if a.on_cpu else a
        out = ctx.pool.acquire(a.numel * 4)
        ctx.d["powScalar"](ctx.enc, a.buf, out, ctx.uniform(np.array([e, 0, 0, 0], np.float32)), a.numel)
        return Tensor(out, list(a.dims))
    raise DIError(f"Pow: non-scalar exponent not supported (b.dims={b.dims if b else None})")


def op_expand(ctx, node, ins):
    x, shape = ins
    new = _ints(shape) if shape is not None and shape.cpu_data is not None else list(x.dims)
    if int(np.prod(new)) != (int(np.prod(x.dims)) if x.dims else 1):
        raise DIError(f"Expand {node['name']}: real broadcast {x.dims} -> {new} not implemented")
    return _passthrough(x, new)


def op_equal(ctx, node, ins):
    a, b = ins
    if a.on_cpu and b.on_cpu:
        x, y = np.asarray(a.cpu_data).ravel(), np.asarray(b.cpu_data).ravel()
        n = max(x.size, y.size)
        xs = np.broadcast_to(x, (n,)) if x.size == 1 else x
        ys = np.broadcast_to(y, (n,)) if y.size == 1 else y
        out = (xs.astype(np.float64) == ys.astype(np.float64)).astype(np.uint8)
        return Tensor(None, list(a.dims if x.size >= y.size else b.dims) or [n], "bool", out, True)
    raise DIError(f"Equal {node['name']}: device path not implemented")


def op_where(ctx, node, ins):
    c, a, b = ins
    if c.on_cpu and a.on_cpu and b.on_cpu:
        cc, x, y = (np.asarray(t.cpu_data).ravel() for t in (c, a, b))
        n = max(cc.size, x.size, y.size)
        pick = lambda v: np.broadcast_to(v, (n,)) if v.size == 1 else v
        out = np.where(pick(cc).astype(bool), pick(x), pick(y)).astype((x if x.size >= y.size else y).dtype)
        return Tensor(None, [n], a.dtype or b.dtype or "int64", out, a.is_shape is not False or b.is_shape is not False)
    raise DIError(f"Where {node['name']}: device path not implemented")


def _binary(op: str):
    npf = {"Add": np.add, "Sub": np.subtract, "Mul": np.multiply, "Div": np.divide}[op]

    def run(ctx, node, ins):
        a, b = ins
        if a.on_cpu and b.on_cpu:  # shape arithmetic on the host
            dims = broadcast_shape(list(a.dims), list(b.dims))
            x, y = np.asarray(a.cpu_data), np.asarray(b.cpu_data)
            big = x.dtype == np.int64 or y.dtype == np.int64
            xa = x.reshape(a.dims) if a.dims else x.reshape(())
            ya = y.reshape(b.dims) if b.dims else y.reshape(())
            if big:
                if op == "Div":  # BigInt division truncates toward zero
                    q = np.trunc(xa.astype(np.float64) / ya.astype(np.float64)).astype(np.int64)
                else:
                    q = npf(xa.astype(np.int64), ya.astype(np.int64))
            else:
                q = npf(xa.astype(np.float32), ya.astype(np.float32)).astype(np.float32)
            out = np.broadcast_to(q, dims).ravel().copy() if dims else np.asarray(q).reshape(1)
            return Tensor(None, dims, "int64" if big else "float32", out, bool(a.is_shape or b.is_shape))
        a = ctx.promote(a) if a.on_cpu else a
        b = ctx.promote(b) if b.on_cpu else b
        dims = broadcast_shape(list(a.dims), list(b.dims))
        numel = int(np.prod(dims)) if dims else 1
        out = ctx.pool.acquire(numel * 4)
        if list(a.dims) == dims and list(b.dims) == dims:
            ctx.d["binary"][op](ctx.enc, a.buf, b.buf, out, numel)
        else:
            if len(dims) > 4:
                raise DIError(f"{op} broadcast: rank {len(dims)} > 4 not supported")
            cfg = np.zeros(20, np.uint32)
            cfg[0] = len(dims)
            cfg[4:8] = _pad4(dims)
            cfg[8:12] = _pad4(_bcast_strides(dims, a.dims))
            cfg[12:16] = _pad4(_bcast_strides(dims, b.dims))
            cfg[16] = numel
            ctx.d["binaryBcast"][op](ctx.enc, a.buf, b.buf, out, ctx.uniform(cfg), numel)
        return Tensor(out, dims)
    return run


def _bcast_strides(dims, tdims):
    """Align right; a size-1 dim broadcast against a larger one gets stride 0."""
    st = [0] * len(dims)
    s = 1
    pad = len(dims) - len(tdims)
    for i in range(len(tdims) - 1, -1, -1):
        st[pad + i] = 0 if (tdims[i] == 1 and dims[pad + i] != 1) else s
        s *= tdims[i]
    return st


def _erf_as(v: float) -> float:
    t = 1.0 / (1.0 + 0.3275911 * abs(v))
    y = 1.0 - (((((1.061405429 * t - 1.453152027) * t) + 1.421413741) * t - 0.284496736) * t + 0.254829592) * t \
        * math.exp(-v * v)
    return y if v >= 0 else -y


UNARY_HOST = {  # the host fast path of the shape subgraph (e.g. Shape -> Gather -> Cast -> Sqrt)
    "Sigmoid": lambda v: 1.0 / (1.0 + math.exp(-v)),
    "Sqrt": lambda v: math.sqrt(max(v, 0.0)),
    "Abs": abs,
    "Neg": lambda v: -v,
    "Erf": _erf_as,
}


def _unary(op: str):
    def run(ctx, node, ins):
        x = ins[0]
        if x.on_cpu and op in UNARY_HOST:
            out = np.array([UNARY_HOST[op](float(v)) for v in np.asarray(x.cpu_data).ravel()], np.float32)
            return Tensor(None, list(x.dims or []), "float32", out, True)
        x = ctx.promote(x) if x.on_cpu else x
        out = ctx.pool.acquire(x.byte_length)
        ctx.d["unary"][op](ctx.enc, x.buf, out, x.numel)
        return Tensor(out, list(x.dims))
    return run


def op_group_norm(ctx, node, ins):
    x, g, b = (ctx.promote(t) if t is not None and t.on_cpu else t for t in ins)
    if not x.dims or len(x.dims) < 2:
        raise DIError(f"GroupNorm {node['name']}: expected rank >= 2, got {x.dims}")
    N, C = x.dims[0], x.dims[1]
    HW = int(np.prod(x.dims[2:])) if len(x.dims) > 2 else 1
    G = _attr_int(node, "num_groups", 32)
    if C % G:
        raise DIError(f"GroupNorm: C={C} not divisible by G={G}")
    a = _attr(node, "epsilon")
    eps = float(a["f"]) if a is not None and a["f"] is not None else 1e-5
    cfg = np.zeros(8, np.uint32)
    cfg[:4] = [N, G, C // G, HW]
    cfg[4] = np.array([eps], np.float32).view(np.uint32)[0]
    out = ctx.pool.acquire(N * C * HW * 4)
    ctx.d["groupNorm"](ctx.enc, x.buf, g.buf, b.buf, out, ctx.uniform(cfg), G, N)
    return Tensor(out, list(x.dims))


def op_affine_bcast(ctx, node, ins):
    x, g, b = (ctx.promote(t) if t.on_cpu else t for t in ins)
    dims = list(x.dims)
    if len(dims) > 4:
        raise DIError(f"AffineBcast: rank {len(dims)} > 4")
    numel = int(np.prod(dims))
    cfg = np.zeros(20, np.uint32)
    cfg[0] = len(dims)
    cfg[4:8] = _pad4(dims)
    cfg[8:12] = _pad4(_bcast_strides(dims, dims))
    cfg[12:16] = _pad4(_bcast_strides(dims, g.dims))
    cfg[16] = numel
    out = ctx.pool.acquire(numel * 4)
    ctx.d["affineBcast"](ctx.enc, x.buf, g.buf, b.buf, out, ctx.uniform(cfg), numel)
    return Tensor(out, dims)


def op_silu(ctx, node, ins):
    x = ins[0]
    out = ctx.pool.acquire(x.byte_length)
    ctx.d["unary"]["SiLU"](ctx.enc, x.buf, out, x.numel)
    return Tensor(out, list(x.dims))


def op_instance_norm(ctx, node, ins):
    x, g, b = ins
    if len(x.dims) == 4:
        N, C, HW = x.dims[0], x.dims[1], x.dims[2] * x.dims[3]
    elif len(x.dims) == 3:
        N, C, HW = x.dims
    else:
        raise DIError(f"InstanceNorm needs 3D or 4D input, got {len(x.dims)}D")
    g = ctx.promote(g) if g.on_cpu else g
    b = ctx.promote(b) if b.on_cpu else b
    out = ctx.pool.acquire(x.byte_length)
    ctx.d["instanceNorm"](ctx.enc, x.buf, g.buf, b.buf, out, ctx.uniform(np.array([C, HW, N, 0], np.uint32)), C, N)
    return Tensor(out, list(x.dims))


def op_softmax(ctx, node, ins):
    x = ins[0]
    axis = _attr_int(node, "axis", -1)
    ax = axis + len(x.dims) if axis < 0 else axis
    if ax != len(x.dims) - 1:
        raise DIError(f"Softmax: only last-axis supported, got axis={axis} dims={x.dims}")
    inner = x.dims[ax]
    rows = x.numel // inner
    out = ctx.pool.acquire(x.byte_length)
    ctx.d["softmax"](ctx.enc, x.buf, out, ctx.uniform(np.array([inner, rows], np.uint32)), rows)
    return Tensor(out, list(x.dims))


def op_matmul(ctx, node, ins):
    a, b = ins
    M, K, N = a.dims[-2], a.dims[-1], b.dims[-1]
    batch = int(np.prod(a.dims[:-2])) if len(a.dims) > 2 else 1
    bbatch = int(np.prod(b.dims[:-2])) if len(b.dims) > 2 else 1
    if bbatch not in (1, batch):
        raise DIError(f"MatMul: batch mismatch a={a.dims} b={b.dims}")
    if batch == 1 and bbatch > 1:
        raise DIError("MatMul: batched B with unbatched A not supported")
    out = ctx.pool.acquire(batch * M * N * 4)
    ctx.d["matmul"](ctx.enc, a.buf, b.buf, out, ctx.uniform(np.array([M, N, K, 1 if bbatch > 1 else 0], np.uint32)),
                    M, N, batch)
    return Tensor(out, list(a.dims[:-2]) + [M, N])


def op_gemm(ctx, node, ins):
    a, b, c = ins
    tb = _attr_int(node, "transB", 0)
    M, K = a.dims[0], a.dims[1]
    N = b.dims[0] if tb else b.dims[1]
    out = ctx.pool.acquire(M * N * 4)
    ctx.d["gemm"](ctx.enc, a.buf, b.buf, c.buf, out, ctx.uniform(np.array([M, N, K, tb], np.uint32)), M, N)
    return Tensor(out, [M, N])


def op_conv(ctx, node, ins):
    x, w, bias = ins
    ks = _attr_ints(node, "kernel_shape", [3, 3])
    if ks[0] != ks[1]:
        raise DIError(f"Conv: non-square kernel {ks} not supported")
    st = _attr_ints(node, "strides", [1, 1])
    if st[0] != st[1]:
        raise DIError(f"Conv: non-square stride {st} not supported")
    K, S = ks[0], st[0]
    pads = _attr_ints(node, "pads", [(K - 1) >> 1] * 4)
    if len(set(pads)) != 1:
        raise DIError(f"Conv: asymmetric pads {pads} not supported")
    P = pads[0]
    N, Ci, H, W = x.dims
    if N != 1:
        raise DIError(f"Conv: batch N={N} not supported")
    Co = w.dims[0]
    Ho, Wo = (H + 2 * P - K) // S + 1, (W + 2 * P - K) // S + 1
    out = ctx.pool.acquire(N * Co * Ho * Wo * 4)
    cfg = np.array([Ci, Co, K, K * K, H, W, P, S, Ho, Wo, 0, 0], np.uint32)
    ctx.d["convMM"](ctx.enc, x.buf, w.buf, bias.buf, out, ctx.uniform(cfg), Co, Ho * Wo)
    return Tensor(out, [N, Co, Ho, Wo])


def op_resize(ctx, node, ins):
    x = ins[0]
    mode = _attr_str(node, "mode", "nearest")
    if mode != "nearest":
        raise DIError(f"Resize mode {mode} not supported")
    sc = ins[2].cpu_data if len(ins) > 2 and ins[2] is not None and ins[2].cpu_data is not None else None
    sh = float(np.asarray(sc).ravel()[2]) if sc is not None else 2.0
    sw = float(np.asarray(sc).ravel()[3]) if sc is not None else 2.0
    N, C, H, W = x.dims
    Ho, Wo = int(math.floor(H * sh + 0.5)), int(math.floor(W * sw + 0.5))
    numel = N * C * Ho * Wo
    out = ctx.pool.acquire(numel * 4)
    ctx.d["resizeNearest"](ctx.enc, x.buf, out, ctx.uniform(np.array([C, H, W, Ho, Wo, numel, 0, 0], np.uint32)),
                           numel)
    return Tensor(out, [N, C, Ho, Wo])


OPS = {
    "Identity": op_identity, "Reshape": op_reshape, "Shape": op_shape, "Unsqueeze": op_unsqueeze,
    "Squeeze": op_squeeze, "Constant": op_constant, "ConstantOfShape": op_constant_of_shape, "Cast": op_cast,
    "Slice": op_slice, "Gather": op_gather, "Transpose": op_transpose, "Concat": op_concat,
    "ReduceMean": op_reduce_mean, "Pow": op_pow, "Expand": op_expand, "Equal": op_equal, "Where": op_where,
    "GroupNorm": op_group_norm, "AffineBcast": op_affine_bcast, "Silu": op_silu,
    "InstanceNormalization": op_instance_norm, "Softmax": op_softmax, "MatMul": op_matmul, "Gemm": op_gemm,
    "Conv": op_conv, "Resize": op_resize,
}
for _op in ("Add", "Sub", "Mul", "Div"):
    OPS[_op] = _binary(_op)
for _op in ("Sigmoid", "Sqrt", "Erf", "Abs", "Neg", "Sin", "Cos"):
    OPS[_op] = _unary(_op)

# ops that read only host metadata: their inputs are never promoted (wgsl-executor.js:1310)
METADATA_OPS = {"Reshape", "Shape", "Unsqueeze", "Squeeze", "Gather", "Slice", "Concat", "Constant",
                "ConstantOfShape", "Cast", "Expand", "Equal", "Where", "Identity", "Transpose"}
BINARY_SHAPE_AWARE = {"Add", "Sub", "Mul", "Div"}
# ops with a host path for 1-element host constants; every other device op gets them promoted (the
# reference keeps such scalars unpromoted for all ops, so e.g. a MatMul on one would fail there)
HOST_SCALAR_OPS = BINARY_SHAPE_AWARE | {"Pow", "Sigmoid", "Sqrt", "Erf", "Abs", "Neg"}


def plan_execution(graph) -> dict:
    """wgsl-executor.js:1157-1171: op coverage of a graph."""
    unsupported: dict[str, int] = {}
    n_ok = 0
    for n in graph["nodes"]:
        if n["op_type"] in OPS:
            n_ok += 1
        else:
            unsupported[n["op_type"]] = unsupported.get(n["op_type"], 0) + 1
    total = len(graph["nodes"])
    return {"total": total, "supportedCount": n_ok, "coverage": n_ok / total if total else 1.0,
            "unsupportedOps": sorted(unsupported.items(), key=lambda kv: -kv[1])}


# ---------------------------------------------------------------------------------------------------
# Backend over libdi and the walk
# ---------------------------------------------------------------------------------------------------
class GpuBackend:
    """libdi device: flat fp32 CUDA buffers, the op-family closures of ops.py as dispatchers."""

    def __init__(self, ctx):
        from . import ops
        self.ctx = ctx
        self.ops = ops
        d = {"unary": {}, "binary": {}, "binaryBcast": {}}
        for op in ("Sigmoid", "Sqrt", "SiLU", "GELU", "Erf", "Abs", "Neg", "Sin", "Cos", "Exp", "Log"):
            d["unary"][op] = ops.unary(ctx, op)
        for op in ("Add", "Sub", "Mul", "Div", "Max", "Min"):
            d["binary"][op] = ops.binary(ctx, op)
            d["binaryBcast"][op] = ops.binaryBcast(ctx, op)
        for name in ("softmax", "instanceNorm", "layerNorm", "matmul", "gemm", "convMM", "resizeNearest",
                     "reduceMean", "concatCopy", "transpose", "powScalar", "slice", "affineBcast", "groupNorm"):
            d[name] = getattr(ops, name)(ctx)
        self.dispatchers = d

    def alloc(self, nbytes: int):
        return self.ops.createOutput(self.ctx, nbytes)

    @staticmethod
    def nbytes(buf) -> int:
        return int(buf.numel()) * 4

    def write(self, buf, arr: np.ndarray) -> None:
        import torch
        a = np.ascontiguousarray(arr, np.float32).ravel()
        buf.view(-1)[: a.size].copy_(torch.from_numpy(a))

    def copy(self, src, dst, nbytes: int) -> None:
        n = nbytes // 4
        dst.view(-1)[:n].copy_(src.view(-1)[:n])

    def read(self, buf, nbytes: int) -> np.ndarray:
        return self.ops.readBack(self.ctx, buf, nbytes)

    def encoder(self):
        return self.ops.createCommandEncoder(self.ctx)

    def uniform(self, arr):
        return self.ops.createUniform(self.ctx, arr)

    def sync(self) -> None:
        self.ops.submit(self.ctx, None)


class _RunCtx:
    """The `ctx` the reference passes to every op: pool, dispatchers, encoder, weights, promote."""

    def __init__(self, backend, pool, weights):
        from .graph import f16_bytes_to_f32
        self.backend = backend
        self.pool = pool
        self.weights = weights
        self.d = backend.dispatchers
        self.enc = backend.encoder()
        self.uniform = backend.uniform
        self.f16_to_f32 = f16_bytes_to_f32
        self.promoted: list = []  # pool buffers of promoted host tensors (never named in the environment)

    def promote(self, t: Tensor) -> Tensor:
        """A host tensor uploaded to a pool buffer as fp32 (wgsl-executor.js:1279-1293)."""
        if t is None or t.buf is not None or t.cpu_data is None:
            return t
        f = np.asarray(t.cpu_data).astype(np.float32).ravel()
        buf = self.pool.acquire(max(4, f.nbytes))
        self.backend.write(buf, f)
        self.promoted.append(buf)
        return Tensor(buf, list(t.dims) if t.dims else [int(f.size)], "float32")


class Executor:
    def __init__(self, backend, graph: dict, weights: WeightCache):
        self.backend = backend
        self.graph = graph
        self.weights = weights
        self.pool = BufferPool(backend)
        if not graph.get("inputs") or not graph.get("outputs"):
            ins, outs = infer_graph_io(graph["nodes"], set(weights.tensors))
            if not graph.get("inputs"):
                graph["inputs"] = ins
            if not graph.get("outputs"):
                graph["outputs"] = outs
        self.consumers: dict[str, int] = {}
        for n in graph["nodes"]:
            for i in n["inputs"]:
                self.consumers[i] = self.consumers.get(i, 0) + 1
        for o in graph["outputs"]:
            self.consumers[o["name"]] = self.consumers.get(o["name"], 0) + 1
        self.graph_input_names = {i["name"] for i in graph.get("inputs") or []}
        self.op_hist: dict[str, int] = {}

    def run(self, inputs: dict) -> dict:
        """One forward.  inputs: name -> Tensor, or a host array (uploaded; `dims` from its shape), or a
        host-only Tensor (cpu_data, e.g. an int64 timestep).  Returns name -> Tensor backed by buffers
        that later runs never reuse."""
        consumers = dict(self.consumers)
        env: dict[str, Tensor] = {}
        for name, val in inputs.items():
            if isinstance(val, Tensor):
                env[name] = val
            elif isinstance(val, np.ndarray):
                buf = self.backend.alloc(max(4, val.size * 4))
                self.backend.write(buf, val.astype(np.float32))
                env[name] = Tensor(buf, list(val.shape))
            else:
                raise DIError(f'unsupported input seed for "{name}": {type(val).__name__}')
        ctx = _RunCtx(self.backend, self.pool, self.weights)
        deferred = []
        self.op_hist = {}
        for ni, node in enumerate(self.graph["nodes"]):
            op = OPS.get(node["op_type"])
            if op is None:
                raise DIError(f"unsupported op @{ni}: {node['op_type']} ({node['name']})")
            self.op_hist[node["op_type"]] = self.op_hist.get(node["op_type"], 0) + 1
            ins = []
            for name in node["inputs"]:
                if not name:
                    ins.append(None)
                elif name in env:
                    ins.append(env[name])
                elif self.weights.has(name):
                    ins.append(self.weights.get(name))
                else:
                    raise DIError(f"tensor not found @{ni} {node['op_type']}: {name}")
            if node["op_type"] not in METADATA_OPS:
                keep_int = node["op_type"] in BINARY_SHAPE_AWARE
                fixed = []
                for t in ins:
                    if t is None or t.buf is not None:
                        fixed.append(t)
                    elif keep_int and t.cpu_data is not None and np.asarray(t.cpu_data).dtype in (np.int64, np.int32):
                        fixed.append(t)
                    elif t.cpu_data is not None and np.asarray(t.cpu_data).size == 1 and \
                            node["op_type"] in HOST_SCALAR_OPS:
                        fixed.append(t)  # scalar host constants feed the Pow / shape fast paths
                    else:
                        fixed.append(ctx.promote(t))
                ins = fixed
            try:
                out = op(ctx, node, ins)
            except DIError as e:
                raise DIError(f"op @{ni} {node['op_type']} ({node['name']}) failed: {e}") from e
            if len(node["outputs"]) > 1:
                raise DIError(f"multi-output op not supported yet: {node['op_type']}")
            env[node["outputs"][0]] = out
            # inputs whose last consumer this was: released only after the walk is submitted, so no
            # later op in the same submission can be handed a buffer an earlier op still reads
            out_buf = out.buf if out is not None else None
            for name in node["inputs"]:
                if not name or name not in env:
                    continue
                t = env[name]
                consumers[name] = consumers.get(name, 0) - 1
                if consumers[name] <= 0 and t is not None and t.buf is not None and t.buf is not out_buf \
                        and not self.weights.has(name) and name not in self.graph_input_names:
                    deferred.append(t.buf)
                    del env[name]
        # graph outputs into fresh buffers (never pool-owned), then fence, then release
        snapshots = {}
        for o in self.graph["outputs"]:
            t = env.get(o["name"])
            if t is None or t.buf is None:
                continue
            stable = self.backend.alloc(max(4, t.numel * 4))
            self.backend.copy(t.buf, stable, t.numel * 4)
            snapshots[o["name"]] = Tensor(stable, list(t.dims))
        self.backend.sync()
        # Everything the walk acquired is idle now.  Unlike the reference, the graph outputs' own buffers
        # (already copied into their snapshots) and the buffers of promoted host tensors go back to the
        # pool too, so repeated runs allocate nothing but the snapshots.
        done = set()
        for buf in deferred + ctx.promoted:
            if id(buf) in done:
                continue
            done.add(id(buf))
            self.pool.release(buf)
        # alias-held intermediates (Reshape / Identity views) and snapshotted outputs still in env go back too
        for name, t in env.items():
            if t is None or t.buf is None or id(t.buf) in done:
                continue
            if self.weights.has(name) or name in self.graph_input_names or not self.pool.owns(t.buf):
                continue
            done.add(id(t.buf))
            self.pool.release(t.buf)
        return {o["name"]: snapshots.get(o["name"], env.get(o["name"])) for o in self.graph["outputs"]}
