"""SD-Turbo U-Net plan: the B200 replacement of unetForwardWGSL (unet-wgsl.js:145-195).

`UNet` owns a libdi plan (weights packed once, every launch recorded, replayed as one CUDA graph).
`unet_forward_wgsl(sample, timestep, cond, opts)` keeps the reference's call shape and result schema
({out, dims, ms}).
"""
from __future__ import annotations

import ctypes
import time

import numpy as np

from . import Context, DIError, WEIGHT_FN, default_context, lib, view


class UNet:
    """SD2.1-architecture U-Net (SD-Turbo), fp16 weights and activations, fp32 accumulation.

    weights: optional callable(name, n) -> float32 array of n values in the diffusers / PyTorch layout
    (e.g. tensors read from an ONNX / safetensors file); names it does not know fall back to the
    seeded generator."""

    def __init__(self, ctx: Context | None = None, B: int = 1, H: int = 64, W: int = 64, ctx_len: int = 77,
                 seed: int = 3, weights=None):
        self.ctx = ctx or default_context()
        self.B, self.H, self.W, self.ctx_len = B, H, W, ctx_len
        self._cb = None
        if weights is not None:
            def _fn(name, n, dst, _user):
                try:
                    arr = weights(name.decode(), int(n))
                except KeyError:
                    return 1
                if arr is None:
                    return 1
                arr = np.ascontiguousarray(arr, np.float32).ravel()
                if arr.size != n:
                    return 1
                ctypes.memmove(dst, arr.ctypes.data, 4 * n)
                return 0
            self._cb = WEIGHT_FN(_fn)
        h = ctypes.c_void_p()
        self.ctx.check(lib().di_unet_create(self.ctx.h, B, H, W, ctx_len, seed, self._cb, None, ctypes.byref(h)),
                       "di_unet_create")
        self.h = h
        ps = [ctypes.c_void_p() for _ in range(4)]
        self.ctx.check(lib().di_unet_io(self.h, *[ctypes.byref(p) for p in ps]), "di_unet_io")
        self.latent = view(ps[0].value, (B, 4, H, W))
        self.t = view(ps[1].value, (B,))
        self.context = view(ps[2].value, (B, ctx_len, 1024))
        self.out = view(ps[3].value, (B, 4, H, W))
        n = ctypes.c_int()
        wb, ab = ctypes.c_size_t(), ctypes.c_size_t()
        lib().di_unet_info(self.h, ctypes.byref(n), ctypes.byref(wb), ctypes.byref(ab))
        self.launches, self.weight_bytes, self.act_bytes = n.value, wb.value, ab.value

    def ops(self):
        """Per-op metadata: dict of numpy arrays kind / flops / bytes / kernels (one entry per recorded op)."""
        n = ctypes.c_int()
        lib().di_unet_ops(self.h, ctypes.byref(n), None, None, None, None)
        k = np.zeros(n.value, np.int32)
        f = np.zeros(n.value, np.float64)
        b = np.zeros(n.value, np.float64)
        kn = np.zeros(n.value, np.int32)
        self.ctx.check(lib().di_unet_ops(self.h, ctypes.byref(n), k.ctypes.data, f.ctypes.data, b.ctypes.data,
                                         kn.ctypes.data), "di_unet_ops")
        return {"kind": k, "flops": f, "bytes": b, "kernels": kn}

    def profile(self, reps: int = 10) -> np.ndarray:
        """Mean device ms of every op (a profiling graph with an event-record node between ops)."""
        n = len(self.ops()["kind"])
        ms = np.zeros(n, np.float32)
        self.ctx.check(lib().di_unet_profile(self.h, reps, ms.ctypes.data), "di_unet_profile")
        return ms

    def profile_kind(self, kind: int, reps: int = 20) -> float:
        """Mean device ms per step of the ops of one kind (0 GEMM/conv, 1 attention, 2 norm, 3 other) alone."""
        ms = ctypes.c_float()
        self.ctx.check(lib().di_unet_profile_kind(self.h, kind, reps, ctypes.byref(ms)), "di_unet_profile_kind")
        return ms.value

    def forward(self) -> None:
        """Enqueue one forward on the context stream (reads self.latent / t / context, writes self.out)."""
        self.ctx.check(lib().di_unet_forward(self.h), "di_unet_forward")

    def __call__(self, latent, t, context):
        """Device tensors in, device tensor out (a view of the plan's output buffer)."""
        self.latent.copy_(latent)
        self.t.copy_(t if hasattr(t, "shape") and t.shape else self.t.new_full((self.B,), float(t)))
        self.context.copy_(context)
        self.forward()
        return self.out

    def forward_host(self, latent: np.ndarray, t, context: np.ndarray) -> np.ndarray:
        """Host arrays in, host array out, synchronous (H2D + forward + D2H through the C ABI)."""
        lat = np.ascontiguousarray(latent, np.float32)
        tv = np.ascontiguousarray(np.broadcast_to(np.asarray(t, np.float32), (self.B,)))
        cx = np.ascontiguousarray(context, np.float32)
        out = np.empty((self.B, 4, self.H, self.W), np.float32)
        self.ctx.check(lib().di_unet_forward_host(self.h, lat.ctypes.data, tv.ctypes.data, cx.ctypes.data,
                                                  out.ctypes.data), "di_unet_forward_host")
        return out

    def set_schedule(self, in_scale: float = 1.0, dt: float = 0.0):
        """Scheduler on the device (scheduler.js:95-110): conv_in sees float(latent * in_scale) and the plan
        writes `self.next` = float(latent + dt * eps) beside `self.out`.  Returns the `next` view."""
        nx = ctypes.c_void_p()
        self.ctx.check(lib().di_unet_sched(self.h, float(in_scale), float(dt), ctypes.byref(nx)), "di_unet_sched")
        self.next = view(nx.value, (self.B, 4, self.H, self.W))
        return self.next

    def close(self):
        if getattr(self, "h", None):
            lib().di_unet_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def unet_flops(B: int = 1, H: int = 64, W: int = 64, Sk: int = 77) -> float:
    """Algorithmic FLOPs (2 per MAC) of one SD2.1 U-Net forward: convs, linears, attention QK^T and PV."""
    f = 2.0 * B * H * W * 320 * 9 * 4 + 2.0 * B * H * W * 4 * 9 * 320 + 2.0 * B * 1280 * (320 + 1280)

    def res(ci, co, h, w):
        x = 2.0 * B * h * w * co * 9 * (ci + co) + 2.0 * B * co * 1280
        return x + (2.0 * B * h * w * co * ci if ci != co else 0.0)

    def tr(c, h, w):
        m, hw = B * h * w, h * w
        lin = 2.0 * m * c * c * (1 + 3 + 1 + 1 + 1 + 1) + 2.0 * m * 8 * c * c + 2.0 * m * 4 * c * c
        return lin + 2.0 * B * Sk * 2 * c * 1024 + 4.0 * B * c * hw * hw + 4.0 * B * c * hw * Sk

    ch = [320, 640, 1280, 1280]
    h, w, c = H, W, 320
    skips = [320]
    for i in range(4):
        for _ in range(2):
            f += res(c, ch[i], h, w)
            c = ch[i]
            if i < 3:
                f += tr(c, h, w)
            skips.append(c)
        if i < 3:
            f += 2.0 * B * (h // 2) * (w // 2) * c * 9 * c
            h, w = h // 2, w // 2
            skips.append(c)
    f += res(1280, 1280, h, w) * 2 + tr(1280, h, w)
    rch = [1280, 1280, 640, 320]
    for i in range(4):
        for _ in range(3):
            s = skips.pop()
            f += res(c + s, rch[i], h, w)
            c = rch[i]
            if i > 0:
                f += tr(c, h, w)
        if i < 3:
            h, w = h * 2, w * 2
            f += 2.0 * B * h * w * c * 9 * c
    return f


_plans = {}


def unet_forward_wgsl(sample, timestep, cond, opts=None):
    """unetForwardWGSL(sample, timestep, cond, {B,H,W,tokens,dim}) -> {out, dims, ms} (unet-wgsl.js:145-195)."""
    o = dict(opts or {})
    B, H, W = o.get("B", 1), o.get("H", 64), o.get("W", 64)
    tokens, dim = o.get("tokens", 77), o.get("dim", 1024)
    if dim != 1024:
        raise DIError("cross-attention dim must be 1024 (SD2.1)")
    key = (B, H, W, tokens)
    if key not in _plans:
        _plans[key] = UNet(B=B, H=H, W=W, ctx_len=tokens, seed=o.get("seed", 3))
    u = _plans[key]
    t0 = time.perf_counter()
    out = u.forward_host(np.asarray(sample, np.float32).reshape(B, 4, H, W), timestep,
                         np.asarray(cond, np.float32).reshape(B, tokens, dim))
    return {"out": out.ravel(), "dims": [B, 4, H, W], "ms": (time.perf_counter() - t0) * 1e3}
