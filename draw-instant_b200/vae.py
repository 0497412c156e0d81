"""SD VAE decoder plan (config 5's image decode): the libdi replacement of vaeDecodeWGSL (vae-wgsl.js:99-144).

    v = VAEDecoder(ctx, B=1, h=64, w=64, seed=4)
    image = v.forward_host(latent)          # [B, 4, h, w] fp32 -> [B, 3, 8h, 8w] fp32 (latent / 0.18215 applied)
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import Context, default_context, lib, view
from .blocks import _weight_cb


def vae_flops(B: int, h: int, w: int) -> float:
    """Algorithmic FLOPs of one decode (convs, 1x1 shortcuts, attention projections and products)."""
    f = 2.0 * 4 * 4 * h * w  # post_quant_conv
    f += 2.0 * 512 * 9 * 4 * h * w  # conv_in
    conv = lambda ci, co, hw: 2.0 * co * 9 * ci * hw
    f += 2 * (conv(512, 512, h * w) * 2)  # mid resnets
    hw = h * w
    f += 2.0 * hw * 512 * 512 * 4 + 2 * 2.0 * hw * hw * 512  # attention projections + QK / PV
    chans = [512, 512, 256, 128]
    cin = 512
    res = hw
    for i, co in enumerate(chans):
        for j in range(3):
            ci = cin if j == 0 else co
            f += conv(ci, co, res) + conv(co, co, res)
            if ci != co:
                f += 2.0 * co * ci * res
        cin = co
        if i < 3:
            res *= 4
            f += conv(co, co, res)
    f += conv(128, 3, res)
    return B * f


class VAEDecoder:
    """Parameter names are diffusers' AutoencoderKL ("post_quant_conv.weight", "decoder.conv_in.weight",
    ...); `weights(name, n)` may supply any of them (else the seeded generator)."""

    def __init__(self, ctx: Context | None = None, B=1, h=64, w=64, seed=4, weights=None):
        self.ctx = ctx or default_context()
        self._cb = _weight_cb(weights)
        hh = ctypes.c_void_p()
        self.ctx.check(lib().di_vae_create(self.ctx.h, B, h, w, seed, self._cb, None, ctypes.byref(hh)),
                       "di_vae_create")
        self.h = hh
        self.B, self.lh, self.lw = B, h, w
        pl, pi = ctypes.c_void_p(), ctypes.c_void_p()
        lib().di_vae_io(self.h, ctypes.byref(pl), ctypes.byref(pi))
        self.latent = view(pl.value, (B, 4, h, w))
        self.image = view(pi.value, (B, 3, 8 * h, 8 * w))
        n = ctypes.c_int()
        wb, ab = ctypes.c_size_t(), ctypes.c_size_t()
        lib().di_vae_info(self.h, ctypes.byref(n), ctypes.byref(wb), ctypes.byref(ab))
        self.launches, self.weight_bytes, self.act_bytes = n.value, wb.value, ab.value

    def forward(self):
        self.ctx.check(lib().di_vae_forward(self.h), "di_vae_forward")

    def forward_host(self, latent) -> np.ndarray:
        lat = np.ascontiguousarray(latent, np.float32)
        out = np.empty((self.B, 3, 8 * self.lh, 8 * self.lw), np.float32)
        self.ctx.check(lib().di_vae_forward_host(self.h, lat.ctypes.data_as(ctypes.c_void_p),
                                                 out.ctypes.data_as(ctypes.c_void_p)), "di_vae_forward_host")
        return out

    def ops(self):
        n = ctypes.c_int()
        lib().di_vae_ops(self.h, ctypes.byref(n), None, None, None, None)
        k = np.empty(n.value, np.int32)
        f = np.empty(n.value, np.float64)
        b = np.empty(n.value, np.float64)
        kr = np.empty(n.value, np.int32)
        lib().di_vae_ops(self.h, ctypes.byref(n), k.ctypes.data, f.ctypes.data, b.ctypes.data, kr.ctypes.data)
        return {"kind": k, "flops": f, "bytes": b, "kernels": kr}

    def profile_kind(self, kind: int, reps: int = 10) -> float:
        ms = ctypes.c_float()
        self.ctx.check(lib().di_vae_profile_kind(self.h, kind, reps, ctypes.byref(ms)), "di_vae_profile_kind")
        return ms.value

    def __del__(self):
        try:
            if getattr(self, "h", None):
                lib().di_vae_destroy(self.h)
                self.h = None
        except Exception:  # interpreter shutdown
            pass
