"""Batched one-step SD-Turbo text-to-image (config 5): text encoder -> U-Net at t = 999 with the Euler
scheduler on the device -> VAE decoder, as one libdi pipeline (the GPU part of pipeline.js's SD-Turbo
generate path: encodeSDPrompt, scaleModelInput, unetForwardWGSL, step, vaeDecodeWGSL).

    p = Text2Image(ctx, B=64, seed=4)
    img = p.forward_host(ids, latent)       # int32 [B, 77], fp32 [B, 4, 64, 64] -> fp32 [B, 3, 512, 512]
    img = p.generate(ids, noise_seed=0)     # latent from sampleNoiseLatent(B, 64, 64, seed, initNoiseSigma)
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import Context, default_context, lib, view
from .blocks import _weight_cb
from .scheduler import sample_noise_latent
from .text_encoder import CONTEXT, WIDTH, sd_pad_ids, text_flops
from .unet import unet_flops
from .vae import vae_flops


class Text2Image:
    def __init__(self, ctx: Context | None = None, B=1, h=64, w=64, text_layers=24, seed=4, weights=None):
        self.ctx = ctx or default_context()
        self._cb = _weight_cb(weights)
        hh = ctypes.c_void_p()
        self.ctx.check(lib().di_t2i_create(self.ctx.h, B, h, w, text_layers, seed, self._cb, None,
                                           ctypes.byref(hh)), "di_t2i_create")
        self.h = hh
        self.B, self.lh, self.lw, self.text_layers = B, h, w, text_layers
        ps = [ctypes.c_void_p() for _ in range(5)]
        lib().di_t2i_io(self.h, *[ctypes.byref(p) for p in ps])
        self.ids = view(ps[0].value, (B, CONTEXT), "i32")
        self.latent = view(ps[1].value, (B, 4, h, w))
        self.image = view(ps[2].value, (B, 3, 8 * h, 8 * w))
        self.context = view(ps[3].value, (B, CONTEXT, WIDTH))
        self.eps = view(ps[4].value, (B, 4, h, w))
        n = ctypes.c_int()
        wb, ab = ctypes.c_size_t(), ctypes.c_size_t()
        s0 = ctypes.c_float()
        lib().di_t2i_info(self.h, ctypes.byref(n), ctypes.byref(wb), ctypes.byref(ab), ctypes.byref(s0))
        self.launches, self.weight_bytes, self.act_bytes = n.value, wb.value, ab.value
        self.sigma0 = s0.value  # initNoiseSigma of the one-step schedule

    def flops(self) -> dict:
        return {"text": text_flops(self.B, CONTEXT, self.text_layers), "unet": unet_flops(self.B, self.lh, self.lw),
                "vae": vae_flops(self.B, self.lh, self.lw)}

    def forward(self, stage: int = -1) -> None:
        """Enqueue the pipeline (stage -1) or one stage (0 text, 1 U-Net + scheduler, 2 VAE)."""
        self.ctx.check(lib().di_t2i_forward(self.h, stage), "di_t2i_forward")

    def forward_host(self, ids, latent) -> np.ndarray:
        a = np.ascontiguousarray(ids, np.int32).reshape(self.B, CONTEXT)
        lat = np.ascontiguousarray(latent, np.float32).reshape(self.B, 4, self.lh, self.lw)
        out = np.empty((self.B, 3, 8 * self.lh, 8 * self.lw), np.float32)
        self.ctx.check(lib().di_t2i_forward_host(self.h, a.ctypes.data_as(ctypes.c_void_p),
                                                 lat.ctypes.data_as(ctypes.c_void_p),
                                                 out.ctypes.data_as(ctypes.c_void_p)), "di_t2i_forward_host")
        return out

    def generate(self, ids, noise_seed: int = 0) -> np.ndarray:
        lat = sample_noise_latent(self.B, self.lh, self.lw, noise_seed, self.sigma0)
        return self.forward_host(sd_pad_ids(ids), lat)

    def close(self):
        if getattr(self, "h", None):
            lib().di_t2i_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
