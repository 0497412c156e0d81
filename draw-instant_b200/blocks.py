"""Fused blocks: planned replacements of the reference's fused-*.js modules.

ResNetBlock      fused-resnet.js (GN+SiLU -> conv3x3 -> +temb -> GN+SiLU -> conv3x3 -> +x), fp32 NCHW I/O
TransformerBlock fused-block-full.js, as the SD2.1 Transformer2DModel block, fp16 token-major I/O
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import Context, WEIGHT_FN, default_context, lib, view


def _weight_cb(weights):
    if weights is None:
        return None

    def _fn(name, n, dst, _user):
        arr = weights(name.decode(), int(n))
        if arr is None:
            return 1
        arr = np.ascontiguousarray(arr, np.float32).ravel()
        if arr.size != n:
            return 1
        ctypes.memmove(dst, arr.ctypes.data, 4 * n)
        return 0

    return WEIGHT_FN(_fn)


class ResNetBlock:
    """Config-1 ResNet block.  Parameter names: norm1.{weight,bias}, conv1.{weight,bias},
    time_emb_proj.{weight,bias}, norm2.*, conv2.*; defaults drawn from `seed`."""

    def __init__(self, ctx: Context | None = None, N=1, C=320, H=64, W=64, Tdim=1280, seed=0, eps=1e-5,
                 temb_silu=True, weights=None):
        self.ctx = ctx or default_context()
        self._cb = _weight_cb(weights)
        h = ctypes.c_void_p()
        self.ctx.check(lib().di_resnet_block_create(self.ctx.h, N, C, H, W, Tdim, seed, eps, int(temb_silu), self._cb,
                                                    None, ctypes.byref(h)), "di_resnet_block_create")
        self.h = h
        ps = [ctypes.c_void_p() for _ in range(3)]
        lib().di_resnet_block_io(self.h, *[ctypes.byref(p) for p in ps])
        self.x = view(ps[0].value, (N, C, H, W))
        self.temb = view(ps[1].value, (N, Tdim))
        self.y = view(ps[2].value, (N, C, H, W))
        self.shape = dict(B=N, C=C, G=32, H=H, W=W, K=3)

    def run(self):
        self.ctx.check(lib().di_resnet_block_run(self.h), "di_resnet_block_run")

    def __call__(self, x, temb):
        self.x.copy_(x)
        self.temb.copy_(temb)
        self.run()
        return self.y

    def __del__(self):
        if getattr(self, "h", None):
            lib().di_resnet_block_destroy(self.h)
            self.h = None


class TransformerBlock:
    """Config-2 SD2.1 transformer block; parameter names prefixed "block." (diffusers Transformer2DModel)."""

    def __init__(self, ctx: Context | None = None, B=2, S=1024, C=640, Sk=77, Cctx=1024, seed=1, weights=None):
        self.ctx = ctx or default_context()
        self._cb = _weight_cb(weights)
        h = ctypes.c_void_p()
        self.ctx.check(lib().di_transformer_block_create(self.ctx.h, B, S, C, Sk, Cctx, seed, self._cb, None,
                                                         ctypes.byref(h)), "di_transformer_block_create")
        self.h = h
        ps = [ctypes.c_void_p() for _ in range(3)]
        lib().di_transformer_block_io(self.h, *[ctypes.byref(p) for p in ps])
        self.hidden = view(ps[0].value, (B, S, C), "f16")
        self.context = view(ps[1].value, (B, Sk, Cctx), "f16")
        self.out = view(ps[2].value, (B, S, C), "f16")
        self.shape = dict(B=B, S=S, D=C, D_FFN=4 * C, H=C // 64, HEAD_DIM=64)

    def run(self):
        self.ctx.check(lib().di_transformer_block_run(self.h), "di_transformer_block_run")

    def __call__(self, hidden, context):
        self.hidden.copy_(hidden)
        self.context.copy_(context)
        self.run()
        return self.out

    def __del__(self):
        if getattr(self, "h", None):
            lib().di_transformer_block_destroy(self.h)
            self.h = None
