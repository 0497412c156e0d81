"""OpenCLIP ViT-H text encoder plan (SD2.x / SD-Turbo conditioning): the libdi replacement of the ONNX
Runtime session that text-encoder.js:69-174 creates (loadSDTextEncoder / encodeSDPrompt).

    te = TextEncoder(ctx, B=1, layers=24, seed=4)
    emb = te.forward_host(ids)              # int32 [B, 77] -> [B, 77, 1024] fp32 (last_hidden_state)

Tokenisation stays on the host (the reference reuses transformers.js' CLIP tokenizer); `sd_pad_ids`
applies the SD-Turbo pad rule that encodeSDPrompt applies to the tokenizer output.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import Context, default_context, lib, view
from .blocks import _weight_cb

VOCAB, WIDTH, HEADS, MLP, CONTEXT = 49408, 1024, 16, 4096, 77
EOS = 49407


def sd_pad_ids(ids) -> np.ndarray:
    """text-encoder.js:136-141: keep the first end-of-text id (49407) and rewrite everything after it to 0
    (the OpenCLIP-H pad id).  Works row-wise on [B, 77] or on one row."""
    a = np.array(ids, dtype=np.int32, copy=True)
    for r in a.reshape(-1, a.shape[-1]):
        hit = np.nonzero(r == EOS)[0]
        if hit.size:
            r[hit[0] + 1:] = 0
    return a


def text_flops(B: int, S: int = CONTEXT, layers: int = 24) -> float:
    """Algorithmic FLOPs of one forward: per token q/k/v/out (4 D^2) and MLP (2 D F) products per layer,
    plus the causal QK^T and PV products (query i sees i + 1 keys)."""
    per_tok = 2.0 * (4 * WIDTH * WIDTH + 2 * WIDTH * MLP)
    attn = 2.0 * HEADS * S * (S + 1) * 64
    return B * layers * (S * per_tok + attn)


class TextEncoder:
    """Parameter names are HF CLIPTextModel's ("text_model.embeddings.token_embedding.weight",
    "text_model.encoder.layers.0.self_attn.q_proj.weight", ...); `weights(name, n)` may supply any of them."""

    def __init__(self, ctx: Context | None = None, B=1, S=CONTEXT, layers=24, seed=4, weights=None):
        self.ctx = ctx or default_context()
        self._cb = _weight_cb(weights)
        hh = ctypes.c_void_p()
        self.ctx.check(lib().di_text_create(self.ctx.h, B, S, layers, seed, self._cb, None, ctypes.byref(hh)),
                       "di_text_create")
        self.h = hh
        self.B, self.S, self.layers = B, S, layers
        pi, ph = ctypes.c_void_p(), ctypes.c_void_p()
        lib().di_text_io(self.h, ctypes.byref(pi), ctypes.byref(ph))
        self.ids = view(pi.value, (B, S), "i32")
        self.hidden = view(ph.value, (B, S, WIDTH))
        n = ctypes.c_int()
        wb, ab = ctypes.c_size_t(), ctypes.c_size_t()
        lib().di_text_info(self.h, ctypes.byref(n), ctypes.byref(wb), ctypes.byref(ab))
        self.launches, self.weight_bytes, self.act_bytes = n.value, wb.value, ab.value

    def forward(self):
        self.ctx.check(lib().di_text_forward(self.h), "di_text_forward")

    def forward_host(self, ids) -> np.ndarray:
        a = np.ascontiguousarray(ids, np.int32).reshape(self.B, self.S)
        out = np.empty((self.B, self.S, WIDTH), np.float32)
        self.ctx.check(lib().di_text_forward_host(self.h, a.ctypes.data_as(ctypes.c_void_p),
                                                  out.ctypes.data_as(ctypes.c_void_p)), "di_text_forward_host")
        return out

    def encode_ids(self, ids) -> dict:
        """encodeSDPrompt's tail (text-encoder.js:136-148) once the prompt is tokenised."""
        emb = self.forward_host(sd_pad_ids(ids))
        return {"embedding": emb, "shape": [self.B, self.S, WIDTH], "tokens": self.S}

    def close(self):
        if getattr(self, "h", None):
            lib().di_text_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
