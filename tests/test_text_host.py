"""Host side of the text encoder (pad rule, FLOP count) and the oracle's causal attention against a
NumPy statement of the same formula.  No GPU."""
from __future__ import annotations

import importlib

import numpy as np


def test_sd_pad_ids(dib):
    te = importlib.import_module("draw_instant_b200.text_encoder")
    row = np.full(77, te.EOS, np.int32)
    row[:3] = [49406, 320, 1125]
    out = te.sd_pad_ids(row)
    assert list(out[:4]) == [49406, 320, 1125, te.EOS] and np.all(out[4:] == 0)
    batch = np.stack([row, np.arange(77, dtype=np.int32)])
    out = te.sd_pad_ids(batch)
    assert np.all(out[1] == np.arange(77)) and np.all(out[0, 4:] == 0)


def test_text_flops_per_batch_of_64(dib):
    te = importlib.import_module("draw_instant_b200.text_encoder")
    # about 3.0 TFLOP per batch of 64 prompts (24 layers, width 1024, MLP 4096)
    assert abs(te.text_flops(64) / 1e12 - 2.98) < 0.05


def test_oracle_causal_attention_numpy(oracle):
    rng = np.random.default_rng(3)
    B, S, H = 2, 9, 3
    q, k, v = (rng.standard_normal((B, S, H, 64)).astype(np.float32) for _ in range(3))
    s = np.einsum("bihd,bjhd->bhij", q, k) / 8.0
    s = np.where(np.tril(np.ones((S, S), bool)), s, -np.inf)
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    ref = np.einsum("bhij,bjhd->bihd", p, v)
    assert np.abs(oracle.attention_causal(q, k, v) - ref).max() < 1e-4
