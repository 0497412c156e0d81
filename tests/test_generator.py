"""The seeded parameter generator exists twice: in the product (libdi's host code, di_synth_*) and in the
CPU oracle.  Both are restatements of the same documented scheme; every parity test relies on them
producing identical weights, so they must agree bit for bit.  CPU only (host functions)."""
from __future__ import annotations

import numpy as np
import pytest


@pytest.mark.parametrize("seed,name,n,bound", [(0, "conv1.weight", 320 * 320 * 9, 0.0186),
                                              (3, "down_blocks.0.resnets.0.conv1.bias", 320, 1 / 53.6),
                                              (1, "block.proj_in.weight", 640 * 640, 0.068), (7, "x", 1, 1.0)])
def test_uniform_bit_exact(dib, oracle, seed, name, n, bound):
    got = np.empty(n, np.float32)
    dib.lib().di_synth_uniform(seed, name.encode(), n, bound, got.ctypes.data)
    ref = oracle.gen_uniform(seed, name, n, bound)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("seed,name,n,mean,std", [(0, "norm1.weight", 320, 1.0, 0.02), (3, "latent", 16384, 0.0, 1.0),
                                                 (1, "block.norm.bias", 641, 0.0, 0.02)])
def test_normal_bit_exact(dib, oracle, seed, name, n, mean, std):
    got = np.empty(n, np.float32)
    dib.lib().di_synth_normal(seed, name.encode(), n, mean, std, got.ctypes.data)
    ref = oracle.gen_normal(seed, name, n, mean, std)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
