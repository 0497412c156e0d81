"""Pins of the CPU oracle against what the reference itself fixes: scheduler timesteps, the f16->f32
bit conversion, the Abramowitz-Stegun erf bound, the LCG noise recurrence, and the generator's
determinism.  CPU only."""
from __future__ import annotations

import math

import numpy as np


def test_timesteps_pinned(oracle):
    # scheduler.js:4-5: "[999, 749, 499, 249] for a 4-step schedule"; n=1 -> [999] (scheduler.js:69-77)
    assert oracle.sched_timesteps(4).tolist() == [999, 749, 499, 249]
    assert oracle.sched_timesteps(1).tolist() == [999]
    assert oracle.sched_timesteps(2).tolist() == [999, 499]


def test_sigmas_shape_and_monotone(oracle):
    s = oracle.sched_sigmas(4)
    assert s.shape == (5,) and s[-1] == 0.0
    assert np.all(np.diff(s[:-1]) < 0)
    # diffusers' published scaled_linear schedule: sigma(999) ~= 14.6146
    assert abs(float(s[0]) - 14.6146) < 2e-3


def test_f16_to_f32_bit_exact(oracle):
    # every one of the 65536 half patterns, against numpy's independent IEEE conversion (wgsl-unet.js:23-47)
    h = np.arange(65536, dtype=np.uint16)
    got = oracle.f16_to_f32(h)
    ref = h.view(np.float16).astype(np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(got[~nan].view(np.uint32), ref[~nan].view(np.uint32))
    assert np.all(np.isnan(got[nan]))


def test_f32_to_f16_round_to_nearest_even(oracle):
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(200000).astype(np.float32) * 10.0 ** rng.integers(-9, 5, 200000),
                        np.array([65504, 65519.99, 65520, 1e-8, 2 ** -25, 2 ** -24, 3 * 2 ** -26], np.float32)])
    x = x.astype(np.float32)
    assert np.array_equal(oracle.f32_to_f16(x), x.astype(np.float16).view(np.uint16))


def test_erf_approximation_bound(oracle):
    x = np.linspace(-4, 4, 4001, dtype=np.float32)
    got = oracle.unary(10, x)
    ref = np.array([math.erf(float(v)) for v in x])
    assert np.max(np.abs(got - ref)) < 1e-6  # A&S 7.1.26: 1.5e-7 plus fp32 rounding


def test_noise_lcg_recurrence(oracle):
    # scheduler.js:121-133 with seed 1: first state = 1*1664525 + 1013904223 (int32 wrap)
    z = oracle.noise_latent(1, 2, 2, 1, 1.0).ravel()
    s1 = (1 * 1664525 + 1013904223) & 0xFFFFFFFF
    s2 = (s1 * 1664525 + 1013904223) & 0xFFFFFFFF
    u1, u2 = max(s1 / 2 ** 32, 1e-9), s2 / 2 ** 32
    r = math.sqrt(-2 * math.log(u1))
    assert abs(z[0] - r * math.cos(2 * math.pi * u2)) < 1e-6
    assert abs(z[1] - r * math.sin(2 * math.pi * u2)) < 1e-6


def test_generator_deterministic_and_scaled(oracle):
    a = oracle.gen_uniform(7, "w", 100000, 0.5)
    b = oracle.gen_uniform(7, "w", 100000, 0.5)
    c = oracle.gen_uniform(7, "w2", 100000, 0.5)
    assert np.array_equal(a, b) and not np.array_equal(a, c)
    assert a.min() >= -0.5 and a.max() < 0.5 and abs(a.mean()) < 5e-3
    n = oracle.gen_normal(3, "n", 200000, 1.0, 0.02)
    assert abs(n.mean() - 1.0) < 1e-3 and abs(n.std() - 0.02) < 1e-3
