"""The host scheduler mirror (draw-instant_b200/scheduler.py) against the pins of scheduler.js and the
oracle's independent C restatement: bit-exact timesteps, sigmas, noise, input scaling and Euler steps."""
from __future__ import annotations

import importlib

import numpy as np
import pytest

from conftest import load_package


@pytest.fixture(scope="module")
def sch():
    load_package()
    return importlib.import_module("draw_instant_b200.scheduler")


def test_timesteps_pinned(sch):
    assert sch.make_euler_scheduler(4).timesteps.tolist() == [999, 749, 499, 249]  # scheduler.js:4
    assert sch.make_euler_scheduler(1).timesteps.tolist() == [999]


@pytest.mark.parametrize("n", [1, 2, 3, 4, 8, 50])
def test_matches_oracle_bit_exact(sch, oracle, n):
    s = sch.make_euler_scheduler(n)
    np.testing.assert_array_equal(s.timesteps, oracle.sched_timesteps(n))
    np.testing.assert_array_equal(s.sigmas, oracle.sched_sigmas(n))
    assert s.sigmas[-1] == 0 and np.all(np.diff(s.sigmas) < 0)
    assert s.init_noise_sigma == float(s.sigmas[0])


@pytest.mark.parametrize("seed", [0, 1, 42, 2**31 - 1])
def test_noise_bit_exact(sch, oracle, seed):
    sigma = float(np.float32(14.6146))  # a float32 value, as init_noise_sigma always is
    a = sch.sample_noise_latent(1, 8, 8, seed, sigma)
    b = oracle.noise_latent(1, 8, 8, seed, sigma)
    np.testing.assert_array_equal(a, b)


def test_scale_and_step_bit_exact(sch, oracle):
    s = sch.make_euler_scheduler(4)
    rng = np.random.default_rng(0)
    x = rng.standard_normal(512).astype(np.float32) * 10
    e = rng.standard_normal(512).astype(np.float32)
    for i in range(4):
        y = np.empty_like(x)
        oracle.lib().o_sched_scale_input(x, y, x.size, float(s.sigmas[i]))
        np.testing.assert_array_equal(s.scale_model_input(x, i), y)
        z = np.empty_like(x)
        oracle.lib().o_sched_step(x, e, z, x.size, float(s.sigmas[i]), float(s.sigmas[i + 1]))
        np.testing.assert_array_equal(s.step(x, e, i), z)


@pytest.mark.parametrize("n", [1, 2, 4, 7, 50])
def test_libdi_euler_sigmas_match_host_scheduler(dib, oracle, n):
    """The C++ schedule the text-to-image pipeline bakes into the U-Net plan (host-only entry point,
    no GPU) equals the Python mirror and the oracle bit for bit."""
    import ctypes
    sig = np.empty(n + 1, np.float32)
    ts = np.empty(n, np.float32)
    assert dib.lib().di_euler_sigmas(n, sig.ctypes.data_as(ctypes.c_void_p), ts.ctypes.data_as(ctypes.c_void_p)) == 0
    sched = importlib.import_module("draw_instant_b200.scheduler")
    s = sched.make_euler_scheduler(n)
    assert np.array_equal(sig, s.sigmas) and np.array_equal(ts, s.timesteps)
    assert np.array_equal(sig, oracle.sched_sigmas(n)) and np.array_equal(ts, oracle.sched_timesteps(n))
