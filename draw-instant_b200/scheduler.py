"""Euler Discrete scheduler for SD-Turbo: the host-side mirror of scheduler.js.

The reference keeps the scheduler on the host (pure JavaScript, no device work); this is the same
arithmetic in numpy with JavaScript's semantics made explicit, so timesteps, sigmas and the seeded noise
are bit-identical to what scheduler.js produces:
  * every intermediate is an IEEE double (JS number), rounded to float32 exactly where the reference
    stores into a Float32Array;
  * Math.round(x) = floor(x + 0.5);
  * the LCG is `s = (s * 1664525 + 1013904223) | 0` (32-bit wrap) and `(s >>> 0) / 2^32`.

    sch = make_euler_scheduler(4)        # timesteps [999, 749, 499, 249], sigmas[5] ending in 0
    x = sample_noise_latent(1, 64, 64, seed, sch.init_noise_sigma)
    for i in range(sch.num_inference):
        eps = unet(sch.scale_model_input(x, i), sch.timesteps[i], context)
        x = sch.step(x, eps, i)
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

NUM_TRAIN_TIMESTEPS = 1000  # scheduler.js:22-24
BETA_START = 0.00085
BETA_END = 0.012


def scaled_linear_betas(n: int = NUM_TRAIN_TIMESTEPS, start: float = BETA_START, end: float = BETA_END) -> np.ndarray:
    """scheduler.js:26-36: ((sqrt(start) + (sqrt(end) - sqrt(start)) * i/(n-1))^2, stored as float32."""
    t = np.arange(n, dtype=np.float64) / (n - 1)
    v = np.sqrt(start) + (np.sqrt(end) - np.sqrt(start)) * t
    return (v * v).astype(np.float32)


def cumulative_alphas(betas: np.ndarray) -> np.ndarray:
    """scheduler.js:38-46: running product in double, each partial product stored as float32."""
    out = np.empty(len(betas), np.float32)
    acc = 1.0
    for i, b in enumerate(betas.astype(np.float64)):
        acc *= 1.0 - b
        out[i] = acc
    return out


def sigmas_from_alphas(alphas: np.ndarray) -> np.ndarray:
    """scheduler.js:49-55: sqrt((1 - a) / a) in double, stored as float32."""
    a = alphas.astype(np.float64)
    return np.sqrt((1.0 - a) / a).astype(np.float32)


def js_round(x: float) -> float:
    """Math.round: nearest integer, halves toward +infinity."""
    return float(np.floor(x + 0.5))


def interp(sigmas: np.ndarray, t: float) -> float:
    """scheduler.js:58-64: linear interpolation at fractional timestep t (double)."""
    if t <= 0:
        return float(sigmas[0])
    if t >= len(sigmas) - 1:
        return float(sigmas[-1])
    i = int(np.floor(t))
    f = t - i
    return float(sigmas[i]) * (1 - f) + float(sigmas[i + 1]) * f


def trailing_timesteps(num_inference: int) -> np.ndarray:
    """scheduler.js:68-77: round(T - (i + 1) * step + step) - 1 with step = T / n, as float32."""
    step = NUM_TRAIN_TIMESTEPS / num_inference
    return np.array([js_round(NUM_TRAIN_TIMESTEPS - (i + 1) * step + step) - 1 for i in range(num_inference)],
                    np.float32)


@dataclass
class EulerScheduler:
    """The object makeEulerScheduler returns (scheduler.js:79-112)."""
    timesteps: np.ndarray
    sigmas: np.ndarray  # float32[num_inference + 1], last = 0
    num_inference: int
    init_noise_sigma: float

    def scale_model_input(self, latent: np.ndarray, i: int) -> np.ndarray:
        """latent / sqrt(sigma_i^2 + 1) (scheduler.js:95-101)."""
        s = float(self.sigmas[i])
        inv = 1.0 / np.sqrt(s * s + 1.0)
        return (np.asarray(latent, np.float32).astype(np.float64) * inv).astype(np.float32)

    def step(self, latent: np.ndarray, noise_pred: np.ndarray, i: int) -> np.ndarray:
        """Euler, epsilon prediction: latent + (sigma_{i+1} - sigma_i) * eps (scheduler.js:105-110)."""
        dt = float(self.sigmas[i + 1]) - float(self.sigmas[i])
        x = np.asarray(latent, np.float32).astype(np.float64)
        e = np.asarray(noise_pred, np.float32).astype(np.float64)
        return (x + dt * e).astype(np.float32)


def make_euler_scheduler(num_inference: int = 4) -> EulerScheduler:
    """scheduler.js:79-112."""
    betas = scaled_linear_betas()
    sig_full = sigmas_from_alphas(cumulative_alphas(betas))
    ts = trailing_timesteps(num_inference)
    sigmas = np.zeros(num_inference + 1, np.float32)
    for i in range(num_inference):
        sigmas[i] = interp(sig_full, float(ts[i]))
    return EulerScheduler(ts, sigmas, num_inference, float(sigmas[0]))


def sample_noise_latent(B: int = 1, H: int = 64, W: int = 64, seed: int = 0, init_sigma: float = 1.0) -> np.ndarray:
    """scheduler.js:117-134: seeded 32-bit LCG + Box-Muller, [B, 4, H, W] float32 scaled by init_sigma."""
    n = B * 4 * H * W
    out = np.empty(n, np.float32)
    s = (int(seed) & 0xFFFFFFFF) or 1  # (seed | 0) || 1; the LCG below works on the unsigned bits

    def rand() -> float:
        nonlocal s
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        return s / 4294967296.0

    two_pi = 2 * np.pi
    for i in range(0, n, 2):
        u1 = max(rand(), 1e-9)
        u2 = rand()
        r = np.sqrt(-2 * np.log(u1))
        out[i] = r * np.cos(two_pi * u2) * init_sigma
        if i + 1 < n:
            out[i + 1] = r * np.sin(two_pi * u2) * init_sigma
    return out.reshape(B, 4, H, W)


# reference spellings
makeEulerScheduler = make_euler_scheduler
sampleNoiseLatent = sample_noise_latent
