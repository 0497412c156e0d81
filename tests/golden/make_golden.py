"""Generates wgsl_ops_cases.npz: the 27 known-answer cases of the reference's kernel self-test.

Each case restates, in numpy float64 (JavaScript's number type) with results stored as float32 (the
test's Float32Array), the synthetic inputs and the CPU reference formulas of wgsl-ops-test.js:36-435,
together with that test's pass gate (max |got - ref| < tol).  The reference cannot run in this
environment (no JavaScript runtime, no WebGPU), so its own CPU formulas are the pin.

    python tests/golden/make_golden.py      # rewrites tests/golden/wgsl_ops_cases.npz
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent / "wgsl_ops_cases.npz"
f32 = np.float32


def erf_as(t):
    """Abramowitz-Stegun 7.1.26 as written in wgsl-ops-test.js:50-55 (double precision)."""
    s = np.sign(t)
    a = np.abs(t)
    u = 1 / (1 + 0.3275911 * a)
    y = 1 - (((((1.061405429 * u - 1.453152027) * u) + 1.421413741) * u - 0.284496736) * u + 0.254829592) * u * np.exp(-a * a)
    return s * y


def cases():
    out = {}

    def put(name, tol, **arrays):
        out[name] = (tol, arrays)

    # unary, wgsl-ops-test.js:38-76
    N = 1024
    X = ((np.arange(N) - N / 2) / (N / 4)).astype(f32)
    x = X.astype(np.float64)
    refs = {
        "Sigmoid": 1 / (1 + np.exp(-x)),
        "Sqrt": np.sqrt(np.maximum(x, 0)),
        "SiLU": x / (1 + np.exp(-x)),
        "GELU": x * 0.5 * (1 + erf_as(x * 0.70710678)),
        "Erf": erf_as(x),
        "Abs": np.abs(x),
        "Neg": -x,
    }
    for op, r in refs.items():
        put(f"unary {op}", 1e-4, X=X, ref=r.astype(f32))

    # binary, :78-101
    N = 512
    i = np.arange(N)
    A = ((i + 1) * 0.1).astype(f32)
    B = (np.sin(i * 0.1) + 1.5).astype(f32)
    a, b = A.astype(np.float64), B.astype(np.float64)
    for op, r in {"Add": a + b, "Sub": a - b, "Mul": a * b, "Div": a / b, "Max": np.maximum(a, b),
                  "Min": np.minimum(a, b)}.items():
        put(f"binary {op}", 1e-3, A=A, B=B, ref=r.astype(f32))

    # softmax, :103-125
    rows, inner = 4, 64
    X = (np.sin(np.arange(rows * inner) * 0.1) * 2).astype(f32)
    xr = X.astype(np.float64).reshape(rows, inner)
    e = np.exp(xr - xr.max(1, keepdims=True))
    put("softmax", 1e-4, X=X, cfg=np.array([inner, rows], np.uint32), ref=(e / e.sum(1, keepdims=True)).astype(f32).ravel())

    # instance norm, :127-158
    Nn, C, H, W = 2, 4, 8, 8
    HW = H * W
    X = (np.sin(np.arange(Nn * C * HW) * 0.07) * 3 + 1).astype(f32)
    g = np.full(C, 1.2, f32)
    bt = np.full(C, -0.3, f32)
    xr = X.astype(np.float64).reshape(Nn, C, HW)
    mean = xr.mean(2, keepdims=True)
    var = (xr * xr).sum(2, keepdims=True) / HW - mean * mean
    inv = 1 / np.sqrt(np.maximum(var, 0) + 1e-5)
    ref = (xr - mean) * inv * g.astype(np.float64)[None, :, None] + bt.astype(np.float64)[None, :, None]
    put("instancenorm", 1e-3, X=X, gamma=g, beta=bt, cfg=np.array([C, HW, Nn, 0], np.uint32), ref=ref.astype(f32).ravel())

    # matmul, :160-183
    M, Nc, K = 32, 48, 24
    A = np.sin(np.arange(M * K) * 0.3).astype(f32)
    B = np.cos(np.arange(K * Nc) * 0.17).astype(f32)
    ref = A.astype(np.float64).reshape(M, K) @ B.astype(np.float64).reshape(K, Nc)
    put("matmul 32x48x24", 1e-3, A=A, B=B, cfg=np.array([M, Nc, K, 0], np.uint32), batch=np.array([1]),
        ref=ref.astype(f32).ravel())

    # batched matmul, shared B and batched B, :185-233
    Bt, M, Nc, K = 2, 20, 24, 12
    A = np.sin(np.arange(Bt * M * K) * 0.21).astype(f32)
    Bs = np.cos(np.arange(K * Nc) * 0.13).astype(f32)
    ref = A.astype(np.float64).reshape(Bt, M, K) @ Bs.astype(np.float64).reshape(K, Nc)
    put("matmul batched sharedB", 1e-3, A=A, B=Bs, cfg=np.array([M, Nc, K, 0], np.uint32), batch=np.array([Bt]),
        ref=ref.astype(f32).ravel())
    Bb = np.cos(np.arange(Bt * K * Nc) * 0.13).astype(f32)
    ref = A.astype(np.float64).reshape(Bt, M, K) @ Bb.astype(np.float64).reshape(Bt, K, Nc)
    put("matmul batched batchedB", 1e-3, A=A, B=Bb, cfg=np.array([M, Nc, K, 1], np.uint32), batch=np.array([Bt]),
        ref=ref.astype(f32).ravel())

    # conv2d 3x3 and 1x1, :235-303
    def conv_ref(X, Wt, bias, Ci, Co, H, W, K):
        P = (K - 1) // 2
        x = np.pad(X.astype(np.float64).reshape(Ci, H, W), ((0, 0), (P, P), (P, P)))
        w = Wt.astype(np.float64).reshape(Co, Ci, K, K)
        y = np.zeros((Co, H, W)) + bias.astype(np.float64)[:, None, None]
        for ky in range(K):
            for kx in range(K):
                y += np.einsum("oc,chw->ohw", w[:, :, ky, kx], x[:, ky:ky + H, kx:kx + W])
        return y.astype(f32).ravel()

    Ci, Co, H, W = 3, 4, 8, 8
    X = np.sin(np.arange(Ci * H * W) * 0.2).astype(f32)
    Wt = (np.cos(np.arange(Co * Ci * 9) * 0.13) * 0.5).astype(f32)
    bias = (0.1 * np.arange(Co)).astype(f32)
    put("conv2d 3x3", 1e-3, X=X, W=Wt, bias=bias, cfg=np.array([Ci, Co, H, W], np.uint32), K=np.array([3]),
        ref=conv_ref(X, Wt, bias, Ci, Co, H, W, 3))
    Ci, Co, H, W = 8, 6, 4, 4
    X = np.sin(np.arange(Ci * H * W) * 0.1).astype(f32)
    Wt = (np.cos(np.arange(Co * Ci) * 0.2) * 0.3).astype(f32)
    bias = (0.05 * np.arange(Co)).astype(f32)
    put("conv2d 1x1", 1e-3, X=X, W=Wt, bias=bias, cfg=np.array([Ci, Co, H, W], np.uint32), K=np.array([1]),
        ref=conv_ref(X, Wt, bias, Ci, Co, H, W, 1))

    # layer norm, :305-336
    rows, inner = 8, 128
    X = (np.sin(np.arange(rows * inner) * 0.05) * 2 + 1).astype(f32)
    g = (0.9 + np.arange(inner) * 0.01).astype(f32)
    bt = (-0.1 + np.arange(inner) * 0.005).astype(f32)
    xr = X.astype(np.float64).reshape(rows, inner)
    mean = xr.mean(1, keepdims=True)
    var = (xr * xr).sum(1, keepdims=True) / inner - mean * mean
    ref = (xr - mean) / np.sqrt(np.maximum(var, 0) + 1e-5) * g.astype(np.float64) + bt.astype(np.float64)
    put("layernorm", 1e-3, X=X, gamma=g, beta=bt, cfg=np.array([inner, rows], np.uint32), ref=ref.astype(f32).ravel())

    # gemm transB=0 / 1, :338-388
    M, Nc, K = 16, 24, 12
    A = np.sin(np.arange(M * K) * 0.1).astype(f32)
    C = (0.01 * np.arange(Nc)).astype(f32)
    B = np.cos(np.arange(K * Nc) * 0.15).astype(f32)
    ref = A.astype(np.float64).reshape(M, K) @ B.astype(np.float64).reshape(K, Nc) + C.astype(np.float64)
    put("gemm transB=0", 1e-3, A=A, B=B, C=C, cfg=np.array([M, Nc, K, 0], np.uint32), ref=ref.astype(f32).ravel())
    ref = A.astype(np.float64).reshape(M, K) @ B.astype(np.float64).reshape(Nc, K).T + C.astype(np.float64)
    put("gemm transB=1", 1e-3, A=A, B=B, C=C, cfg=np.array([M, Nc, K, 1], np.uint32), ref=ref.astype(f32).ravel())

    # resize nearest 2x, :390-411
    C, Hi, Wi, Ho, Wo = 3, 4, 4, 8, 8
    X = np.sin(np.arange(C * Hi * Wi) * 0.3).astype(f32)
    oy = (np.arange(Ho) * Hi) // Ho
    ox = (np.arange(Wo) * Wi) // Wo
    ref = X.reshape(C, Hi, Wi)[:, oy][:, :, ox]
    put("resize nearest 2x", 1e-5, X=X, cfg=np.array([C, Hi, Wi, Ho, Wo, C * Ho * Wo, 0, 0], np.uint32),
        ref=ref.astype(f32).ravel())

    # powScalar, :413-432
    N = 256
    X = ((np.arange(N) - N / 2) / (N / 8)).astype(f32)
    x = X.astype(np.float64)
    for e in (2, 3, 0.5):
        with np.errstate(invalid="ignore"):
            r = np.where((x < 0) & (float(e) != int(e)), 0.0, np.power(x, e))
        put(f"powScalar e={e}", 1e-3, X=X, cfg=np.array([e, 0, 0, 0], f32), ref=r.astype(f32))
    return out


def main():
    flat = {}
    names = []
    for name, (tol, arrays) in cases().items():
        names.append(name)
        flat[f"{name}|tol"] = np.array([tol])
        for k, v in arrays.items():
            flat[f"{name}|{k}"] = np.asarray(v)
    flat["names"] = np.array(names)
    np.savez_compressed(OUT, **flat)
    print(f"{len(names)} cases -> {OUT}")


if __name__ == "__main__":
    main()
