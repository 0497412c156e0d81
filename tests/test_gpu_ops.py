"""The wgsl-ops.js op families on the GPU, through the closure mirror (draw-instant_b200/ops.py) and the C ABI.

1. The reference's own 27 self-test cases (wgsl-ops-test.js:36-435) with its gates, from the committed
   golden fixture.
2. The families that self-test does not cover (broadcast, affine, transpose, slice, concat, reduceMean,
   the fp32 GroupNorm with and without SiLU, convMM with stride 2 and batch) against the CPU oracle on
   seeded inputs, plus sizes that exercise the tensor-core tiling (ragged M/N/K, several tiles).
3. Edge cases: zero-length launches, unknown ops, malformed cfg blocks."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import golden_cases, load_package

pytestmark = pytest.mark.gpu
CASES = golden_cases()


@pytest.fixture(scope="module")
def ops(dib):
    import importlib
    return importlib.import_module("draw_instant_b200.ops")


def run_case(O, ctx, name, a):
    enc = O.createCommandEncoder(ctx)
    S = lambda k: O.createStorage(ctx, a[k])
    kind = name.split()[0]
    n_out = a["ref"].size
    Y = O.createOutput(ctx, 4 * n_out)
    if kind == "unary":
        O.unary(ctx, name.split()[1])(enc, S("X"), Y, n_out)
    elif kind == "binary":
        O.binary(ctx, name.split()[1])(enc, S("A"), S("B"), Y, n_out)
    elif kind == "softmax":
        O.softmax(ctx)(enc, S("X"), Y, O.createUniform(ctx, a["cfg"]), int(a["cfg"][1]))
    elif kind == "instancenorm":
        O.instanceNorm(ctx)(enc, S("X"), S("gamma"), S("beta"), Y, O.createUniform(ctx, a["cfg"]),
                            int(a["cfg"][0]), int(a["cfg"][2]))
    elif kind == "matmul":
        M, N = int(a["cfg"][0]), int(a["cfg"][1])
        O.matmul(ctx)(enc, S("A"), S("B"), Y, O.createUniform(ctx, a["cfg"]), M, N, int(a["batch"][0]))
    elif kind == "conv2d":
        Ci, Co, H, W = (int(v) for v in a["cfg"])
        O.conv2d(ctx, int(a["K"][0]))(enc, S("X"), S("W"), S("bias"), Y, O.createUniform(ctx, a["cfg"]), Co, H, W)
    elif kind == "layernorm":
        O.layerNorm(ctx)(enc, S("X"), S("gamma"), S("beta"), Y, O.createUniform(ctx, a["cfg"]), int(a["cfg"][1]))
    elif kind == "gemm":
        O.gemm(ctx)(enc, S("A"), S("B"), S("C"), Y, O.createUniform(ctx, a["cfg"]), int(a["cfg"][0]), int(a["cfg"][1]))
    elif kind == "resize":
        O.resizeNearest(ctx)(enc, S("X"), Y, O.createUniform(ctx, a["cfg"]), n_out)
    elif kind == "powScalar":
        O.powScalar(ctx)(enc, S("X"), Y, O.createUniform(ctx, a["cfg"]), n_out)
    else:
        raise AssertionError(name)
    O.submit(ctx, [enc.finish()])
    return O.readBack(ctx, Y, 4 * n_out)


@pytest.mark.parametrize("name,tol,arrays", CASES, ids=[c[0] for c in CASES])
def test_reference_selftest_case(ctx, ops, name, tol, arrays):
    got = run_case(ops, ctx, name, arrays).astype(np.float64)
    ref = arrays["ref"].astype(np.float64)
    d = np.max(np.abs(got - ref))
    assert d < tol, f"{name}: maxAbsDiff {d:.3e} >= {tol}"


# ---- families beyond the self-test, against the oracle ----
def bcast_cfg(out_shape, strides_a, strides_b):
    r = len(out_shape)
    pad = lambda v: list(v) + [0] * (4 - len(v))
    return np.array([r, 0, 0, 0] + pad(out_shape) + pad(strides_a) + pad(strides_b) + [int(np.prod(out_shape)), 0, 0, 0],
                    np.uint32)


def strides_of(shape, full):
    """Row-major strides of `shape` broadcast against `full` (0 where the dim is 1 and full is not)."""
    st, acc = [], 1
    for d in reversed(shape):
        st.append(acc)
        acc *= d
    st = st[::-1]
    return [0 if s == 1 and f != 1 else t for s, f, t in zip(shape, full, st)]


@pytest.mark.parametrize("op,code", [("Add", 0), ("Sub", 1), ("Mul", 2), ("Div", 3), ("Pow", 4), ("Max", 5), ("Min", 6)])
def test_binary_bcast(ctx, ops, oracle, op, code):
    rng = np.random.default_rng(code)
    full = (2, 5, 7, 33)
    sa, sb = (2, 1, 7, 33), (1, 5, 1, 33)
    A = rng.standard_normal(np.prod(sa)).astype(np.float32)
    B = (rng.random(np.prod(sb)) + 0.5).astype(np.float32)
    if op == "Pow":
        B = np.round(B * 3).astype(np.float32)
    cfg = bcast_cfg(full, strides_of(sa, full), strides_of(sb, full))
    enc = ops.createCommandEncoder(ctx)
    Y = ops.createOutput(ctx, 4 * int(np.prod(full)))
    ops.binaryBcast(ctx, op)(enc, ops.createStorage(ctx, A), ops.createStorage(ctx, B), Y,
                             ops.createUniform(ctx, cfg), int(np.prod(full)))
    got = ops.readBack(ctx, Y, 4 * int(np.prod(full)))
    ref = oracle.binary_bcast(code, A, B, cfg)
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-5)


def test_affine_bcast(ctx, ops, oracle):
    rng = np.random.default_rng(7)
    full = (1, 320, 16, 16)
    sg = (1, 320, 1, 1)
    A = rng.standard_normal(np.prod(full)).astype(np.float32)
    G = rng.standard_normal(320).astype(np.float32)
    Bt = rng.standard_normal(320).astype(np.float32)
    cfg = bcast_cfg(full, strides_of(full, full), strides_of(sg, full))
    enc = ops.createCommandEncoder(ctx)
    Y = ops.createOutput(ctx, 4 * A.size)
    ops.affineBcast(ctx)(enc, *(ops.createStorage(ctx, v) for v in (A, G, Bt)), Y, ops.createUniform(ctx, cfg), A.size)
    got = ops.readBack(ctx, Y, 4 * A.size)
    np.testing.assert_allclose(got, oracle.affine_bcast(A, G, Bt, cfg), rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("shape,perm", [((2, 3, 4, 5), (0, 2, 1, 3)), ((2, 10, 64, 77), (0, 1, 3, 2)), ((6, 7), (1, 0)),
                                        ((3, 4, 5), (2, 0, 1))])
def test_transpose(ctx, ops, oracle, shape, perm):
    X = np.arange(np.prod(shape), dtype=np.float32)
    out_shape = [shape[p] for p in perm]
    st = strides_of(shape, shape)
    pad = lambda v: list(v) + [0] * (4 - len(v))
    cfg = np.array([len(shape), 0, 0, 0] + pad(out_shape) + pad(st) + pad(perm) + [X.size, 0, 0, 0], np.uint32)
    enc = ops.createCommandEncoder(ctx)
    Y = ops.createOutput(ctx, 4 * X.size)
    ops.transpose(ctx)(enc, ops.createStorage(ctx, X), Y, ops.createUniform(ctx, cfg), X.size)
    got = ops.readBack(ctx, Y, 4 * X.size)
    np.testing.assert_array_equal(got, oracle.transpose(X, cfg))
    np.testing.assert_array_equal(got, np.transpose(X.reshape(shape), perm).ravel())  # index work: bit-exact


def test_slice(ctx, ops, oracle):
    shape = (2, 1280, 8, 8)
    X = np.arange(np.prod(shape), dtype=np.float32)
    start, out_shape = (0, 640, 0, 0), (2, 640, 8, 8)
    pad = lambda v: list(v) + [0] * (4 - len(v))
    n = int(np.prod(out_shape))
    cfg = np.array([4, 0, 0, 0] + pad(out_shape) + pad(strides_of(shape, shape)) + pad(start) + [n, 0, 0, 0], np.uint32)
    enc = ops.createCommandEncoder(ctx)
    Y = ops.createOutput(ctx, 4 * n)
    ops.slice(ctx)(enc, ops.createStorage(ctx, X), Y, ops.createUniform(ctx, cfg), n)
    got = ops.readBack(ctx, Y, 4 * n)
    np.testing.assert_array_equal(got, oracle.slice_(X, cfg))
    np.testing.assert_array_equal(got, X.reshape(shape)[:, 640:].ravel())


def test_concat_copy(ctx, ops, oracle):
    a = np.arange(2 * 3 * 5, dtype=np.float32).reshape(2, 3 * 5)
    b = -np.arange(2 * 4 * 5, dtype=np.float32).reshape(2, 4 * 5) - 1
    Y = ops.createOutput(ctx, 4 * 2 * 7 * 5)
    enc = ops.createCommandEncoder(ctx)
    for x, off in ((a, 0), (b, 15)):
        cfg = np.array([x.shape[1], 35, off, x.size], np.uint32)
        ops.concatCopy(ctx)(enc, ops.createStorage(ctx, x), Y, ops.createUniform(ctx, cfg), x.size)
    got = ops.readBack(ctx, Y, 4 * 70)
    np.testing.assert_array_equal(got, np.concatenate([a, b], 1).ravel())


@pytest.mark.parametrize("inner,rows", [(1, 5), (77, 3), (4096, 20), (1000, 1)])
def test_reduce_mean(ctx, ops, oracle, inner, rows):
    X = np.random.default_rng(inner).standard_normal(inner * rows).astype(np.float32)
    enc = ops.createCommandEncoder(ctx)
    Y = ops.createOutput(ctx, 4 * rows)
    ops.reduceMean(ctx)(enc, ops.createStorage(ctx, X), Y, ops.createUniform(ctx, np.array([inner, rows], np.uint32)), rows)
    got = ops.readBack(ctx, Y, 4 * rows)
    np.testing.assert_allclose(got, oracle.reduce_mean(X, inner, rows), rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("N,C,HW,G,silu", [(1, 320, 64 * 64, 32, False), (2, 640, 16 * 16, 32, True), (1, 4, 9, 2, True)])
def test_group_norm_fp32(ctx, ops, oracle, N, C, HW, G, silu):
    rng = np.random.default_rng(C + HW)
    X = (rng.standard_normal(N * C * HW) * 2 + 0.5).astype(np.float32)
    g = (1 + 0.02 * rng.standard_normal(C)).astype(np.float32)
    b = (0.02 * rng.standard_normal(C)).astype(np.float32)
    cfg = np.zeros(8, np.uint32)
    cfg[:4] = (N, G, C // G, HW)
    cfg[4] = np.array([1e-5], np.float32).view(np.uint32)[0]
    enc = ops.createCommandEncoder(ctx)
    Y = ops.createOutput(ctx, 4 * X.size)
    ops.groupNorm(ctx, silu)(enc, *(ops.createStorage(ctx, v) for v in (X, g, b)), Y, ops.createUniform(ctx, cfg), G, N)
    got = ops.readBack(ctx, Y, 4 * X.size)
    ref = oracle.group_norm(X, g, b, N, C, HW, G, 1e-5, silu=silu)
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("Ci,Co,H,W,K,S,PAD", [(320, 320, 32, 32, 3, 2, 1), (4, 320, 16, 16, 3, 1, 1),
                                               (320, 4, 16, 16, 3, 1, 1), (640, 1280, 8, 8, 1, 1, 0),
                                               (5, 7, 9, 11, 3, 2, 1)])
def test_convmm_vs_oracle(ctx, ops, oracle, Ci, Co, H, W, K, S, PAD):
    rng = np.random.default_rng(Ci * Co)
    X = rng.standard_normal(Ci * H * W).astype(np.float32)
    Wt = (rng.standard_normal(Co * Ci * K * K) / np.sqrt(Ci * K * K)).astype(np.float32)
    b = rng.standard_normal(Co).astype(np.float32)
    Ho, Wo = (H + 2 * PAD - K) // S + 1, (W + 2 * PAD - K) // S + 1
    cfg = np.array([Ci, Co, K, K * K, H, W, PAD, S, Ho, Wo, 0, 0], np.uint32)
    enc = ops.createCommandEncoder(ctx)
    Y = ops.createOutput(ctx, 4 * Co * Ho * Wo)
    ops.convMM(ctx)(enc, *(ops.createStorage(ctx, v) for v in (X, Wt, b)), Y, ops.createUniform(ctx, cfg), Co, Ho * Wo)
    got = ops.readBack(ctx, Y, 4 * Co * Ho * Wo)
    ref = oracle.conv(X, Wt, b, 1, Ci, H, W, Co, K, S, PAD).ravel()
    assert np.max(np.abs(got - ref)) < 1e-3 * max(1.0, np.max(np.abs(ref)))


@pytest.mark.parametrize("M,N,K,bb,batch", [(300, 200, 500, 0, 1), (4096, 320, 320, 0, 1), (77, 1024, 64, 1, 3),
                                            (1, 1, 1, 0, 1), (129, 257, 65, 0, 2)])
def test_matmul_fp32_accuracy(ctx, ops, oracle, M, N, K, bb, batch):
    """The bf16x3 split keeps the fp32 op family at fp32-level error (well under the 1e-3 gates)."""
    rng = np.random.default_rng(M + N + K)
    A = rng.standard_normal(batch * M * K).astype(np.float32)
    B = rng.standard_normal((batch if bb else 1) * K * N).astype(np.float32)
    cfg = np.array([M, N, K, bb], np.uint32)
    enc = ops.createCommandEncoder(ctx)
    Y = ops.createOutput(ctx, 4 * batch * M * N)
    ops.matmul(ctx)(enc, ops.createStorage(ctx, A), ops.createStorage(ctx, B), Y, ops.createUniform(ctx, cfg), M, N, batch)
    got = ops.readBack(ctx, Y, 4 * batch * M * N).astype(np.float64)
    Bm = B.astype(np.float64).reshape((batch if bb else 1), K, N)
    ref = np.matmul(A.astype(np.float64).reshape(batch, M, K), Bm).ravel()
    assert np.max(np.abs(got - ref)) / np.sqrt(K) < 3e-4


def test_zero_length_and_bad_ops(ctx, ops, dib):
    enc = ops.createCommandEncoder(ctx)
    X = ops.createStorage(ctx, np.zeros(4, np.float32))
    Y = ops.createOutput(ctx, 16)
    ops.unary(ctx, "SiLU")(enc, X, Y, 0)  # empty launch is a no-op
    with pytest.raises(dib.DIError):
        ops.unary(ctx, "Tanh")
    with pytest.raises(dib.DIError):  # cfg K*K inconsistent with K
        bad = np.array([1, 1, 3, 8, 4, 4, 1, 1, 4, 4, 0, 0], np.uint32)
        ops.convMM(ctx)(enc, X, X, X, Y, ops.createUniform(ctx, bad), 1, 16)
    with pytest.raises(dib.DIError):  # rank 5 broadcast
        ops.binaryBcast(ctx, "Add")(enc, X, X, Y, ops.createUniform(ctx, np.array([5] + [0] * 19, np.uint32)), 4)
    ctx.clear_fault()


def test_f16_bytes_to_f32_all_patterns(ctx, dib, oracle):
    """WeightCache conversion (wgsl-unet.js:23-47) on the device: all 65536 fp16 bit patterns, bit-exact."""
    import torch
    h = np.arange(65536, dtype=np.uint16)
    src = torch.from_numpy(h.view(np.int16).copy()).cuda()
    dst = torch.empty(65536, dtype=torch.float32, device="cuda")
    ctx.check(dib.lib().di_f16_bytes_to_f32(ctx.h, src.data_ptr(), dst.data_ptr(), 65536), "f16_bytes_to_f32")
    got = dst.cpu().numpy().view(np.uint32)
    ref = oracle.f16_to_f32(h).view(np.uint32)
    np.testing.assert_array_equal(got, ref)
    # Inf / NaN patterns keep their payload in the fp32 mantissa: sign | 0x7f800000 | mant << 13
    sp = h[(h >> 10 & 0x1F) == 31].astype(np.uint32)
    np.testing.assert_array_equal(got[sp], ((sp & 0x8000) << 16) | 0x7F800000 | ((sp & 0x3FF) << 13))
