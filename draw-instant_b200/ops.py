"""The wgsl-ops.js op families as closures over libdi (fp32 tensors in the reference's layouts).

Each factory mirrors one export of wgsl-ops.js: it takes the device (here a `Context`) and returns a
dispatch closure with the reference's exact parameter order, ``(encoder, *buffers, cfgBuf, *counts)``.
Buffers are flat CUDA tensors (torch, plumbing only); a uniform (`createUniform`) is a host array whose
values go to the kernel by value, as the executor's packed cfg blocks do (wgsl-executor.js OPS.*).

    enc = createCommandEncoder(ctx)
    unary(ctx, "SiLU")(enc, X, Y, n)
    submit(ctx, [enc]); got = readBack(ctx, Y, n * 4)

Launches are asynchronous on the context's stream (the analogue of recording into the command
encoder); `submit` + `readBack` synchronise.  There is no CPU fallback: every closure raises when
libdi.so is missing or a buffer is not a CUDA tensor.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import BINARY, UNARY, Context, DIError, lib, ptr

__all__ = ["unary", "binary", "binaryBcast", "affineBcast", "softmax", "instanceNorm", "groupNorm", "matmul",
           "convMM", "conv2d", "layerNorm", "gemm", "resizeNearest", "reduceMean", "transpose", "powScalar", "slice",
           "concatCopy", "createStorage", "createOutput", "createUniform", "readBack", "createCommandEncoder",
           "submit", "Uniform"]


class Uniform:
    """A cfg block (wgsl-ops.js createUniform): the raw bytes of a u32 / f32 array, padded to 16 bytes."""

    def __init__(self, arr):
        a = np.ascontiguousarray(arr)
        if a.dtype not in (np.uint32, np.float32, np.int32):
            raise DIError(f"uniform arrays are 32-bit, got {a.dtype}")
        raw = a.tobytes()
        self.raw = raw + b"\0" * (max(16, len(raw)) - len(raw))
        self._buf = ctypes.create_string_buffer(self.raw, len(self.raw))

    def u32(self, n: int):
        if 4 * n > len(self.raw):
            raise DIError(f"uniform holds {len(self.raw) // 4} words, the op reads {n}")
        return ctypes.cast(self._buf, ctypes.POINTER(ctypes.c_uint32))

    def f32(self, i: int) -> float:
        return float(np.frombuffer(self.raw, np.float32)[i])

    def ptr(self):
        return ctypes.cast(self._buf, ctypes.c_void_p)

    def destroy(self):
        pass


class Encoder:
    """Stands for GPUCommandEncoder: launches go straight to the context's stream."""

    def __init__(self, ctx: Context):
        self.ctx = ctx

    def finish(self):
        return self


def createCommandEncoder(ctx: Context) -> Encoder:
    return Encoder(ctx)


def submit(ctx: Context, encoders) -> None:
    """queue.submit + onSubmittedWorkDone: waits for the stream and surfaces device faults."""
    ctx.check(lib().di_wait(ctx.h), "submit")


def createStorage(ctx: Context, data):
    """Uploads a host array (fp32 / u32) into a new device buffer (a flat CUDA tensor)."""
    import torch
    a = np.ascontiguousarray(data)
    if a.dtype == np.float64:
        a = a.astype(np.float32)
    t = torch.from_numpy(a.view(np.float32).copy()).to(f"cuda:{ctx.device}")
    return t.view(-1)


def createOutput(ctx: Context, size_bytes: int):
    import torch
    return torch.empty((size_bytes + 3) // 4, dtype=torch.float32, device=f"cuda:{ctx.device}")


def createUniform(ctx: Context, arr) -> Uniform:
    return Uniform(arr)


def readBack(ctx: Context, buf, size_bytes: int) -> np.ndarray:
    submit(ctx, None)
    return buf.view(-1)[: size_bytes // 4].cpu().numpy().copy()


def _n(buf) -> int:
    return int(buf.numel())


def _run(ctx: Context, rc: int, what: str) -> None:
    ctx.check(rc, what)


def unary(ctx: Context, op: str):
    """wgsl-ops.js:110-122: Y[i] = f(X[i]) for i < N."""
    if op not in UNARY:
        raise DIError(f"unknown unary op: {op}")
    code = UNARY[op]

    def dispatch(encoder, X, Y, N):
        _run(ctx, lib().di_unary(ctx.h, code, ptr(X), ptr(Y), int(N)), f"unary {op}")
    return dispatch


def binary(ctx: Context, op: str):
    """wgsl-ops.js:250-262: Y[i] = A[i % len(A)] (op) B[i % len(B)]."""
    if op not in BINARY:
        raise DIError(f"unknown binary op: {op}")
    code = BINARY[op]

    def dispatch(encoder, A, B, Y, N):
        n = min(int(N), _n(Y))
        _run(ctx, lib().di_binary(ctx.h, code, ptr(A), _n(A), ptr(B), _n(B), ptr(Y), n), f"binary {op}")
    return dispatch


def binaryBcast(ctx: Context, op: str):
    """wgsl-ops.js:190-200: rank-4 broadcast with the cfg u32[20] {rank,_,_,_,outDim[4],aStride[4],bStride[4],numel,...}."""
    if op not in BINARY:
        raise DIError(f"unknown binary op: {op}")
    code = BINARY[op]

    def dispatch(encoder, A, B, Y, cfgBuf, numel):
        _run(ctx, lib().di_binary_bcast(ctx.h, code, ptr(A), ptr(B), ptr(Y), cfgBuf.u32(20)), f"binaryBcast {op}")
    return dispatch


def affineBcast(ctx: Context):
    """wgsl-ops.js:239-248: Y = A * GAMMA[bc] + BETA[bc] with the broadcast cfg u32[20]."""
    def dispatch(encoder, A, GAMMA, BETA, Y, cfgBuf, numel):
        _run(ctx, lib().di_affine_bcast(ctx.h, ptr(A), ptr(GAMMA), ptr(BETA), ptr(Y), cfgBuf.u32(20)), "affineBcast")
    return dispatch


def softmax(ctx: Context):
    """wgsl-ops.js:285-295: row softmax, cfg [innerLen, rows]."""
    def dispatch(encoder, X, Y, cfgBuf, rows):
        _run(ctx, lib().di_softmax(ctx.h, ptr(X), ptr(Y), cfgBuf.u32(2)), "softmax")
    return dispatch


def instanceNorm(ctx: Context):
    """wgsl-ops.js:374-385: per (n, c) normalisation over HW, cfg [C, HW, N, _], eps 1e-5."""
    def dispatch(encoder, X, gamma, beta, Y, cfgBuf, C, N):
        _run(ctx, lib().di_instance_norm(ctx.h, ptr(X), ptr(gamma), ptr(beta), ptr(Y), cfgBuf.u32(4)), "instanceNorm")
    return dispatch


def groupNorm(ctx: Context, fuse_silu: bool = False):
    """wgsl-ops.js:460-470: cfg {N, G, cpg, HW (u32), eps (f32)} (wgsl-executor.js:738-743);
    `fuse_silu` is the fuseSilu rewrite's GroupNorm+SiLU (fused-resnet.js:121-166)."""
    def dispatch(encoder, X, gamma, beta, Y, cfgBuf, G, N):
        _run(ctx, lib().di_group_norm(ctx.h, ptr(X), ptr(gamma), ptr(beta), ptr(Y), cfgBuf.ptr(), int(fuse_silu)),
             "groupNorm")
    return dispatch


def matmul(ctx: Context):
    """wgsl-ops.js:558-569: Y[z] = A[z] . B[z or 0], cfg [M, N, K, bBatched], batch on dispatch z."""
    def dispatch(encoder, A, B, Y, cfgBuf, M, N, batch=1):
        _run(ctx, lib().di_matmul(ctx.h, ptr(A), ptr(B), ptr(Y), cfgBuf.u32(4), int(batch)), "matmul")
    return dispatch


def convMM(ctx: Context):
    """wgsl-ops.js:700-711: NCHW conv, cfg u32[12] {C_in, C_out, K, K*K, H, W, PAD, S, H_out, W_out, 0, 0}
    (wgsl-executor.js:1088); batch 1 as the executor dispatches it."""
    def dispatch(encoder, X, Wt, bias, Y, cfgBuf, C_out, HW):
        _run(ctx, lib().di_conv(ctx.h, ptr(X), ptr(Wt), ptr(bias), ptr(Y), cfgBuf.u32(12), 1), "convMM")
    return dispatch


def conv2d(ctx: Context, K: int):
    """wgsl-ops.js:753-765: the direct 3x3 / 1x1 stride-1 'same' conv, cfg [C_in, C_out, H, W], PAD=(K-1)/2."""
    if K not in (1, 3):
        raise DIError(f"conv2d: only K=1 or K=3 supported, got {K}")

    def dispatch(encoder, X, Wt, bias, Y, cfgBuf, C_out, H, W):
        ci, co, h, w = (int(cfgBuf.u32(4)[i]) for i in range(4))
        cfg = (ctypes.c_uint32 * 12)(ci, co, K, K * K, h, w, (K - 1) // 2, 1, h, w, 0, 0)
        _run(ctx, lib().di_conv(ctx.h, ptr(X), ptr(Wt), ptr(bias), ptr(Y), cfg, 1), f"conv2d K={K}")
    return dispatch


def layerNorm(ctx: Context):
    """wgsl-ops.js:803-813: row LayerNorm over innerLen, cfg [innerLen, rows], eps 1e-5."""
    def dispatch(encoder, X, gamma, beta, Y, cfgBuf, rows):
        _run(ctx, lib().di_layer_norm(ctx.h, ptr(X), ptr(gamma), ptr(beta), ptr(Y), cfgBuf.u32(2)), "layerNorm")
    return dispatch


def gemm(ctx: Context):
    """wgsl-ops.js:899-910: Y = A . B(^T) + C[col], cfg [M, N, K, transB]."""
    def dispatch(encoder, A, B, C, Y, cfgBuf, M, N):
        _run(ctx, lib().di_gemm(ctx.h, ptr(A), ptr(B), ptr(C), ptr(Y), cfgBuf.u32(4)), "gemm")
    return dispatch


def resizeNearest(ctx: Context):
    """wgsl-ops.js:945-955: nearest resize, cfg [C, H_in, W_in, H_out, W_out, numel, _, _]."""
    def dispatch(encoder, X, Y, cfgBuf, numel):
        _run(ctx, lib().di_resize_nearest(ctx.h, ptr(X), ptr(Y), cfgBuf.u32(8)), "resizeNearest")
    return dispatch


def reduceMean(ctx: Context):
    """wgsl-ops.js:974-985: mean over the innermost axis, cfg [innerLen, rows]."""
    def dispatch(encoder, X, Y, cfgBuf, rows):
        _run(ctx, lib().di_reduce_mean(ctx.h, ptr(X), ptr(Y), cfgBuf.u32(2)), "reduceMean")
    return dispatch


def transpose(ctx: Context):
    """wgsl-ops.js:1035-1045: rank-4 permutation, cfg u32[20] as the broadcast block."""
    def dispatch(encoder, X, Y, cfgBuf, numel):
        _run(ctx, lib().di_transpose(ctx.h, ptr(X), ptr(Y), cfgBuf.u32(20)), "transpose")
    return dispatch


def powScalar(ctx: Context):
    """wgsl-ops.js:1074-1085: Y = X^e, cfg f32 [e, 0, 0, 0]; sign-aware for integer e, 0 for x<0 otherwise."""
    def dispatch(encoder, X, Y, cfgBuf, N):
        _run(ctx, lib().di_pow_scalar(ctx.h, ptr(X), ptr(Y), cfgBuf.f32(0), int(N)), "powScalar")
    return dispatch


def slice(ctx: Context):
    """wgsl-ops.js:1125-1135: strided rank-4 slice, cfg u32[20]."""
    def dispatch(encoder, X, Y, cfgBuf, numel):
        _run(ctx, lib().di_slice(ctx.h, ptr(X), ptr(Y), cfgBuf.u32(20)), "slice")
    return dispatch


def concatCopy(ctx: Context):
    """wgsl-ops.js:1159-1168: copy X into a slab of the concatenated Y, cfg u32[4]."""
    def dispatch(encoder, X, Y, cfgBuf, numel):
        _run(ctx, lib().di_concat_copy(ctx.h, ptr(X), ptr(Y), cfgBuf.u32(4)), "concatCopy")
    return dispatch
