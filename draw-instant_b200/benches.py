"""The reference's fusion benchmarks (runXBench, fused-*.js) on libdi, with its timing method.

Each ``runXBench(onProgress)`` keeps the reference's name, argument and result schema:
``{shape, naive, fused, speedup, tflopsNaive?, tflopsFused?, bytesSaved?, correctness: {maxAbsDiff, l2},
dispatchesNaive, dispatchesFused, naiveRuns, fusedRuns}`` (milliseconds per iteration, medians), plus
what this build adds: ``kernelsNaive`` / ``kernelsFused`` (device kernels per iteration) and the dtypes.

  naive  the reference's unfused op sequence, one wgsl-ops family call per op, fp32 NCHW (the executor's
         path through libdi's op entry points, ops.py)
  fused  the fused block as the U-Net runs it: fp16 NHWC / token-major, tensor cores, fused epilogues

Inputs come from the seeded generator (di_synth_uniform) instead of Math.random, so runs repeat exactly.
Timing is measurePair (bench-timing.js:32-98): both paths warmed for 400 ms, one batch size N calibrated
for ~30 ms batches, per-iteration time = (t(2N) - t(N)) / N, the two paths interleaved, 7 repeats;
times are device times between CUDA events on the context's stream.
"""
from __future__ import annotations

import ctypes
import time

import numpy as np

from . import Context, default_context, lib
from . import ops as O

TARGET_BATCH_MS = 30.0
MIN_N, MAX_N = 2, 200
REPEATS = 7
WARM_MS = 400.0


def measure_pair(run_a, run_b, repeats: int | None = None):
    """bench-timing.js:49-98 with device-side timing: returns {"a": [ms...], "b": [ms...]}."""
    import torch
    repeats = REPEATS if repeats is None else repeats

    def time_batch(run, count):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(count):
            run()
        e1.record()
        e1.synchronize()
        return e0.elapsed_time(e1)

    until = time.perf_counter() + WARM_MS / 1e3
    while time.perf_counter() < until:
        run_a()
        run_b()
        torch.cuda.synchronize()

    def calibrate(run):
        c1, c2 = time_batch(run, 2), time_batch(run, 4)
        per = max((c2 - c1) / 2, 1e-5)
        return max(MIN_N, min(MAX_N, round(TARGET_BATCH_MS / per)))

    n = min(calibrate(run_a), calibrate(run_b))

    def slope(run):
        t1 = time_batch(run, n)
        t2 = time_batch(run, 2 * n)
        return (t2 - t1) / n

    a, b = [], []
    for _ in range(repeats):
        a.append(slope(run_a))
        b.append(slope(run_b))
    return {"a": a, "b": b}


def measure_one(run, repeats: int | None = None):
    return measure_pair(run, run, repeats)["a"]


def _med(xs):
    s = sorted(xs)
    return s[len(s) // 2]


def _rand(seed, name, n, s):
    out = np.empty(n, np.float32)
    lib().di_synth_uniform(seed, name.encode(), n, float(s), out.ctypes.data_as(ctypes.c_void_p))
    return out


def _cuda(a, dtype=None):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.to(dtype) if dtype is not None else t


def _diff(naive, fused):
    a = np.asarray(naive, np.float64).ravel()
    b = np.asarray(fused, np.float64).ravel()
    d = np.abs(a - b)
    return {"maxAbsDiff": float(d.max()), "l2": float(np.sqrt(np.mean(d * d)))}


def _result(shape, timing, flops=None, bytes_saved=None, disp=(1, 1), kern=(1, 1), corr=None, dt=("fp32", "fp16")):
    naive, fused = _med(timing["a"]), _med(timing["b"])
    r = {"shape": shape, "naive": naive, "fused": fused, "speedup": naive / fused}
    if flops is not None:
        r["tflopsNaive"] = flops / (naive / 1e3) / 1e12
        r["tflopsFused"] = flops / (fused / 1e3) / 1e12
    if bytes_saved is not None:
        r["bytesSaved"] = bytes_saved
    r["correctness"] = corr
    r["dispatchesNaive"], r["dispatchesFused"] = disp
    r["kernelsNaive"], r["kernelsFused"] = kern
    r["naiveRuns"], r["fusedRuns"] = timing["a"], timing["b"]
    r["dtypeNaive"], r["dtypeFused"] = dt
    return r


def _pack_conv(ctx, w32, Co, Ci):
    import torch
    wp = torch.empty((Co, 9 * Ci), dtype=torch.float16, device="cuda")
    wf = _cuda(w32)
    ctx.check(lib().di_pack_conv3x3(ctx.h, 1, wf.data_ptr(), Co, Ci, wp.data_ptr()), "pack_conv3x3")
    return wp


def _to_nhwc16(x, N, C, H, W):
    return _cuda(np.transpose(x.reshape(N, C, H, W), (0, 2, 3, 1)).copy()).half()


def runConvBench(onProgress=lambda s: None, ctx: Context | None = None, seed: int = 11):
    """fused-conv.js:174-284: y = silu(conv3x3(x) + b) + r at [1, 1280, 16, 16]."""
    import torch
    ctx = ctx or default_context()
    B, C, H, W, K = 1, 1280, 16, 16, 3
    shape = {"B": B, "C": C, "H": H, "W": W, "K": K}
    onProgress("allocating buffers…")
    n_io, n_w = B * C * H * W, C * C * K * K
    X, Wt, R = _rand(seed, "conv.x", n_io, 0.05), _rand(seed, "conv.w", n_w, 0.03), _rand(seed, "conv.r", n_io, 0.05)
    bias = np.zeros(C, np.float32)
    Xd, Wd, Bd, Rd = _cuda(X), _cuda(Wt), _cuda(bias), _cuda(R)
    Yn = torch.empty(n_io, device="cuda")
    enc = O.createCommandEncoder(ctx)
    conv = O.convMM(ctx)
    silu = O.unary(ctx, "SiLU")
    add = O.binary(ctx, "Add")
    cfg = O.createUniform(ctx, np.array([C, C, K, K * K, H, W, 1, 1, H, W, 0, 0], np.uint32))

    def run_naive():
        conv(enc, Xd, Wd, Bd, Yn, cfg, C, H * W)
        silu(enc, Yn, Yn, n_io)
        add(enc, Yn, Rd, Yn, n_io)

    X16, R16 = _to_nhwc16(X, B, C, H, W), _to_nhwc16(R, B, C, H, W)
    Wp = _pack_conv(ctx, Wt, C, C)
    Yf = torch.empty((B, H, W, C), dtype=torch.float16, device="cuda")

    def run_fused():
        ctx.check(lib().di_conv3x3_nhwc_act(ctx.h, 1, X16.data_ptr(), C, None, 0, B, H, W, 1, Wp.data_ptr(), C,
                                            Bd.data_ptr(), None, R16.data_ptr(), 1, Yf.data_ptr()), "conv_act")

    onProgress("correctness check…")
    run_naive()
    run_fused()
    torch.cuda.synchronize()
    corr = _diff(Yn.cpu().numpy(), Yf.float().permute(0, 3, 1, 2).reshape(-1).cpu().numpy())
    onProgress("timing naive vs fused (interleaved)…")
    t = measure_pair(run_naive, run_fused)
    flops = 2 * B * C * H * W * C * K * K
    return _result(shape, t, flops, 4 * n_io * 4, (3, 1), (7, 1), corr)


def runGroupNormBench(onProgress=lambda s: None, ctx: Context | None = None, seed: int = 12):
    """fused-groupnorm.js:280-383: GroupNorm(32) at [1, 1280, 16, 16]."""
    import torch
    ctx = ctx or default_context()
    B, C, G, H, W = 1, 1280, 32, 16, 16
    HW, n = H * W, B * C * H * W
    X = _rand(seed, "gn.x", n, 1.0)
    gamma = 1 + _rand(seed, "gn.g", C, 0.1)
    beta = _rand(seed, "gn.b", C, 0.1)
    Xd, Gd, Bd = _cuda(X), _cuda(gamma), _cuda(beta)
    Yn = torch.empty(n, device="cuda")
    cfg = np.zeros(8, np.uint32)
    cfg[:4] = (B, G, C // G, HW)
    cfg[4] = np.array([1e-5], np.float32).view(np.uint32)[0]
    u = O.createUniform(ctx, cfg)
    gn = O.groupNorm(ctx)
    enc = O.createCommandEncoder(ctx)

    def run_naive():
        gn(enc, Xd, Gd, Bd, Yn, u, G, B)

    X16 = _to_nhwc16(X, B, C, H, W)
    Yf = torch.empty_like(X16)

    def run_fused():
        ctx.check(lib().di_group_norm_nhwc(ctx.h, 1, X16.data_ptr(), C, None, 0, B, HW, G, 1e-5, Gd.data_ptr(),
                                           Bd.data_ptr(), 0, Yf.data_ptr()), "gn")

    run_naive()
    run_fused()
    torch.cuda.synchronize()
    corr = _diff(Yn.cpu().numpy(), Yf.float().permute(0, 3, 1, 2).reshape(-1).cpu().numpy())
    t = measure_pair(run_naive, run_fused)
    return _result({"B": B, "C": C, "G": G, "H": H, "W": W}, t, None, 2 * n * 4, (2, 1), (2, 2), corr)


def runResNetBench(onProgress=lambda s: None, ctx: Context | None = None, seed: int = 13):
    """fused-resnet.js:267-420: conv2(silu(GN2(conv1(silu(GN1(x)))))) + x at [1, 1280, 16, 16] (no
    timestep add, as in the reference bench: the fused plan gets a zero time projection)."""
    import torch
    from .blocks import ResNetBlock
    ctx = ctx or default_context()
    B, C, G, H, W, K = 1, 1280, 32, 16, 16, 3
    HW, n = H * W, B * C * H * W
    P = {"norm1.weight": 1 + _rand(seed, "r.g1", C, 0.02), "norm1.bias": _rand(seed, "r.b1", C, 0.02),
         "conv1.weight": _rand(seed, "r.w1", C * C * 9, 0.02), "conv1.bias": np.zeros(C, np.float32),
         "time_emb_proj.weight": np.zeros(C * 1280, np.float32), "time_emb_proj.bias": np.zeros(C, np.float32),
         "norm2.weight": 1 + _rand(seed, "r.g2", C, 0.02), "norm2.bias": _rand(seed, "r.b2", C, 0.02),
         "conv2.weight": _rand(seed, "r.w2", C * C * 9, 0.02), "conv2.bias": np.zeros(C, np.float32)}
    X = _rand(seed, "r.x", n, 1.0)
    D = {k: _cuda(v) for k, v in P.items()}
    Xd = _cuda(X)
    h1, h2 = torch.empty(n, device="cuda"), torch.empty(n, device="cuda")
    Yn = torch.empty(n, device="cuda")
    cfg_gn = np.zeros(8, np.uint32)
    cfg_gn[:4] = (B, G, C // G, HW)
    cfg_gn[4] = np.array([1e-5], np.float32).view(np.uint32)[0]
    ugn = O.createUniform(ctx, cfg_gn)
    ucv = O.createUniform(ctx, np.array([C, C, K, K * K, H, W, 1, 1, H, W, 0, 0], np.uint32))
    gn, conv, silu, add = O.groupNorm(ctx), O.convMM(ctx), O.unary(ctx, "SiLU"), O.binary(ctx, "Add")
    enc = O.createCommandEncoder(ctx)

    def run_naive():  # 8 dispatches: GN, SiLU, conv, GN, SiLU, conv, add (GN = stats + normalise)
        gn(enc, Xd, D["norm1.weight"], D["norm1.bias"], h1, ugn, G, B)
        silu(enc, h1, h1, n)
        conv(enc, h1, D["conv1.weight"], D["conv1.bias"], h2, ucv, C, HW)
        gn(enc, h2, D["norm2.weight"], D["norm2.bias"], h1, ugn, G, B)
        silu(enc, h1, h1, n)
        conv(enc, h1, D["conv2.weight"], D["conv2.bias"], Yn, ucv, C, HW)
        add(enc, Yn, Xd, Yn, n)

    blk = ResNetBlock(ctx, N=B, C=C, H=H, W=W, seed=seed, weights=lambda name, k: P.get(name))
    blk.x.copy_(Xd.view(B, C, H, W))
    blk.temb.zero_()

    def run_fused():
        blk.run()

    run_naive()
    run_fused()
    torch.cuda.synchronize()
    corr = _diff(Yn.cpu().numpy(), blk.y.reshape(-1).cpu().numpy())
    t = measure_pair(run_naive, run_fused)
    flops = 2 * 2 * B * C * H * W * C * K * K
    return _result({"B": B, "C": C, "G": G, "H": H, "W": W, "K": K}, t, flops, 6 * n * 4, (9, 4), (15, 9), corr,
                   ("fp32", "fp32 io, fp16 tensor-core operands"))


def _attn_bench(B, H, Sq, Skv, seed, tag):
    import torch
    ctx = default_context()
    d = 64
    Q = _rand(seed, tag + ".q", B * H * Sq * d, 0.5)
    Kt = _rand(seed, tag + ".k", B * H * Skv * d, 0.5)
    V = _rand(seed, tag + ".v", B * H * Skv * d, 0.5)
    Qd, Kd, Vd = _cuda(Q), _cuda(Kt), _cuda(V)
    KT = torch.empty(B * H * d * Skv, device="cuda")
    S = torch.empty(B * H * Sq * Skv, device="cuda")
    P = torch.empty_like(S)
    On = torch.empty(B * H * Sq * d, device="cuda")
    scale = _cuda(np.array([1 / np.sqrt(d)], np.float32))
    enc = O.createCommandEncoder(ctx)
    tr, mm, sm, mul = O.transpose(ctx), O.matmul(ctx), O.softmax(ctx), O.binary(ctx, "Mul")
    # [BH, Skv, d] -> [BH, d, Skv]: output dim k reads input dim perm[k] (wgsl-ops.js:990-1030 cfg layout)
    u_tr = O.createUniform(ctx, np.array([3, 0, 0, 0, B * H, d, Skv, 0, Skv * d, d, 1, 0, 0, 2, 1, 0,
                                          B * H * Skv * d, 0, 0, 0], np.uint32))
    u_qk = O.createUniform(ctx, np.array([Sq, Skv, d, 1], np.uint32))
    u_sm = O.createUniform(ctx, np.array([Skv, B * H * Sq], np.uint32))
    u_pv = O.createUniform(ctx, np.array([Sq, d, Skv, 1], np.uint32))

    def run_naive():  # K^T, scores = Q K^T, * 1/sqrt(d), softmax, out = P V
        tr(enc, Kd, KT, u_tr, B * H * Skv * d)
        mm(enc, Qd, KT, S, u_qk, Sq, Skv, B * H)
        mul(enc, S, scale, S, B * H * Sq * Skv)
        sm(enc, S, P, u_sm, B * H * Sq)
        mm(enc, P, Vd, On, u_pv, Sq, d, B * H)

    Q16, K16, V16 = Qd.half(), Kd.half(), Vd.half()
    Of = torch.empty_like(Q16)

    def run_fused():
        ctx.check(lib().di_attention(ctx.h, 1, Q16.data_ptr(), K16.data_ptr(), V16.data_ptr(), Of.data_ptr(), B, H,
                                     Sq, Skv, 1), "attention")

    run_naive()
    run_fused()
    torch.cuda.synchronize()
    corr = _diff(On.cpu().numpy(), Of.float().reshape(-1).cpu().numpy())
    t = measure_pair(run_naive, run_fused)
    flops = 4 * B * H * Sq * Skv * d
    return t, flops, corr, 2 * B * H * Sq * Skv * 4


def runAttnBench(onProgress=lambda s: None, seed: int = 14):
    """fused-attn.js:364-476: softmax(Q K^T / 8) V at B=2, H=20, S=256, d=64."""
    B, H, S = 2, 20, 256
    t, flops, corr, saved = _attn_bench(B, H, S, S, seed, "attn")
    r = _result({"B": B, "H": H, "S": S, "HEAD_DIM": 64, "D": H * 64}, t, flops, saved, (3, 1), (9, 1), corr)
    return r


def runCrossAttnBench(onProgress=lambda s: None, seed: int = 15):
    """fused-cross-attn.js:220-318: S_q = 256 queries against S_kv = 77 keys, B=2, 20 heads."""
    B, H, Sq, Skv = 2, 20, 256, 77
    t, flops, corr, saved = _attn_bench(B, H, Sq, Skv, seed, "xattn")
    return _result({"B": B, "HEADS": H, "S_Q": Sq, "S_KV": Skv, "HEAD_DIM": 64}, t, None, saved, (3, 1), (9, 1), corr)


def runTEmbedBench(onProgress=lambda s: None, ctx: Context | None = None, seed: int = 16):
    """fused-tembed.js:175-267: t -> [cos(t f) | sin(t f)] -> Linear(320, 1280) -> SiLU -> Linear(1280, 1280)."""
    import torch
    ctx = ctx or default_context()
    E, Hd, tval = 320, 1280, 500.0
    W1, b1 = _rand(seed, "te.w1", Hd * E, 0.05), _rand(seed, "te.b1", Hd, 0.05)
    W2, b2 = _rand(seed, "te.w2", Hd * Hd, 0.03), _rand(seed, "te.b2", Hd, 0.03)
    freqs = np.exp(-np.log(10000.0) * np.arange(160) / 160).astype(np.float32)
    D = {k: _cuda(v) for k, v in dict(W1=W1, b1=b1, W2=W2, b2=b2, f=freqs).items()}
    tt = _cuda(np.array([tval], np.float32))
    arg, c, s_ = (torch.empty(160, device="cuda") for _ in range(3))
    emb, h, yn = torch.empty(E, device="cuda"), torch.empty(Hd, device="cuda"), torch.empty(Hd, device="cuda")
    enc = O.createCommandEncoder(ctx)
    mul, cos, sin, cat = O.binary(ctx, "Mul"), O.unary(ctx, "Cos"), O.unary(ctx, "Sin"), O.concatCopy(ctx)
    gemm, silu = O.gemm(ctx), O.unary(ctx, "SiLU")
    u_c0 = O.createUniform(ctx, np.array([160, 320, 0, 160], np.uint32))
    u_c1 = O.createUniform(ctx, np.array([160, 320, 160, 160], np.uint32))
    u_g1 = O.createUniform(ctx, np.array([1, Hd, E, 1], np.uint32))
    u_g2 = O.createUniform(ctx, np.array([1, Hd, Hd, 1], np.uint32))

    def run_naive():
        mul(enc, D["f"], tt, arg, 160)
        cos(enc, arg, c, 160)
        sin(enc, arg, s_, 160)
        cat(enc, c, emb, u_c0, 160)
        cat(enc, s_, emb, u_c1, 160)
        gemm(enc, emb, D["W1"], D["b1"], h, u_g1, 1, Hd)
        silu(enc, h, h, Hd)
        gemm(enc, h, D["W2"], D["b2"], yn, u_g2, 1, Hd)

    yf = torch.empty(Hd, device="cuda")

    def run_fused():
        ctx.check(lib().di_tembed(ctx.h, tt.data_ptr(), 1, D["W1"].data_ptr(), D["b1"].data_ptr(), D["W2"].data_ptr(),
                                  D["b2"].data_ptr(), E, Hd, yf.data_ptr()), "tembed")

    run_naive()
    run_fused()
    torch.cuda.synchronize()
    corr = _diff(yn.cpu().numpy(), yf.cpu().numpy())
    t = measure_pair(run_naive, run_fused)
    r = _result(None, t, None, None, (8, 1), (14, 2), corr, ("fp32", "fp32"))
    r.pop("shape")
    r["dims"] = {"EMB_DIM": E, "HID_DIM": Hd}
    return r


ALL = {"conv": runConvBench, "groupnorm": runGroupNormBench, "resnet": runResNetBench, "attn": runAttnBench,
       "cross-attn": runCrossAttnBench, "tembed": runTEmbedBench}


def run_all(names=None):
    """One JSON-able summary per bench (the shape bench-headless.mjs prints), run times dropped."""
    out = []
    for nm in names or list(ALL):
        r = ALL[nm](lambda s: None)
        out.append({"bench": nm, **{k: v for k, v in r.items() if k not in ("naiveRuns", "fusedRuns")}})
    return out
