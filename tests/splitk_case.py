"""Child process of test_gpu_splitk.py: runs GEMMs under the tiling forced by DI_GEMM_TILING (read once per
process) and prints the worst relative error against torch fp32 and whether repeats are bit-identical."""
from __future__ import annotations

import json
import sys

import numpy as np
import torch

from conftest import load_package


def main():
    dib = load_package()
    ctx = dib.Context(0)
    L = dib.lib()
    g = torch.Generator().manual_seed(7)
    out = {}

    def rnd(*shape, scale=1.0, dt=torch.float16):
        return (torch.randn(*shape, generator=g) * scale).to(dt).cuda()

    def rel(a, b):
        return float((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-6))

    # linear + bias + residual / SiLU / GELU (M not a multiple of 32, N not a multiple of 32)
    for act in (0, 1, 2):
        M, K, N = 1000, 1024, 208
        x, w = rnd(M, K), rnd(N, K, scale=1 / 32)
        b = torch.randn(N, generator=g).cuda()
        r = rnd(M, N)
        ys = []
        for _ in range(3):
            y = torch.empty(M, N, dtype=torch.float16, device="cuda")
            ctx.check(L.di_linear_act(ctx.h, dib.DI_F16, x.data_ptr(), M, K, w.data_ptr(), N, b.data_ptr(),
                                      r.data_ptr(), act, y.data_ptr()), "di_linear_act")
            ys.append(y)
        torch.cuda.synchronize()
        z = x.float() @ w.float().T + b
        z = torch.nn.functional.silu(z) if act == 1 else torch.nn.functional.gelu(z) if act == 2 else z
        ref = z + r.float()
        out[f"linear_act{act}"] = [rel(ys[0], ref), all(torch.equal(ys[0], t) for t in ys[1:])]
    # conv3x3 with bias + per-image row vector + residual
    N_, H, W, C, Co = 2, 16, 16, 128, 192
    x = rnd(N_, H, W, C)
    w32 = torch.randn(Co, C, 3, 3, generator=g) / 34
    wp = torch.empty(Co * 9 * C, dtype=torch.float16, device="cuda")
    w32c = w32.cuda()
    ctx.check(L.di_pack_conv3x3(ctx.h, dib.DI_F16, w32c.data_ptr(), Co, C, wp.data_ptr()), "pack")
    ctx.check(L.di_wait(ctx.h), "wait")
    b = torch.randn(Co, generator=g).cuda()
    temb = torch.randn(N_, Co, generator=g).cuda()
    r = rnd(N_, H, W, Co)
    ys = []
    for _ in range(3):
        y = torch.empty(N_, H, W, Co, dtype=torch.float16, device="cuda")
        ctx.check(L.di_conv3x3_nhwc(ctx.h, dib.DI_F16, x.data_ptr(), C, None, 0, N_, H, W, 1, wp.data_ptr(), Co,
                                    b.data_ptr(), temb.data_ptr(), r.data_ptr(), y.data_ptr()), "conv")
        ys.append(y)
    torch.cuda.synchronize()
    ref = torch.nn.functional.conv2d(x.float().permute(0, 3, 1, 2), w32.half().float().cuda(), b, padding=1)
    ref = ref.permute(0, 2, 3, 1) + temb[:, None, None, :] + r.float()
    out["conv"] = [rel(ys[0], ref), all(torch.equal(ys[0], t) for t in ys[1:])]
    # GEGLU (split partials finished by the reduce kernel)
    M, K, F = 300, 512, 256
    x, w = rnd(M, K), rnd(2 * F, K, scale=1 / 23)
    b = torch.randn(2 * F, generator=g).cuda()
    y = torch.empty(M, F, dtype=torch.float16, device="cuda")
    ctx.check(L.di_linear_geglu(ctx.h, dib.DI_F16, x.data_ptr(), M, K, w.data_ptr(), F, b.data_ptr(),
                                y.data_ptr()), "geglu")
    torch.cuda.synchronize()
    z = x.float() @ w.float().T + b  # packed: per 128 columns, 64 value columns then their 64 gates
    o = torch.arange(F)
    nv = (o // 64) * 128 + o % 64
    ref = z[:, nv] * torch.nn.functional.gelu(z[:, nv + 64])
    out["geglu"] = [rel(y, ref), True]
    out["fault"] = ctx.fault()
    print(json.dumps(out))


if __name__ == "__main__":
    sys.exit(main())
