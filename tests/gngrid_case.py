"""Child process of test_gpu_gngrid.py: the single-launch GroupNorm (DI_GN_GRID=1, read once per process)
through di_group_norm_nhwc on several shapes and inside a U-Net forward, printed as JSON with the oracle
comparison."""
from __future__ import annotations

import importlib
import json
import sys

import numpy as np

from conftest import cosine, load_package, rel_err


def main():
    dib = load_package()
    import oracle
    oracle.build()
    import torch
    ctx = dib.Context(0)
    rng = np.random.default_rng(5)
    gn_rel, gn_same = [], True
    # (N, HW, C1, C2, silu): one image, ragged slices, concat input, several images, small map
    for N, HW, C1, C2, silu in [(1, 4096, 320, 0, 1), (1, 1000, 640, 0, 1), (3, 4096, 320, 320, 0),
                                (16, 64, 1280, 0, 1), (2, 256, 1280, 1280, 1)]:
        C = C1 + C2
        x = (rng.standard_normal((N, HW, C)) * 2 + 0.5).astype(np.float16).astype(np.float32)
        g = (1 + 0.1 * rng.standard_normal(C)).astype(np.float32)
        b = (0.1 * rng.standard_normal(C)).astype(np.float32)
        X1 = torch.from_numpy(np.ascontiguousarray(x[..., :C1])).half().cuda()
        X2 = torch.from_numpy(np.ascontiguousarray(x[..., C1:])).half().cuda() if C2 else None
        Gt, Bt = torch.from_numpy(g).cuda(), torch.from_numpy(b).cuda()
        outs = []
        for _ in range(2):
            Y = torch.empty((N, HW, C), dtype=torch.float16, device="cuda")
            ctx.check(dib.lib().di_group_norm_nhwc(ctx.h, 1, X1.data_ptr(), C1, X2.data_ptr() if C2 else None, C2,
                                                   N, HW, 32, 1e-5, Gt.data_ptr(), Bt.data_ptr(), silu,
                                                   Y.data_ptr()), "gn")
            torch.cuda.synchronize()
            outs.append(Y.float().cpu().numpy())
        ref = oracle.group_norm(np.ascontiguousarray(np.transpose(x, (0, 2, 1))), g, b, N, C, HW, 32, 1e-5,
                                silu=bool(silu))
        gn_rel.append(rel_err(outs[0], np.transpose(ref, (0, 2, 1))))
        gn_same = gn_same and bool(np.array_equal(outs[0], outs[1]))
    unet = importlib.import_module("draw_instant_b200.unet")
    B, H, W, seed = 2, 16, 16, 3
    u = unet.UNet(ctx, B=B, H=H, W=W, seed=seed)
    lat = oracle.gen_normal(seed, "latent", B * 4 * H * W).reshape(B, 4, H, W)
    cx = oracle.gen_normal(seed, "context", B * 77 * 1024).reshape(B, 77, 1024)
    got = u.forward_host(lat, 999.0, cx)
    again = u.forward_host(lat, 999.0, cx)
    ref = oracle.unet_forward(lat, 999.0, cx.astype(np.float16).astype(np.float32), seed)
    print(json.dumps({"gn_rel": max(gn_rel), "gn_same": gn_same, "cos": cosine(got, ref), "rel": rel_err(got, ref),
                      "same": bool(np.array_equal(got, again)), "finite": bool(np.all(np.isfinite(got))),
                      "fault": ctx.fault()}))


if __name__ == "__main__":
    sys.exit(main())
