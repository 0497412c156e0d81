"""Child process of test_gpu_gnstats.py: a U-Net forward with GroupNorm statistics taken from the GEMM
epilogues (DI_GN_STATS=1, read once per process), printed as JSON with the oracle comparison."""
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
    unet = importlib.import_module("draw_instant_b200.unet")
    ctx = dib.Context(0)
    B, H, W, seed = 2, 16, 16, 3
    u = unet.UNet(ctx, B=B, H=H, W=W, seed=seed)
    lat = oracle.gen_normal(seed, "latent", B * 4 * H * W).reshape(B, 4, H, W)
    cx = oracle.gen_normal(seed, "context", B * 77 * 1024).reshape(B, 77, 1024)
    got = u.forward_host(lat, 999.0, cx)
    again = u.forward_host(lat, 999.0, cx)
    ref = oracle.unet_forward(lat, 999.0, cx.astype(np.float16).astype(np.float32), seed)
    print(json.dumps({"cos": cosine(got, ref), "rel": rel_err(got, ref), "same": bool(np.array_equal(got, again)),
                      "finite": bool(np.all(np.isfinite(got))), "fault": ctx.fault()}))


if __name__ == "__main__":
    sys.exit(main())
