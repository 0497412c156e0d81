"""Standalone driver for profiling the config-3 attention (not a test): runs di_attention three times on
Q/K/V [8, 5, 4096, 64] head-major bf16 drawn like bench.py's (seed-2 generator, N(0,1)/8), self-attention
by default or cross-attention (K/V [8, 5, 77, 64]) with --cross: the command the committed ncu capture
of the config-3 attention kernel profiles."""
from __future__ import annotations

import sys

import torch

from conftest import load_package


def main():
    dib = load_package()
    ctx = dib.Context(0)
    L = dib.lib()
    g = torch.Generator(device="cuda").manual_seed(2)
    mk = lambda *s: (torch.randn(*s, device="cuda", generator=g) / 8).bfloat16()
    q, k, v = mk(8, 5, 4096, 64), mk(8, 5, 4096, 64), mk(8, 5, 4096, 64)
    skv = 4096
    if "--cross" in sys.argv:
        k, v, skv = mk(8, 5, 77, 64), mk(8, 5, 77, 64), 77
    o = torch.empty_like(q)
    for _ in range(3):
        ctx.check(L.di_attention(ctx.h, 2, q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), 8, 5, 4096, skv, 1),
                  "di_attention")
    torch.cuda.synchronize()
    assert ctx.fault() == 0
    print("ok", float(o.float().abs().mean()))


if __name__ == "__main__":
    main()
