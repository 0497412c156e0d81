"""di_group_norm_nhwc_noalloc: the GroupNorm entry point for callers that cannot let the library allocate
device memory (a fixed pre-reserved budget, an external allocator owning the device, allocation-free
latency-critical paths).  It must give the same result as di_group_norm_nhwc and as the CPU oracle, on
consecutive calls that share its fixed scratch array, allocate nothing once its first call on the device
has been made, and refuse sizes that need more scratch than the array holds.

Kept in its own file, named to be collected last, so a run that stops at the first failure has already
run every other test.  Works alone in a fresh process and after the rest of the suite."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import cosine, rel_err

pytestmark = pytest.mark.gpu

_DT = {"f16": 1, "bf16": 2}


def _run(ctx, dib, fn, dtype, x1, x2, C1, C2, N, HW, g, b, silu, y):
    import torch
    rc = getattr(dib.lib(), fn)(ctx.h, _DT[dtype], x1.data_ptr(), C1, x2.data_ptr() if x2 is not None else None, C2,
                                N, HW, 32, 1e-5, g.data_ptr(), b.data_ptr(), silu, y.data_ptr())
    ctx.check(rc, fn)
    torch.cuda.synchronize()
    return y.float().cpu().numpy()


def _inputs(rng, N, HW, C1, C2, dtype):
    import torch
    tdt = torch.float16 if dtype == "f16" else torch.bfloat16
    C = C1 + C2
    x = torch.from_numpy((rng.standard_normal((N, HW, C)) * 1.5 + 0.3).astype(np.float32)).to(tdt).cuda()
    x1 = x[..., :C1].contiguous()
    x2 = x[..., C1:].contiguous() if C2 else None
    g = torch.from_numpy((1 + 0.1 * rng.standard_normal(C)).astype(np.float32)).cuda()
    b = torch.from_numpy((0.1 * rng.standard_normal(C)).astype(np.float32)).cuda()
    y = torch.empty((N, HW, C), dtype=tdt, device="cuda")
    return x, x1, x2, g, b, y


def test_noalloc_matches_group_norm_on_two_calls(ctx, dib, oracle):
    import torch
    rng = np.random.default_rng(11)
    # second call: another shape, a concat input, batch 2; third: bf16
    cases = [(1, 4096, 320, 0, 1, "f16"), (2, 256, 1280, 640, 1, "f16"), (1, 1024, 640, 0, 0, "bf16")]
    for N, HW, C1, C2, silu, dtype in cases:
        C = C1 + C2
        x, x1, x2, g, b, y = _inputs(rng, N, HW, C1, C2, dtype)
        got = _run(ctx, dib, "di_group_norm_nhwc_noalloc", dtype, x1, x2, C1, C2, N, HW, g, b, silu, y)
        ref = _run(ctx, dib, "di_group_norm_nhwc", dtype, x1, x2, C1, C2, N, HW, g, b, silu, torch.empty_like(y))
        assert np.all(np.isfinite(got))
        assert rel_err(got, ref) < 1e-2
        # and against the CPU oracle on the same (storage-rounded) input, channels-first for the oracle
        xn = np.ascontiguousarray(np.transpose(x.float().cpu().numpy(), (0, 2, 1)))
        o = oracle.group_norm(xn, g.cpu().numpy(), b.cpu().numpy(), N, C, HW, 32, 1e-5, silu=bool(silu))
        o = np.transpose(o, (0, 2, 1))
        assert rel_err(got, o) < 1e-2
        assert cosine(got, o) > 0.9999
    assert ctx.fault() == 0


def test_noalloc_allocates_nothing_after_first_call(ctx, dib):
    """After one call on the device (the start-up call), a call on a new, larger shape leaves the device's
    free memory unchanged: no cudaMalloc, no workspace growth, no module load."""
    import torch
    rng = np.random.default_rng(5)
    _, x1, x2, g, b, y = _inputs(rng, 1, 256, 320, 0, "f16")
    _run(ctx, dib, "di_group_norm_nhwc_noalloc", "f16", x1, x2, 320, 0, 1, 256, g, b, 1, y)
    _, x1, x2, g, b, y = _inputs(rng, 4, 4096, 640, 320, "f16")  # all inputs and outputs exist beforehand
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(2):  # only the library call inside the measured region (no readback, no torch ops)
        ctx.check(dib.lib().di_group_norm_nhwc_noalloc(ctx.h, 1, x1.data_ptr(), 640, x2.data_ptr(), 320, 4, 4096, 32,
                                                       1e-5, g.data_ptr(), b.data_ptr(), 1, y.data_ptr()), "noalloc")
        torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info()[0]
    assert free1 == free0, f"free device memory changed by {free0 - free1} bytes"
    assert np.all(np.isfinite(y.float().cpu().numpy()))
    assert ctx.fault() == 0


def test_noalloc_rejects_oversize(ctx, dib):
    import torch
    # N=256 images x 16 cluster partials x 32 groups x 8 B = 1 MiB -> fits; N=257 needs more than the fixed 1 MiB
    x = torch.zeros((257, 4096, 64), dtype=torch.float16, device="cuda")
    g = torch.ones(64, device="cuda")
    b = torch.zeros(64, device="cuda")
    y = torch.empty_like(x)
    rc = dib.lib().di_group_norm_nhwc_noalloc(ctx.h, 1, x.data_ptr(), 64, None, 0, 257, 4096, 32, 1e-5, g.data_ptr(),
                                              b.data_ptr(), 0, y.data_ptr())
    assert rc == dib.DI_EINVAL
    assert b"fixed maximum" in dib.lib().di_last_error(ctx.h)
