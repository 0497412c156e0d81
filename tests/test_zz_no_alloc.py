"""di_group_norm_nhwc_noalloc: the GroupNorm entry point for callers that cannot let the library allocate
device memory (a fixed pre-reserved budget, an external allocator owning the device, allocation-free
latency-critical paths).  It must give the same result as di_group_norm_nhwc, on consecutive calls that
share its fixed scratch array, and refuse sizes that need more scratch than the array holds.

Kept in its own file, named to be collected last, so a run that stops at the first failure has already
run every other test.  Works alone in a fresh process and after the rest of the suite."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu


def _run(ctx, dib, fn, x1, x2, C1, C2, N, HW, g, b, silu):
    import torch
    y = torch.empty((N, HW, C1 + C2), dtype=torch.float16, device="cuda")
    rc = getattr(dib.lib(), fn)(ctx.h, 1, x1.data_ptr(), C1, x2.data_ptr() if x2 is not None else None, C2, N, HW,
                                32, 1e-5, g.data_ptr(), b.data_ptr(), silu, y.data_ptr())
    ctx.check(rc, fn)
    torch.cuda.synchronize()
    return y.float().cpu().numpy()


def test_noalloc_matches_group_norm_on_two_calls(ctx, dib):
    import torch
    rng = np.random.default_rng(11)
    cases = [(1, 4096, 320, 0, 1), (2, 256, 1280, 640, 1)]  # second call: other shape, concat input, batch 2
    for N, HW, C1, C2, silu in cases:
        C = C1 + C2
        x = torch.from_numpy((rng.standard_normal((N, HW, C)) * 1.5 + 0.3).astype(np.float32)).half().cuda()
        x1 = x[..., :C1].contiguous()
        x2 = x[..., C1:].contiguous() if C2 else None
        g = torch.from_numpy((1 + 0.1 * rng.standard_normal(C)).astype(np.float32)).cuda()
        b = torch.from_numpy((0.1 * rng.standard_normal(C)).astype(np.float32)).cuda()
        ref = _run(ctx, dib, "di_group_norm_nhwc", x1, x2, C1, C2, N, HW, g, b, silu)
        got = _run(ctx, dib, "di_group_norm_nhwc_noalloc", x1, x2, C1, C2, N, HW, g, b, silu)
        assert np.all(np.isfinite(got))
        assert rel_err(got, ref) < 1e-2
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
