"""The sticky device-fault path (the analogue of unet-wgsl.js:32-38's _gpuError / getUNetGpuFault), on a
B200 without faulting the GPU: a probe kernel's bounded mbarrier wait runs out on a phase that nothing
completes, records its flag in the device error word and returns.  The context must report the fault,
refuse nothing it should not, clear it on request, and compute correctly afterwards."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

DEVERR_WAIT_PROBE = 64


def test_timed_out_wait_sets_sticky_fault_and_clears(ctx, dib, oracle):
    import torch
    L = dib.lib()
    assert ctx.fault() == 0
    ctx.check(L.di_debug_wait_timeout(ctx.h, 2000), "di_debug_wait_timeout")  # 2 ms limit
    torch.cuda.synchronize()  # the kernel returned: the context is alive
    f = ctx.fault()
    assert f & DEVERR_WAIT_PROBE, f"fault flags {f}"
    assert L.di_wait(ctx.h) == dib.DI_EFAULT  # sticky until cleared
    ctx.clear_fault()
    assert ctx.fault() == 0
    assert L.di_wait(ctx.h) == dib.DI_OK
    # the context still computes correctly: a GroupNorm against the oracle
    rng = np.random.default_rng(9)
    N, HW, C = 1, 1024, 320
    x = (rng.standard_normal((N, HW, C)) * 2 + 0.5).astype(np.float32)
    X = torch.from_numpy(x).half().cuda()
    g = torch.from_numpy((1 + 0.1 * rng.standard_normal(C)).astype(np.float32)).cuda()
    b = torch.from_numpy((0.1 * rng.standard_normal(C)).astype(np.float32)).cuda()
    Y = torch.empty_like(X)
    ctx.check(L.di_group_norm_nhwc(ctx.h, 1, X.data_ptr(), C, None, 0, N, HW, 32, 1e-5, g.data_ptr(), b.data_ptr(), 1,
                                   Y.data_ptr()), "gn")
    torch.cuda.synchronize()
    xn = np.ascontiguousarray(np.transpose(X.float().cpu().numpy(), (0, 2, 1)))
    ref = np.transpose(oracle.group_norm(xn, g.cpu().numpy(), b.cpu().numpy(), N, C, HW, 32, 1e-5, silu=True),
                       (0, 2, 1))
    assert rel_err(Y.float().cpu().numpy(), ref) < 1e-2
    assert ctx.fault() == 0


def test_wait_probe_rejects_bad_limit(ctx, dib):
    assert dib.lib().di_debug_wait_timeout(ctx.h, 0) == dib.DI_EINVAL
    assert dib.lib().di_debug_wait_timeout(ctx.h, 2_000_000) == dib.DI_EINVAL
