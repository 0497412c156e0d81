"""The optional GroupNorm path whose statistics come from the producing GEMM's epilogue (and from the
split-K reduce) as exact fixed-point sums: U-Net parity against the oracle and bit-identical replays,
in a child process with DI_GN_STATS=1."""
from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
HERE = Path(__file__).resolve().parent


def test_unet_with_epilogue_gn_stats(ctx):
    env = dict(os.environ, DI_GN_STATS="1")
    r = subprocess.run([sys.executable, str(HERE / "gnstats_case.py")], cwd=HERE, env=env, capture_output=True,
                       text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-2000:]
    res = json.loads(r.stdout.strip().splitlines()[-1])
    assert res["fault"] == 0 and res["finite"] and res["same"]
    assert res["cos"] >= 0.999
    assert res["rel"] <= 1e-2
