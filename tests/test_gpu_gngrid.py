"""The optional single-launch GroupNorm (statistics, grid barrier and normalise in one kernel): direct
calls against the oracle with bit-identical repeat calls, and U-Net parity with bit-identical replays, in
a child process with DI_GN_GRID=1."""
from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
HERE = Path(__file__).resolve().parent


def test_single_launch_group_norm(ctx):
    env = dict(os.environ, DI_GN_GRID="1")
    r = subprocess.run([sys.executable, str(HERE / "gngrid_case.py")], cwd=HERE, env=env, capture_output=True,
                       text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-2000:]
    res = json.loads(r.stdout.strip().splitlines()[-1])
    assert res["fault"] == 0 and res["finite"] and res["same"] and res["gn_same"]
    assert res["gn_rel"] < 1e-2
    assert res["cos"] >= 0.999
    assert res["rel"] <= 1e-2
