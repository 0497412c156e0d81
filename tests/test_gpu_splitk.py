"""GEMMs under forced tilings (K splits finished by the reduce kernel or summed across a thread-block
cluster through distributed shared memory, paired and single CTAs, several tile widths) in child
processes, against torch fp32, with bit-identical repeats.  A forced tiling "bn,splits,2" is a cluster
split-K with `splits` CTAs per cluster (GEGLU keeps the reduce kernel)."""
from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
HERE = Path(__file__).resolve().parent


@pytest.mark.parametrize("tiling", ["128,4", "256,3,1", "160,2", "128,1", "128,4,2", "256,8,2", "160,3,2", "192,2,2",
                                    "128,6,2"])
def test_split_k_forced(ctx, tiling):
    env = dict(os.environ, DI_GEMM_TILING=tiling)
    r = subprocess.run([sys.executable, str(HERE / "splitk_case.py")], cwd=HERE, env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    res = json.loads(r.stdout.strip().splitlines()[-1])
    assert res.pop("fault") == 0
    for name, (err, same) in res.items():
        assert err < 1e-2, (name, err)
        assert same, name
