"""The opt-in variants that the default path does not take, each checked against the CPU oracle by the
existing parity tests run in a child process with its switch set (the switches are read once per
process):
  DI_LN_FOLD=1      LayerNorm folded into its consumer GEMM (config 2 transformer block, U-Net 8x8 / 16x16)
  DI_GN_CLUSTER=1   GroupNorm in one launch per 16-CTA cluster (GroupNorm shapes, config 1 ResNet block)
  DI_CLUSTER_SPLIT=1  split-K summed across a thread-block cluster (config 2 block, U-Net small cases)"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
HERE = Path(__file__).resolve().parent


@pytest.mark.parametrize("env,select", [
    ("DI_LN_FOLD", "test_gpu_plans.py::test_transformer_block_config2 test_gpu_plans.py::test_unet_config4_small"),
    ("DI_GN_CLUSTER", "test_gpu_kernels.py::test_group_norm_nhwc test_gpu_plans.py::test_resnet_block_config1"),
    ("DI_CLUSTER_SPLIT", "test_gpu_plans.py::test_transformer_block_config2 test_gpu_plans.py::test_unet_config4_small"),
])
def test_opt_in_variant_parity(ctx, env, select):
    e = dict(os.environ, **{env: "1"})
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", "-p", "no:cacheprovider",
                        *select.split()], cwd=HERE, env=e, capture_output=True, text=True, timeout=1500)
    assert r.returncode == 0, (env, r.stdout[-3000:], r.stderr[-2000:])
