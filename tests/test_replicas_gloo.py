"""The multi-GPU host logic (draw-instant_b200/replicas.py) as world-size-2 gloo ranks on the CPU:
sharding covers every image once, the output all-gather returns rank order, the job time is the max."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from conftest import ROOT


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    import sys
    sys.path.insert(0, str(ROOT / "tests"))
    from conftest import load_package
    load_package()
    import importlib
    R = importlib.import_module("draw_instant_b200.replicas")
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    R.init("gloo")
    first, count = R.shard(7, rank, world)
    # a stand-in "replica output": image index * 10 + rank-independent content
    out = torch.stack([torch.full((4, 2, 2), float(first + i) * 10) for i in range(count)])
    pad = torch.full((4 - count, 4, 2, 2), -1.0) if count < 4 else torch.empty(0, 4, 2, 2)
    full = R.gather(torch.cat([out, pad]))
    t = R.max_over_ranks(1.5 + rank)
    R.barrier()
    q.put((rank, first, count, full[:, 0, 0, 0].tolist(), t))
    R.finish()


@pytest.mark.timeout(120)
def test_two_rank_shard_gather_max():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=100) for _ in range(world))
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    (r0, f0, c0, g0, t0), (r1, f1, c1, g1, t1) = res
    assert (f0, c0, f1, c1) == (0, 4, 4, 3)  # 7 images: 4 + 3, contiguous, in rank order
    assert g0 == g1 == [0.0, 10.0, 20.0, 30.0, 40.0, 50.0, 60.0, -1.0]
    assert t0 == t1 == 2.5


def test_shard_covers_every_image_once():
    from conftest import load_package
    load_package()
    import importlib
    R = importlib.import_module("draw_instant_b200.replicas")
    for B in (1, 7, 8, 64):
        for world in (1, 2, 4, 8):
            seen = []
            for r in range(world):
                f, c = R.shard(B, r, world)
                seen += list(range(f, f + c))
            assert seen == list(range(B))
