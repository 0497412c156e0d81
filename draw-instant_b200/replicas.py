"""Multi-GPU plumbing of the denoising path: one full U-Net replica per GPU, latents sharded by image.

The path has no data-path collective (images are independent); the only exchange is one all-gather of
the replicas' outputs at the end (NCCL over NVLink on GPUs; gloo on CPU for the host-logic tests), and
the job's time is the maximum over ranks.  One process per GPU, environment from torchrun
(RANK / WORLD_SIZE / LOCAL_RANK / MASTER_ADDR / MASTER_PORT)."""
from __future__ import annotations

import os


def env():
    """(rank, world, local_rank) from the launcher's environment (1 process when unset)."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def init(backend: str = "nccl", device=None) -> None:
    """Joins the process group when WORLD_SIZE > 1 (rendezvous on MASTER_ADDR, e.g. 127.0.0.1)."""
    import torch.distributed as dist
    _, world, _ = env()
    if world > 1 and not dist.is_initialized():
        if device is not None:
            dist.init_process_group(backend, device_id=device)
        else:
            dist.init_process_group(backend)


def shard(global_batch: int, rank: int, world: int) -> tuple[int, int]:
    """(first image, count) of this rank's contiguous share; earlier ranks take the remainder."""
    base, extra = divmod(global_batch, world)
    count = base + (1 if rank < extra else 0)
    first = rank * base + min(rank, extra)
    return first, count


def gather(t):
    """All ranks' outputs concatenated along dim 0 in rank order (equal shares; one all_gather)."""
    import torch
    import torch.distributed as dist
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return t
    parts = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(parts, t.contiguous())
    return torch.cat(parts, 0)


def max_over_ranks(value: float, device=None) -> float:
    """The job-level time: the maximum of every rank's measurement."""
    import torch
    import torch.distributed as dist
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier() -> None:
    import torch.distributed as dist
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()


def finish() -> None:
    import torch.distributed as dist
    if dist.is_initialized():
        dist.destroy_process_group()
