"""Multi-GPU plumbing: one process per GPU, (batch x head) units sharded with no hot-path collective.

Every (batch, head) pair is an independent VMonarch problem (the R step, the L step and the exact
recompute never mix heads; reference vmonarch.py:41-69 operates per (b, h) slice), so ranks split
the units contiguously and run with no communication. torch.distributed (NCCL on GPUs, gloo on
CPU) is used only for barriers, the max-over-ranks timing reduction and an optional gather of the
outputs for verification, always outside the timed region.
"""
from __future__ import annotations

import os
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class RankInfo:
    rank: int
    world: int
    local_rank: int


def env_rank() -> RankInfo:
    return RankInfo(int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
                    int(os.environ.get("LOCAL_RANK", 0)))


def unit_range(n_units: int, rank: int, world: int) -> range:
    """Contiguous block of units for `rank` (sizes differ by at most one)."""
    base, extra = divmod(n_units, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def init(backend: str, timeout_s: float = 120.0) -> RankInfo:
    """Initialise the default process group from the torchrun environment (no-op when world == 1)."""
    info = env_rank()
    if info.world > 1 and not dist.is_initialized():
        import datetime
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        kw = {}
        if backend == "nccl":
            kw["device_id"] = torch.device("cuda", info.local_rank)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return info


def barrier() -> None:
    if dist.is_initialized():
        dist.barrier()


def max_over_ranks(x: float, device: torch.device) -> float:
    if not dist.is_initialized():
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_units(local: torch.Tensor, n_units: int, world: int) -> torch.Tensor:
    """All-gather per-rank unit blocks (dim 0) into the full (n_units, ...) tensor; verification only.
    Blocks are padded to the largest block so every rank sends the same size."""
    if world == 1 or not dist.is_initialized():
        return local
    biggest = -(-n_units // world)
    pad = torch.zeros((biggest, *local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    bufs = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(bufs, pad)
    return torch.cat([bufs[r][: len(unit_range(n_units, r, world))] for r in range(world)], 0)
