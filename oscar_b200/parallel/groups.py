"""Tensor/data-parallel process groups over ``torch.distributed`` (NCCL on GPUs, gloo on CPU).

One process per GPU.  ``TPGroup`` wraps the tensor-parallel group and its collectives;
the plain NCCL collectives here are the *baseline* communication path.  The fused
GEMM + collective kernels live in :mod:`oscar_b200.parallel.fused` and use the
symmetric-memory buffers this module can allocate.
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class TPGroup:
    rank: int = 0
    world: int = 1
    group: object = None
    dp_rank: int = 0
    dp_world: int = 1

    @property
    def enabled(self) -> bool:
        return self.world > 1

    def all_reduce_(self, t: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            dist.all_reduce(t, group=self.group)
        return t

    def all_gather(self, t: torch.Tensor) -> torch.Tensor:
        """Concatenate along dim 0 in rank order."""
        if self.world == 1:
            return t
        out = torch.empty((self.world * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(out, t.contiguous(), group=self.group)
        return out

    def barrier(self):
        if self.world > 1:
            dist.barrier(group=self.group)

    def shard(self, n: int) -> tuple[int, int]:
        """Contiguous [begin, end) of ``n`` items owned by this rank (n divisible by world)."""
        if n % self.world:
            raise ValueError(f"{n} is not divisible by tensor-parallel size {self.world}")
        per = n // self.world
        return self.rank * per, (self.rank + 1) * per


def init_distributed(backend: str | None = None, timeout_s: float = 300.0) -> tuple[int, int, int]:
    """Initialise the default process group from torchrun env vars; returns (rank, world, local_rank)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        kwargs = dict(backend=backend, rank=rank, world_size=world,
                      timeout=datetime.timedelta(seconds=timeout_s))
        if backend == "nccl":
            torch.cuda.set_device(local)
            kwargs["device_id"] = torch.device("cuda", local)
        dist.init_process_group(**kwargs)
    return rank, world, local


def make_groups(tp: int, dp: int = 1) -> TPGroup:
    """Split the world into ``dp`` replicas of ``tp`` consecutive ranks."""
    if not dist.is_initialized():
        if tp * dp != 1:
            raise RuntimeError("tp*dp > 1 requires an initialised process group")
        return TPGroup()
    world = dist.get_world_size()
    rank = dist.get_rank()
    if tp * dp != world:
        raise ValueError(f"tp({tp}) * dp({dp}) != world size {world}")
    my = None
    for d in range(dp):
        ranks = list(range(d * tp, (d + 1) * tp))
        g = dist.new_group(ranks) if tp < world else dist.group.WORLD
        if rank in ranks:
            my = g
    return TPGroup(rank=rank % tp, world=tp, group=my, dp_rank=rank // tp, dp_world=dp)
