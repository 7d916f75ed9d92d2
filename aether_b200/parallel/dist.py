"""Process-group bootstrap: one process per GPU (torchrun env contract).

Replaces the reference's single-process ``ncclCommInitAll`` over local devices
(runtime/src/nccl_real.rs:29-100) with the standard one-process-per-GPU model:
RANK / WORLD_SIZE / LOCAL_RANK / MASTER_ADDR / MASTER_PORT from the
environment, NCCL for CUDA and gloo for CPU, and a short timeout so ranks that
wait on a missing peer fail with an error instead of hanging.
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class DistInfo:
    rank: int = 0
    world: int = 1
    local_rank: int = 0
    device: torch.device = torch.device("cpu")
    backend: str = "none"

    @property
    def is_main(self) -> bool:
        return self.rank == 0


def env_world() -> int:
    return int(os.environ.get("WORLD_SIZE", "1"))


def init(backend: str | None = None, timeout_s: float = 300.0, device: str | None = None) -> DistInfo:
    rank = int(os.environ.get("RANK", "0"))
    world = env_world()
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    use_cuda = torch.cuda.is_available() and device != "cpu"
    dev = torch.device("cuda", local % max(1, torch.cuda.device_count())) if use_cuda else torch.device("cpu")
    if use_cuda:
        torch.cuda.set_device(dev)
    if world > 1 and not dist.is_initialized():
        be = backend or ("nccl" if use_cuda else "gloo")
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        kw = {}
        if be == "nccl":
            kw["device_id"] = dev
        dist.init_process_group(be, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s), **kw)
        return DistInfo(rank, world, local, dev, be)
    if dist.is_initialized():
        return DistInfo(dist.get_rank(), dist.get_world_size(), local, dev, dist.get_backend())
    return DistInfo(rank, 1, local, dev, "none")


def barrier() -> None:
    if dist.is_initialized():
        dist.barrier()


def all_reduce_max(x: float, device) -> float:
    if not dist.is_initialized():
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def shutdown() -> None:
    if dist.is_initialized():
        dist.destroy_process_group()
