"""Process / device bootstrap: one process per GPU, NCCL for device tensors and gloo for host
tensors on the same default group (`train_gpt.py:54-64`).  Without CUDA the group is gloo only,
which is how the CPU tests run the same trainer with world_size > 1."""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class DistEnv:
    rank: int
    world_size: int
    local_rank: int
    device: torch.device
    grad_accum_steps: int
    grad_scale: float
    master: bool
    cpu_group: object | None = None

    def barrier(self):
        if self.world_size > 1 or dist.is_initialized():
            dist.barrier()


def init_distributed(accum_base: int = 8, timeout_s: float = 600.0, force_cpu: bool = False) -> DistEnv:
    """Reads RANK / WORLD_SIZE / LOCAL_RANK (defaults: single process).  `accum_base` is the
    number of micro-batches one optimizer step is made of across all ranks: each rank runs
    `accum_base // world_size` of them so that 1, 2, 4 and 8 ranks give the same update."""
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    assert accum_base % world == 0, f"world_size must divide {accum_base}"
    use_cuda = torch.cuda.is_available() and not force_cpu
    device = torch.device("cuda", local) if use_cuda else torch.device("cpu")
    if use_cuda:
        torch.cuda.set_device(device)
    cpu_group = None
    if world > 1 or "MASTER_ADDR" in os.environ:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29500")
        if not dist.is_initialized():
            backend = "cuda:nccl,cpu:gloo" if use_cuda else "gloo"
            kw = dict(device_id=device) if use_cuda else {}
            dist.init_process_group(backend=backend, rank=rank, world_size=world,
                                    timeout=datetime.timedelta(seconds=timeout_s), **kw)
        dist.barrier()
    accum = accum_base // world
    return DistEnv(rank, world, local, device, accum, 1.0 / accum, rank == 0, cpu_group)


def shutdown():
    if dist.is_initialized():
        dist.destroy_process_group()


def broadcast_model(model: torch.nn.Module, src: int = 0):
    """Rank `src`'s parameters and persistent buffers become everyone's (`train_gpt.py:2255-2257`)."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return
    for p in model.parameters():
        dist.broadcast(p.detach(), src)
    for b in model.buffers():
        dist.broadcast(b, src)
