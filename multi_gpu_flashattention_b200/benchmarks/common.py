"""Shared plumbing of the benchmark entry points: process-group start-up from
torchrun-style environment variables, device binding, and max-over-ranks
reductions (every timing is taken on the device and reduced with MAX, as the
reference does with MPI_Reduce(MAX) per iteration)."""
from __future__ import annotations

import datetime
import os
import sys

import torch
import torch.distributed as dist

from ..utils.device import select_local_device


class Ctx:
    def __init__(self, rank, world, device, cpu_group):
        self.rank, self.world, self.device, self.cpu_group = rank, world, device, cpu_group

    def barrier(self):
        if self.world > 1:
            dist.barrier()

    def max(self, values):
        t = torch.tensor(values, dtype=torch.float64, device=self.device)
        if self.world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    def log(self, msg):
        print(msg, flush=True)

    def log0(self, msg):
        if self.rank == 0:
            print(msg, flush=True)

    def close(self):
        if self.world > 1 and dist.is_initialized():
            dist.barrier()
            dist.destroy_process_group()


def init(need_world_gt1: bool = False, timeout_s: int = 120) -> Ctx:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    dev = select_local_device(fallback_local_rank=rank)
    device = torch.device("cuda", dev)
    cpu_group = None
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=timeout_s),
                                device_id=device)
        cpu_group = dist.new_group(backend="gloo")
    elif need_world_gt1:
        print("Need at least 2 processes. Got 1.", flush=True)
        sys.exit(1)
    return Ctx(rank, world, device, cpu_group)


def exchange_handles(obj, world):
    handles = [None] * world
    dist.all_gather_object(handles, obj.ipc_handle())
    obj.connect(handles)
