"""Early transport probes of the reference (ring/ring_test.c, ring/ring_cuda.cu).

    torchrun --nproc-per-node N -m multi_gpu_flashattention_b200.benchmarks.probes ring_test
    torchrun --nproc-per-node 2 -m multi_gpu_flashattention_b200.benchmarks.probes ring_cuda [--cpu]

ring_test: every rank sends 4 doubles (100 r + i) to its right neighbour and
  receives its left neighbour's over the host transport (gloo), printing the
  neighbours, the time and the received values (ring_test.c:26-57).
ring_cuda: exactly 2 ranks; one staged step of a 256 KB fp32 shard
  (128 x 8 x 64 floats, value 1000 r + i): device -> host, host send/recv,
  host -> device, then the first 4 received values (ring_cuda.cu:22-80).
  --cpu keeps the "device" buffers in host memory (no GPU needed).
The host-transport times are host-clock times between barriers, as in the
reference; nothing here is a device benchmark.
"""
from __future__ import annotations

import argparse
import datetime
import os
import time

import torch
import torch.distributed as dist


def _init(backend):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if not dist.is_initialized():
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
    return rank, world


def ring_test(rank, world, log=print):
    right, left = (rank + 1) % world, (rank - 1) % world
    log(f"[Rank {rank}] neighbors: left={left}, right={right}")
    send = torch.tensor([rank * 100.0 + i for i in range(4)], dtype=torch.float64)
    recv = torch.empty(4, dtype=torch.float64)
    t0 = time.perf_counter()
    reqs = [dist.isend(send, right), dist.irecv(recv, left)]
    for r in reqs:
        r.wait()
    t1 = time.perf_counter()
    log(f"[Rank {rank}] sent to {right}, received from {left} in {(t1 - t0) * 1e3:.3f} ms")
    vals = ", ".join(f"{x:.0f}" for x in recv.tolist())
    log(f"[Rank {rank}] recv_buf = [{vals}]")
    return recv


def ring_cuda(rank, world, device, log=print, cpu_group=None):
    right, left = (rank + 1) % world, (rank - 1) % world
    if device.type == "cuda":
        props = torch.cuda.get_device_properties(device)
        log(f"[Rank {rank}] bound to GPU {device.index}: {props.name} "
            f"({props.total_memory / 1e6:.0f} MB free)")
    n = 128 * 8 * 64
    kv_bytes = n * 4
    log(f"[Rank {rank}] KV shard size = {kv_bytes} bytes ({kv_bytes / 1024.0:.1f} KB)")
    d_send = (torch.full((n,), rank * 1000.0) + torch.arange(n, dtype=torch.float32)).to(device)
    d_recv = torch.empty(n, device=device)
    h_send, h_recv = torch.empty(n), torch.empty(n)
    dist.barrier()
    t0 = time.perf_counter()
    h_send.copy_(d_send)
    reqs = [dist.isend(h_send, right, group=cpu_group), dist.irecv(h_recv, left, group=cpu_group)]
    for r in reqs:
        r.wait()
    d_recv.copy_(h_recv)
    if device.type == "cuda":
        torch.cuda.synchronize(device)
    dist.barrier()
    t1 = time.perf_counter()
    log(f"[Rank {rank}] ring step done in {(t1 - t0) * 1e3:.3f} ms (GPU->host->MPI->host->GPU)")
    first = d_recv[:4].cpu().tolist()
    log(f"[Rank {rank}] received from rank {left}: first 4 values = "
        f"[{', '.join(f'{x:.0f}' for x in first)}]")
    return d_recv.cpu()


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("probe", choices=["ring_test", "ring_cuda"])
    ap.add_argument("--cpu", action="store_true", help="ring_cuda with host buffers")
    a = ap.parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if a.probe == "ring_test":
        if world < 2:
            print(f"Need at least 2 processes. Got {world}.")
            return 1
        rank, world = _init("gloo")
        ring_test(rank, world, log=lambda m: print(m, flush=True))
    else:
        if world != 2:
            if int(os.environ.get("RANK", "0")) == 0:
                print("This test expects exactly 2 processes.")
            return 1
        if a.cpu:
            rank, world = _init("gloo")
            device, group = torch.device("cpu"), None
        else:
            from ..utils.device import select_local_device
            rank = int(os.environ.get("RANK", "0"))
            device = torch.device("cuda", select_local_device(fallback_local_rank=rank))
            torch.cuda.set_device(device)
            rank, world = _init("nccl")
            group = dist.new_group(backend="gloo")
        ring_cuda(rank, world, device, log=lambda m: print(m, flush=True), cpu_group=group)
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
