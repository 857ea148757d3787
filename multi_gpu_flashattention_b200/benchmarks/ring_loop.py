"""Pure ring-exchange benchmark (no attention math).

    torchrun --nproc-per-node N -m multi_gpu_flashattention_b200.benchmarks.ring_loop \
        <kv_size_bytes> [warmup=10] [iters=100] [--backend p2p|ce|nccl|staged]

A kv_size_bytes buffer rotates around the ring for world-1 steps. Before timing,
one untimed pass checks that the first float received at step s equals
1000 * ((rank - s - 1) mod P) (the buffer is initialised to rank*1000 + i), like
ring/loop/ring_loop_nccl.cu:146-176. Timing is on the device (CUDA events
around the rotation), max over ranks per iteration, mean over iterations, and
rank 0 prints the reference's RESULT line
(ring/loop/ring_loop_nccl.cu:227-238) with payload = (world-1) * kv_size.

Backends
  p2p     all-SM push kernel into the right neighbour's slot over NVLink
          (peer stores + arrival/credit flags), one launch per step
  ce      copy engine (cudaMemcpyAsync into the peer mapping) + flag kernels
  nccl    NCCL send/recv per step (the reference's NCCL path)
  staged  device -> pinned host -> gloo send/recv -> device (the staged-MPI path)
--payload-tokens T switches to the bf16 K+V payload [T x 8 heads x 128 x 2]
filled with seeded uniform data (the 1 MB - 256 MB payload sweep); then the
precheck compares whole buffers with the expected owner's data.
"""
from __future__ import annotations

import argparse
import json
import time

import torch
import torch.distributed as dist

from .._ext import C
from . import common


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("kv_size", type=int, nargs="?", default=262144)
    ap.add_argument("warmup", type=int, nargs="?", default=10)
    ap.add_argument("iters", type=int, nargs="?", default=100)
    ap.add_argument("--backend", default="p2p", choices=["p2p", "ce", "nccl", "staged"])
    ap.add_argument("--payload-tokens", type=int, default=0)
    ap.add_argument("--kv-heads", type=int, default=8)
    ap.add_argument("--ctas", type=int, default=0, help="push kernel CTAs (default 2 per SM)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--json", action="store_true")
    return ap.parse_args()


def owner_data(args, owner, nbytes, device):
    """The buffer rank `owner` starts with."""
    if args.payload_tokens:
        g = torch.Generator(device=device).manual_seed(args.seed * 7919 + owner)
        return torch.rand(nbytes // 2, generator=g, device=device).to(torch.bfloat16).view(torch.uint8)
    n = nbytes // 4
    return (owner * 1000.0 + torch.arange(n, device=device, dtype=torch.float32)).view(torch.uint8)


def main():
    args = parse()
    ctx = common.init(need_world_gt1=True)
    P, r, dev = ctx.world, ctx.rank, ctx.device
    nbytes = args.payload_tokens * args.kv_heads * 128 * 2 * 2 if args.payload_tokens else args.kv_size
    if nbytes <= 0 or nbytes % 32 != 0 or args.warmup < 0 or args.iters <= 0:
        ctx.log0("Invalid arguments: kv_size must be a positive multiple of 32, warmup >= 0, iters > 0.")
        ctx.close()
        return 1
    right, left = (r + 1) % P, (r - 1) % P
    props = torch.cuda.get_device_properties(dev)
    ctx.log(f"[Rank {r}] GPU {dev.index}: {props.name} ({props.total_memory / 1e6:.0f} MB total)")
    ctx.log(f"[Rank {r}] KV shard: {nbytes} bytes ({nbytes / 1024:.1f} KB), neighbors: left={left} right={right}")
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    init = owner_data(args, r, nbytes, dev)
    expected_last = owner_data(args, (r + 1) % P, nbytes, dev)

    if args.backend in ("p2p", "ce"):
        n_ctas = args.ctas or 2 * props.multi_processor_count
        ex = C().RingExchange(r, P, dev.index, (nbytes + 4095) // 4096 * 4096, n_ctas)
        common.exchange_handles(ex, P)
        torch.cuda.synchronize()
        ctx.barrier()

        def reset():
            ex.slot(0)[:nbytes].copy_(init)

        def rotate():
            ex.rotate(nbytes, args.backend, status, 2_000_000_000)

        def received():
            return ex.slot((P - 1) & 1)[:nbytes]

        def precheck():
            reset()
            torch.cuda.synchronize()
            ctx.barrier()
            for t in range(P - 1):
                ex.step(t, nbytes, args.backend, status, 2_000_000_000)
                torch.cuda.synchronize()
                ctx.barrier()
                got = ex.slot((t + 1) & 1)[:nbytes]
                check(got, (r - t - 1) % P, t)
            ex.release(P - 1, args.backend, status, 2_000_000_000)
            torch.cuda.synchronize()
            common_c = int(status.item())
            if common_c:
                raise RuntimeError(f"[Rank {r}] transport status {common_c:#x}")
    else:
        cur = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        nxt = torch.empty_like(cur)
        bufs = {"cur": cur, "nxt": nxt}
        if args.backend == "staged":
            h_send = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
            h_recv = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)

        def reset():
            bufs["cur"], bufs["nxt"] = cur, nxt
            cur.copy_(init)

        def one_step():
            c, n = bufs["cur"], bufs["nxt"]
            if args.backend == "nccl":
                reqs = dist.batch_isend_irecv([dist.P2POp(dist.isend, c, right),
                                               dist.P2POp(dist.irecv, n, left)])
                for q in reqs:
                    q.wait()
            else:
                h_send.copy_(c)
                reqs = [dist.isend(h_send, right, group=ctx.cpu_group),
                        dist.irecv(h_recv, left, group=ctx.cpu_group)]
                for q in reqs:
                    q.wait()
                n.copy_(h_recv, non_blocking=True)
            bufs["cur"], bufs["nxt"] = n, c

        def rotate():
            for _ in range(P - 1):
                one_step()

        def received():
            return bufs["cur"]

        def precheck():
            reset()
            torch.cuda.synchronize()
            ctx.barrier()
            for t in range(P - 1):
                one_step()
                torch.cuda.synchronize()
                check(bufs["cur"], (r - t - 1) % P, t)

    def check(got, owner, step):
        if args.payload_tokens:
            ok = torch.equal(got, owner_data(args, owner, nbytes, dev))
            first, exp = "buffer", f"owner {owner} data"
        else:
            first = float(got[:4].view(torch.float32).item())
            exp = owner * 1000.0
            ok = first == exp
        if not ok:
            raise RuntimeError(f"[Rank {r}] {args.backend} precheck mismatch at step {step}: "
                               f"got {first} expect {exp}")

    precheck()
    ctx.barrier()

    sum_comm = sum_total = 0.0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for rep in range(args.warmup + args.iters):
        reset()
        torch.cuda.synchronize()
        ctx.barrier()
        t0 = time.perf_counter()
        e0.record()
        rotate()
        e1.record()
        torch.cuda.synchronize()
        wall = (time.perf_counter() - t0) * 1e3
        comm_ms, total_ms = ctx.max([e0.elapsed_time(e1), wall])
        if rep >= args.warmup:
            sum_comm += comm_ms
            sum_total += total_ms
    if int(status.item()):
        raise RuntimeError(f"[Rank {r}] transport status {int(status.item()):#x}")
    if not torch.equal(received(), expected_last):
        raise RuntimeError(f"[Rank {r}] final buffer is not owner {(r + 1) % P}'s data")

    if r == 0:
        avg_c, avg_t = sum_comm / args.iters, sum_total / args.iters
        payload = (P - 1) * nbytes
        b = args.backend
        print(f"RESULT backend={b} bytes={nbytes} ranks={P} warmup={args.warmup} iters={args.iters} "
              f"avg_{b}_ms={avg_c:.3f} avg_total_ms={avg_t:.3f} "
              f"total_GBps={payload / (avg_t / 1e3) / 1e9:.3f} {b}_GBps={payload / (avg_c / 1e3) / 1e9:.3f}",
              flush=True)
        if args.json:
            gbps = payload / (avg_c / 1e3) / 1e9
            print(json.dumps({"backend": b, "bytes": nbytes, "ranks": P, "avg_ms": avg_c,
                              "per_direction_GBps": gbps,
                              "link_fraction": gbps / 770.0,  # of the measured peer copy
                              "payload_tokens": args.payload_tokens}), flush=True)
    ctx.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
