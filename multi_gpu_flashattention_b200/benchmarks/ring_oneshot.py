"""One-shot legacy ring attention: the reference's ring/attention/gpu programs
(ring_attention_{staged,cuda_aware,nccl}_gpu.cu) and its CPU-compute rings
(ring/attention/ring_attention_{staged,cuda_aware}.cu) as one driver.

    torchrun --nproc-per-node N -m multi_gpu_flashattention_b200.benchmarks.ring_oneshot \
        [--attention gpu|cpu] [--backend staged|nccl|p2p] [--seq 1024] [--dim 64] [--cpu]

One pass, no warm-up (as the reference): rank r holds Q and K == V of tokens
[r*seq, (r+1)*seq) with the reference's formulas (kv[i] = 1000 r + i,
q[i] = (500 r + 0.01 (i mod dim)) * 0.001, no softmax scale;
gpu/ring_attention_staged_gpu.cu:240-262), the shard moves around the ring
P-1 times, every rank prints the per-step phase times in the reference's
format and always dumps ring_output_rank<r>.bin (fp32 [seq, dim]), which
`verify_full <dir> N seq*dim*4` checks.

--attention gpu: fp32 partial attention + merge kernels (legacy_fp32.cu).
--attention cpu: the C++ host attention (csrc/host/cpu_attention.cpp); the KV
  shard still travels through device buffers, as in the reference.
--backend staged: D2H, host send/recv (gloo), H2D. nccl: NCCL send/recv on the
  device buffers (the role of the reference's CUDA-aware MPI). p2p: the
  RingExchange push kernel over NVLink peer memory.
--cpu: run on host memory only (gloo, --attention cpu --backend staged), for
  machines without a GPU.

Phase times of device work come from CUDA events on the launching stream; the
host attention and merge are timed with the host clock.
"""
from __future__ import annotations

import argparse
import datetime
import os
import time

import torch
import torch.distributed as dist

from .._ext import C, sched as _sched
from . import common

LABEL = {"staged": "MPI", "nccl": "NCCL", "p2p": "P2P"}


def parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--attention", default="gpu", choices=["gpu", "cpu"])
    ap.add_argument("--backend", default="staged", choices=["staged", "nccl", "p2p"])
    ap.add_argument("--seq", type=int, default=128 * 8,
                    help="tokens per rank (reference: 128 per block x 8)")
    ap.add_argument("--dim", type=int, default=64)
    ap.add_argument("--cpu", action="store_true", help="host memory only (gloo)")
    ap.add_argument("--out-dir", default=".")
    return ap.parse_args(argv)


def legacy_inputs(rank: int, seq: int, dim: int):
    """fp32 host tensors q, kv [seq, dim] with the reference's formulas."""
    n = seq * dim
    kv = torch.full((n,), rank * 1000.0) + torch.arange(n, dtype=torch.float32)
    q = (torch.full((n,), rank * 500.0) + (torch.arange(n) % dim).to(torch.float32)
         * torch.tensor(0.01)) * torch.tensor(0.001)
    return q.view(seq, dim).contiguous(), kv.view(seq, dim).contiguous()


class _Clock:
    """Phase timer: CUDA events on a GPU, the host clock otherwise."""

    def __init__(self, cuda: bool):
        self.cuda = cuda

    def mark(self):
        if self.cuda:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            return e
        return time.perf_counter()

    def ms(self, a, b):
        if self.cuda:
            b.synchronize()
            return a.elapsed_time(b)
        return (b - a) * 1e3


def run(ctx, args):
    P, r = ctx.world, ctx.rank
    right, left = (r + 1) % P, (r - 1) % P
    seq, dim = args.seq, args.dim
    dev = ctx.device
    cuda = dev.type == "cuda"
    if cuda:
        props = torch.cuda.get_device_properties(dev)
        ctx.log(f"[Rank {r}] GPU {dev.index}: {props.name} ({props.total_memory / 1e6:.0f} MB total)")
    kv_bytes = seq * dim * 4
    ctx.log(f"[Rank {r}] seq_q={seq}, seq_k={seq}, dim={dim}, KV shard={kv_bytes / 1024.0:.1f} KB")

    q_h, kv_h = legacy_inputs(r, seq, dim)
    S = _sched()
    clk = _Clock(cuda)
    pin = dict(pin_memory=True) if cuda else {}
    h_send = torch.empty(seq, dim, **pin)
    h_recv = torch.empty(seq, dim, **pin)

    # running state
    if args.attention == "cpu":
        m_run = torch.full((seq,), -torch.finfo(torch.float32).max)
        l_run = torch.zeros(seq)
        acc_run = torch.zeros(seq, dim)
        m_loc, l_loc, acc_loc = torch.empty(seq), torch.empty(seq), torch.empty(seq, dim)
        q_cpu = q_h
    else:
        q_dev = q_h.to(dev).view(seq, 1, dim)
        m_run = torch.empty(1, seq, device=dev)
        l_run = torch.empty(1, seq, device=dev)
        acc_run = torch.empty(seq, 1, dim, device=dev)
        m_loc, l_loc = torch.empty(1, seq, device=dev), torch.empty(1, seq, device=dev)
        acc_loc = torch.empty(seq, 1, dim, device=dev)

    def attend(kv_buf, first):
        """Partial attention on one KV shard merged into the running state;
        returns (attn_ms, merge_ms)."""
        if args.attention == "cpu":
            t0 = time.perf_counter()
            kvn = kv_buf.numpy()
            S.cpu_attention_partial(q_cpu.numpy(), kvn, kvn, seq, seq, dim, 1.0,
                                    acc_loc.numpy(), m_loc.numpy(), l_loc.numpy())
            t1 = time.perf_counter()
            S.cpu_merge_online_softmax(m_run.numpy(), l_run.numpy(), acc_run.numpy(),
                                       m_loc.numpy(), l_loc.numpy(), acc_loc.numpy(), seq, dim)
            t2 = time.perf_counter()
            return (t1 - t0) * 1e3, (t2 - t1) * 1e3
        kvd = kv_buf.view(seq, 1, dim)
        e0 = clk.mark()
        Cm = C()
        Cm.legacy_partial(q_dev, kvd, kvd, 1.0, None, None, False, acc_loc, m_loc, l_loc, False)
        e1 = clk.mark()
        if first:
            m_run.copy_(m_loc)
            l_run.copy_(l_loc)
            acc_run.copy_(acc_loc)
        else:
            Cm.legacy_merge(m_run, l_run, acc_run, m_loc, l_loc, acc_loc)
        e2 = clk.mark()
        return clk.ms(e0, e1), clk.ms(e1, e2)

    # KV buffers (device, or host with --cpu)
    ex = None
    status = torch.zeros(1, dtype=torch.int32, device=dev) if cuda else None
    if args.backend == "p2p":
        ex = C().RingExchange(r, P, dev.index, (kv_bytes + 4095) // 4096 * 4096,
                              2 * torch.cuda.get_device_properties(dev).multi_processor_count)
        common.exchange_handles(ex, P)
        ex.slot(0)[:kv_bytes].copy_(kv_h.view(-1).view(torch.uint8).to(dev))
        bufs = None
    else:
        bufs = [kv_h.to(dev), torch.empty(seq, dim, device=dev)]
    if args.backend == "nccl":
        # NCCL connects a peer pair on its first send/recv; do that untimed so the
        # step time is the transfer (the reference creates its communicator
        # before timing, too)
        warm = [torch.zeros(1, device=dev), torch.empty(1, device=dev)]
        for w in dist.batch_isend_irecv([dist.P2POp(dist.isend, warm[0], right),
                                         dist.P2POp(dist.irecv, warm[1], left)]):
            w.wait()
    if cuda:
        torch.cuda.synchronize()
    ctx.barrier()

    def slot_view(i):
        return ex.slot(i)[:kv_bytes].view(torch.float32).view(seq, dim)

    t_start = clk.mark()
    # step 0: own shard
    own = slot_view(0) if ex is not None else bufs[0]
    if args.attention == "cpu":
        attend(kv_h, True)
    else:
        attend(own, True)
    ctx.log(f"[Rank {r}] step 0: attention on own KV")
    cur = 0
    for step in range(P - 1):
        src = (r - step - 1) % P
        t1 = clk.mark()
        parts = []
        if args.backend == "staged":
            h_send.copy_(bufs[cur])
            t2 = clk.mark()
            reqs = [dist.isend(h_send, right, group=ctx.cpu_group),
                    dist.irecv(h_recv, left, group=ctx.cpu_group)]
            for q_ in reqs:
                q_.wait()
            t3 = clk.mark()
            bufs[cur ^ 1].copy_(h_recv)
            t4 = clk.mark()
            parts = [("D2H", clk.ms(t1, t2)), ("MPI", clk.ms(t2, t3)), ("H2D", clk.ms(t3, t4))]
            recv_buf, host_copy = bufs[cur ^ 1], h_recv
        else:
            if args.backend == "nccl":
                ops = [dist.P2POp(dist.isend, bufs[cur], right),
                       dist.P2POp(dist.irecv, bufs[cur ^ 1], left)]
                for w in dist.batch_isend_irecv(ops):
                    w.wait()
                recv_buf = bufs[cur ^ 1]
            else:
                ex.step(step, kv_bytes, "p2p", status, 2_000_000_000)
                # the left neighbour's push into our slot may still be in flight
                ex.wait_received(step, "p2p", status, 2_000_000_000)
                recv_buf = slot_view((step + 1) & 1)
            t2 = clk.mark()
            parts = [(LABEL[args.backend], clk.ms(t1, t2))]
            host_copy = None
            if args.attention == "cpu":
                # the host attention needs the shard in host memory
                h_recv.copy_(recv_buf)
                t3 = clk.mark()
                parts.append(("D2H", clk.ms(t2, t3)))
                host_copy = h_recv
        a_ms, m_ms = attend(host_copy if args.attention == "cpu" else recv_buf, False)
        total = sum(v for _, v in parts) + a_ms + m_ms
        body = " ".join(f"{k}={v:.3f}" for k, v in parts)
        ctx.log(f"[Rank {r}] step {step + 1}: KV from rank {src} | {body} "
                f"attn={a_ms:.3f} merge={m_ms:.3f} total={total:.3f} ms")
        cur ^= 1
    if ex is not None:
        ex.release(P - 1, "p2p", status, 2_000_000_000)
    # final normalisation
    if args.attention == "cpu":
        S.cpu_normalize(acc_run.numpy(), l_run.numpy(), seq, dim)
        out = acc_run
    else:
        out = torch.empty_like(acc_run)
        C().legacy_normalize(acc_run, l_run, out)
        out = out.view(seq, dim).cpu()
    ctx.barrier()
    t_end = clk.mark()
    ctx.log(f"[Rank {r}] ring attention done in {clk.ms(t_start, t_end):.3f} ms")
    if status is not None and int(status.item()):
        raise RuntimeError(f"[Rank {r}] transport status {int(status.item()):#x}")
    fname = os.path.join(args.out_dir, f"ring_output_rank{r}.bin")
    out.contiguous().numpy().astype("<f4").tofile(fname)
    ctx.log(f"[Rank {r}] output dumped to {os.path.basename(fname)}")
    return out


def main(argv=None):
    args = parse(argv)
    if args.attention == "gpu" and args.dim != 64:
        print("--attention gpu runs the fp32 kernels with dim 64")
        return 1
    if args.cpu:
        if args.attention != "cpu" or args.backend != "staged":
            print("--cpu runs --attention cpu --backend staged")
            return 1
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        if world < 2:
            print(f"Need at least 2 processes. Got {world}.", flush=True)
            return 1
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
        ctx = common.Ctx(rank, world, torch.device("cpu"), None)
    else:
        ctx = common.init(need_world_gt1=True)
    run(ctx, args)
    ctx.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
