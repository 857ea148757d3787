"""Ring attention in a few lines: shard a sequence over the ranks with a
layout, run `ring_attention` (differentiable), gather the shards back and
compare with attention over the whole sequence on one device.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 examples/ring_attention_quickstart.py \
        [--seq 32768] [--heads 8] [--kv-heads 2] [--head-dim 128] [--layout zigzag]

On GPUs (NCCL) the inputs are bf16 and the fused sm_100a ring runs; without a GPU
the ranks use gloo and the fp32 `torch` backend (use small sizes, e.g. --seq 512
--head-dim 32). Rank 0 prints the largest difference from the single-device
result for the output and for the query gradient.
"""
from __future__ import annotations

import argparse
import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import multi_gpu_flashattention_b200 as mgfa  # noqa: E402
from multi_gpu_flashattention_b200.ops.reference import attention_ref  # noqa: E402


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--seq", type=int, default=32768)
    ap.add_argument("--heads", type=int, default=8)
    ap.add_argument("--kv-heads", type=int, default=2)
    ap.add_argument("--head-dim", type=int, default=128)
    ap.add_argument("--layout", default="zigzag", choices=["contiguous", "zigzag", "striped"])
    a = ap.parse_args(argv)

    cuda = torch.cuda.is_available()
    if "RANK" in os.environ:
        if cuda:
            torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("nccl" if cuda else "gloo", timeout=datetime.timedelta(seconds=300))
    rank = dist.get_rank() if dist.is_initialized() else 0
    world = dist.get_world_size() if dist.is_initialized() else 1
    dev = torch.device("cuda", torch.cuda.current_device()) if cuda else torch.device("cpu")
    dtype = torch.bfloat16 if cuda else torch.float32
    backend = None if cuda else "torch"

    # the full inputs, identical on every rank (seeded)
    g = torch.Generator().manual_seed(0)
    shape = lambda h: (1, a.seq, h, a.head_dim)  # noqa: E731
    q_full = torch.randn(shape(a.heads), generator=g) * 0.5
    k_full = torch.randn(shape(a.kv_heads), generator=g) * 0.5
    v_full = torch.randn(shape(a.kv_heads), generator=g) * 0.5

    # this rank's shard under the layout, then the ring
    lay = mgfa.RingLayout(a.layout, a.seq, world)
    q, k, v = (lay.shard(x, rank).to(dev, dtype) for x in (q_full, k_full, v_full))
    q.requires_grad_()
    out = mgfa.ring_attention(q, k, v, causal=True, layout=lay, backend=backend)
    out.float().square().sum().backward()

    # gather every rank's shard (and dq) and restore the sequence order
    def gather(t):
        if world == 1:
            return [t]
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t.contiguous())
        return parts
    out_all = lay.unshard([p.float().cpu() for p in gather(out.detach())])
    dq_all = lay.unshard([p.float().cpu() for p in gather(q.grad)])

    if rank == 0:
        qr = q_full.to(dtype).float().requires_grad_()
        ref, _ = attention_ref(qr, k_full.to(dtype).float(), v_full.to(dtype).float(), causal=True)
        ref.square().sum().backward()
        print(f"world={world} seq={a.seq} layout={a.layout} dtype={str(dtype)[6:]} "
              f"max|out-ref|={(out_all - ref.detach()).abs().max().item():.3e} "
              f"max|dq-ref|={(dq_all - qr.grad).abs().max().item():.3e}", flush=True)
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
