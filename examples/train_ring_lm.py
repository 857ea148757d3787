"""Train a small decoder-only language model with context-parallel ring
attention: every rank holds one token shard of each sequence, attention runs
around the ring, everything else is per token, and the replicated parameters'
gradients are summed over the ranks.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 examples/train_ring_lm.py \
        [--seq 65536] [--layers 4] [--d-model 1024] [--heads 8] [--kv-heads 2] \
        [--head-dim 128] [--steps 50] [--layout zigzag] [--backend fused]

On GPUs (NCCL) the model runs in bf16 with the sm_100a kernels; without a GPU
the ranks use gloo and the fp32 `torch` backend (use small sizes). The data is
synthetic: a fixed seeded batch of a repeating token pattern with noise, which
a working model learns quickly, so the printed loss should fall well below
ln(vocab). Rank 0 prints one line per step and a final JSON summary.

--save PATH writes a checkpoint (model and optimizer state, step count) at the
end; --resume PATH starts from one. Parameters are replicated, so rank 0 writes
and every rank reads the same file; a resumed run continues exactly where the
saved one stopped (same losses as an uninterrupted run on the same ranks).
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import sys
import time

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from multi_gpu_flashattention_b200.models import RingTransformerLM, shard_targets  # noqa: E402
from multi_gpu_flashattention_b200.parallel.layouts import RingLayout  # noqa: E402


def parse(argv=None):
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--seq", type=int, default=65536)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--vocab", type=int, default=512)
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--d-model", type=int, default=1024)
    ap.add_argument("--heads", type=int, default=8)
    ap.add_argument("--kv-heads", type=int, default=2)
    ap.add_argument("--head-dim", type=int, default=128)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--lr", type=float, default=3e-4)
    ap.add_argument("--layout", default="zigzag", choices=["contiguous", "zigzag", "striped"])
    ap.add_argument("--backend", default=None,
                    help="ring backend (default: fused on GPUs, torch without)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--save", default=None, help="checkpoint written at the end")
    ap.add_argument("--resume", default=None, help="checkpoint to start from")
    return ap.parse_args(argv)


def synthetic_batch(batch: int, seq: int, vocab: int, seed: int) -> torch.Tensor:
    """A repeating pattern of period 97 with 10 % random tokens."""
    g = torch.Generator().manual_seed(seed)
    base = (torch.arange(seq) * 7 % 97) % vocab
    ids = base.repeat(batch, 1)
    noise = torch.rand(batch, seq, generator=g) < 0.1
    return torch.where(noise, torch.randint(0, vocab, (batch, seq), generator=g), ids)


def main(argv=None):
    a = parse(argv)
    use_cuda = torch.cuda.is_available()
    if "RANK" in os.environ:
        if use_cuda:
            torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("nccl" if use_cuda else "gloo",
                                timeout=datetime.timedelta(seconds=300))
    rank = dist.get_rank() if dist.is_initialized() else 0
    world = dist.get_world_size() if dist.is_initialized() else 1
    dev = torch.device("cuda", torch.cuda.current_device()) if use_cuda else torch.device("cpu")
    dtype = torch.bfloat16 if use_cuda else torch.float32
    backend = a.backend or ("fused" if use_cuda else "torch")

    torch.manual_seed(a.seed)  # identical initial parameters on every rank
    model = RingTransformerLM(a.vocab, a.d_model, a.layers, a.heads, a.kv_heads,
                              a.head_dim).to(dev, dtype)
    opt = torch.optim.AdamW(model.parameters(), lr=a.lr, weight_decay=0.0)
    lay = RingLayout(a.layout, a.seq, world, mask="causal")
    ids = synthetic_batch(a.batch, a.seq, a.vocab, a.seed)
    local_ids = lay.shard(ids, rank).to(dev)
    targets = shard_targets(ids, lay, rank).to(dev)

    start = 0
    if a.resume:
        ck = torch.load(a.resume, map_location=dev, weights_only=True)
        model.load_state_dict(ck["model"])
        opt.load_state_dict(ck["optimizer"])
        start = int(ck["step"])
    losses = []
    t0 = time.time()
    for step in range(start, start + a.steps):
        opt.zero_grad(set_to_none=True)
        loss = model.loss(local_ids, targets, lay, rank, backend=backend)
        loss.backward()
        total = loss.detach().float().clone()
        if world > 1:
            for p in model.parameters():
                if p.grad is not None:
                    dist.all_reduce(p.grad)
            dist.all_reduce(total)
        torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        opt.step()
        losses.append(total.item())
        if rank == 0:
            print(f"step {step:4d}  loss {losses[-1]:.4f}", flush=True)
    if use_cuda:
        torch.cuda.synchronize()
    wall = time.time() - t0
    if a.save and rank == 0:
        torch.save({"model": model.state_dict(), "optimizer": opt.state_dict(),
                    "step": start + a.steps}, a.save)
    if rank == 0:
        print(json.dumps({"world": world, "seq": a.seq, "layout": a.layout, "backend": backend,
                          "dtype": str(dtype).replace("torch.", ""), "steps": a.steps,
                          "first_loss": losses[0], "last_loss": losses[-1],
                          "uniform_loss": math.log(a.vocab),
                          "tokens_per_s": a.batch * a.seq * a.steps / wall}), flush=True)
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
