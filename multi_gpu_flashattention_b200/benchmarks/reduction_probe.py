"""Throughput of fp32 vector reductions in the pattern a dQ-fused backward kernel
would produce (one B200): every key tile adds a 128 x D fp32 tile into the dQ
rows of each query tile it sees.

    python -m multi_gpu_flashattention_b200.benchmarks.reduction_probe \
        [--seq 8192] [--heads 32] [--head-dim 128] [--causal|--no-causal] [--reps 5]

Prints the time of one full accumulation (what the fused kernel would add per
backward pass), the reduction payload and its rate. Compare the time with the
separate dQ kernel's (`single_gpu_shapes --backward` and the ncu summary)."""
from __future__ import annotations

import argparse

import torch

from .._ext import C


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--seq", type=int, default=8192)
    ap.add_argument("--heads", type=int, default=32)
    ap.add_argument("--head-dim", type=int, default=128)
    ap.add_argument("--causal", action=argparse.BooleanOptionalAction, default=True)
    ap.add_argument("--reps", type=int, default=5)
    a = ap.parse_args()
    tiles = (a.seq + 127) // 128
    dq = torch.zeros(a.heads, tiles * 128, a.head_dim, device="cuda")
    for _ in range(2):  # warm-up
        C().red_probe(dq, tiles, a.causal)
    torch.cuda.synchronize()
    times = []
    for _ in range(a.reps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        C().red_probe(dq, tiles, a.causal)
        e.record()
        e.synchronize()
        times.append(s.elapsed_time(e))
    pairs = tiles * (tiles + 1) // 2 if a.causal else tiles * tiles
    payload = pairs * a.heads * 128 * a.head_dim * 4
    ms = sum(times) / len(times)
    print(f"seq={a.seq} heads={a.heads} d={a.head_dim} causal={a.causal}: {ms:.3f} ms for "
          f"{payload / 1e9:.2f} GB of fp32 reductions = {payload / (ms * 1e-3) / 1e12:.2f} TB/s",
          flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
