"""Fixed-setting single-GPU attention baseline (the reference's
tests/single_gpu_baseline.py): causal fp16, batch 2, 8 heads, head_dim 64,
sequence lengths 512 / 1024 / 2048, 3 warm-up calls and the mean of 10 timed
calls. The reference times with the host clock; here the 10 calls are
bracketed by CUDA events on the launching stream.

    python -m multi_gpu_flashattention_b200.benchmarks.single_gpu_baseline [--device 0]
"""
from __future__ import annotations

import argparse

import torch

from ..ops.flash import flash_attn_fwd


def run_test(seq_len: int, device: int = 0) -> float:
    dev = torch.device("cuda", device)
    torch.cuda.set_device(dev)
    batch_size, num_heads, head_dim = 2, 8, 64
    q, k, v = (torch.randn(batch_size, seq_len, num_heads, head_dim, dtype=torch.float16,
                           device=dev) for _ in range(3))
    for _ in range(3):
        flash_attn_fwd(q, k, v, causal=True)
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(10):
        flash_attn_fwd(q, k, v, causal=True)
    end.record()
    end.synchronize()
    ms = start.elapsed_time(end) / 10
    print(f"seq_len={seq_len}, time={ms:.2f} ms", flush=True)
    return ms / 1e3


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--device", type=int, default=0)
    a = ap.parse_args()
    print("=== Single-GPU FlashAttention baseline ===")
    for seq_len in (512, 1024, 2048):
        run_test(seq_len, a.device)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
