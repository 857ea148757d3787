"""Fixed workload for profiling the attention kernels under ncu.

    python -m multi_gpu_flashattention_b200.benchmarks.profile_kernels [--seq 8192] [--heads 32]
        [--iters 3] [--no-causal] [--fwd-only]

Runs `iters` x (forward + backward) on seeded N(0,1)*0.5 bf16 inputs
[1, seq, heads, 128]; with ncu use `-s <2 * kernels per iteration> -c <kernels>`
to skip the warm-up iterations (forward = 1 kernel, backward = preprocess +
dK/dV + dQ; filter with -k). --fwd-only runs the forward alone."""
from __future__ import annotations

import argparse

import torch

from ..ops.flash import check_status, flash_attn_bwd, flash_attn_fwd


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--seq", type=int, default=8192)
    ap.add_argument("--heads", type=int, default=32)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--no-causal", action="store_true")
    ap.add_argument("--fwd-only", action="store_true")
    a = ap.parse_args()
    g = torch.Generator(device="cuda").manual_seed(0)
    mk = lambda: (torch.randn(1, a.seq, a.heads, 128, device="cuda", generator=g) * 0.5).bfloat16()
    q, k, v, do = mk(), mk(), mk(), mk()
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    for _ in range(a.iters):
        o, lse = flash_attn_fwd(q, k, v, causal=not a.no_causal, status=st)
        if not a.fwd_only:
            flash_attn_bwd(do, q, k, v, o, lse, causal=not a.no_causal, status=st)
    torch.cuda.synchronize()
    check_status(st)
    print("ok")


if __name__ == "__main__":
    main()
