"""Single-GPU attention timing over shapes (the reference's
tests/benchmark_single_gpu_shapes.py, on this framework's sm_100a kernels).

    python -m multi_gpu_flashattention_b200.benchmarks.single_gpu_shapes \
        [--shapes 256x256 1024x1024 ...] [--batch-size 2] [--num-heads 8]
        [--head-dim 64|128] [--dtype bf16|fp16] [--warmup 10] [--repeats 50] [--causal|--no-causal]
        [--backward] [--csv-out results/single_gpu_shapes.csv]

Same columns as the reference's CSV plus TFLOP/s. Causal active elements are
counted top-left aligned like the reference (query i sees keys 0..i)."""
from __future__ import annotations

import argparse
import csv
import os
from statistics import mean, pstdev

import torch

DTYPES = {"bf16": torch.bfloat16, "fp16": torch.float16}

from ..ops.flash import flash_attn_bwd, flash_attn_fwd

DEFAULT_SHAPES = ["256x256", "512x512", "1024x1024", "2048x2048", "4096x4096", "1024x64",
                  "64x1024"]


def parse_shape(text):
    parts = text.lower().split("x")
    if len(parts) != 2:
        raise ValueError(f"Invalid shape '{text}', expected AxB.")
    sq, sk = int(parts[0]), int(parts[1])
    if sq <= 0 or sk <= 0:
        raise ValueError(f"Invalid shape '{text}', dimensions must be positive.")
    return sq, sk


def active_elements(sq, sk, causal):
    if not causal:
        return sq * sk
    if sq <= sk:
        return sq * (sq + 1) // 2
    return sk * (sk + 1) // 2 + (sq - sk) * sk


def bench(sq, sk, a):
    dev = torch.device("cuda", a.device)
    g = torch.Generator(device=dev).manual_seed(0)
    mk = lambda s: torch.randn(a.batch_size, s, a.num_heads, a.head_dim, device=dev,
                               generator=g, dtype=DTYPES[a.dtype])
    q, k, v = mk(sq), mk(sk), mk(sk)
    out, lse = flash_attn_fwd(q, k, v, causal=a.causal)
    do = torch.randn_like(out)

    def run():
        if a.backward:
            flash_attn_bwd(do, q, k, v, out, lse, causal=a.causal)
        else:
            flash_attn_fwd(q, k, v, causal=a.causal)
    for _ in range(a.warmup):
        run()
    torch.cuda.synchronize(dev)
    torch.cuda.reset_peak_memory_stats(dev)
    times = []
    for _ in range(a.repeats):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        run()
        e.record()
        e.synchronize()
        times.append(s.elapsed_time(e))
    act = active_elements(sq, sk, a.causal) * a.batch_size * a.num_heads
    flops = 4 * act * a.head_dim * (2.5 if a.backward else 1.0)
    return {"seq_q": sq, "seq_k": sk, "batch_size": a.batch_size, "num_heads": a.num_heads,
            "head_dim": a.head_dim, "dtype": str(DTYPES[a.dtype]).replace("torch.", ""), "causal": a.causal,
            "active_elements": act, "avg_ms": mean(times), "std_ms": pstdev(times),
            "min_ms": min(times), "max_ms": max(times),
            "peak_mem_mb": torch.cuda.max_memory_allocated(dev) / 2 ** 20,
            "tflops": flops / (mean(times) * 1e-3) / 1e12}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", nargs="+", default=DEFAULT_SHAPES)
    ap.add_argument("--batch-size", type=int, default=2)
    ap.add_argument("--num-heads", type=int, default=8)
    ap.add_argument("--head-dim", type=int, default=128, choices=[64, 128])
    ap.add_argument("--dtype", default="bf16", choices=sorted(DTYPES))
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--repeats", type=int, default=50)
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--backward", action="store_true")
    g = ap.add_mutually_exclusive_group()
    g.add_argument("--causal", dest="causal", action="store_true")
    g.add_argument("--no-causal", dest="causal", action="store_false")
    ap.set_defaults(causal=True)
    ap.add_argument("--csv-out", default="")
    a = ap.parse_args()
    rows = []
    for sh in a.shapes:
        r = bench(*parse_shape(sh), a)
        rows.append(r)
        print(f"{r['seq_q']}x{r['seq_k']}: {r['avg_ms']:.3f} ms (+/- {r['std_ms']:.3f}) "
              f"{r['tflops']:.1f} TFLOP/s peak_mem={r['peak_mem_mb']:.1f} MB", flush=True)
    if a.csv_out:
        os.makedirs(os.path.dirname(a.csv_out) or ".", exist_ok=True)
        with open(a.csv_out, "w", newline="") as f:
            w = csv.DictWriter(f, fieldnames=list(rows[0].keys()))
            w.writeheader()
            w.writerows(rows)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
