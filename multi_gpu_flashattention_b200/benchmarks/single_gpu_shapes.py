"""Single-GPU attention timing over shapes (the reference's
tests/benchmark_single_gpu_shapes.py, on this framework's sm_100a kernels).

    python -m multi_gpu_flashattention_b200.benchmarks.single_gpu_shapes \
        [--shapes 256x256 1024x1024 ...] [--batch-size 2] [--num-heads 8]
        [--head-dim 64|128] [--dtype float16|bfloat16] [--warmup 5] [--repeats 20]
        [--causal|--no-causal] [--backward] [--graph] [--csv-out results/single_gpu_shapes.csv]

Defaults, table and CSV columns are the reference's (fp16, head_dim 64, batch 2,
8 heads, causal; tests/benchmark_single_gpu_shapes.py:188-210), with a TFLOP/s
column added. Causal active elements are counted top-left aligned like the
reference (query i sees keys 0..i). A shape that fails (e.g. out of memory) is
reported and skipped."""
from __future__ import annotations

import argparse
import csv
import os
from statistics import mean, pstdev

import torch

DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16,
          "fp16": torch.float16, "bf16": torch.bfloat16}

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

    if a.graph:
        # replay CUDA graphs of the call (inputs copied into static buffers)
        from ..ops.graphs import GraphedAttention
        g = GraphedAttention(q, k, v, causal=a.causal, backward=a.backward)
        if a.backward:
            g.forward(q, k, v)

        def run():
            if a.backward:
                g.backward(do)
            else:
                g.forward(q, k, v)
    else:
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
    per_seq = active_elements(sq, sk, a.causal)
    flops = 4 * per_seq * a.batch_size * a.num_heads * a.head_dim * (2.5 if a.backward else 1.0)
    return {"seq_q": sq, "seq_k": sk, "batch_size": a.batch_size, "num_heads": a.num_heads,
            "head_dim": a.head_dim, "dtype": str(DTYPES[a.dtype]).replace("torch.", ""),
            "causal": a.causal, "active_per_seq": per_seq, "total_active": per_seq * a.batch_size,
            "avg_ms": mean(times), "std_ms": pstdev(times), "min_ms": min(times),
            "max_ms": max(times), "peak_mem_mb": torch.cuda.max_memory_allocated(dev) / 2 ** 20,
            "tflops": flops / (mean(times) * 1e-3) / 1e12}


def print_results(rows):
    header = (f"{'shape':>12} {'active/seq':>12} {'avg_ms':>10} {'std_ms':>10} {'min_ms':>10} "
              f"{'max_ms':>10} {'peak_mem(MB)':>14} {'TFLOP/s':>9}")
    print(header)
    print("-" * len(header))
    for r in rows:
        shape = f"{r['seq_q']}x{r['seq_k']}"
        print(f"{shape:>12} {r['active_per_seq']:>12d} {r['avg_ms']:>10.3f} {r['std_ms']:>10.3f} "
              f"{r['min_ms']:>10.3f} {r['max_ms']:>10.3f} {r['peak_mem_mb']:>14.1f} "
              f"{r['tflops']:>9.1f}", flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", nargs="+", default=DEFAULT_SHAPES)
    ap.add_argument("--batch-size", type=int, default=2)
    ap.add_argument("--num-heads", type=int, default=8)
    ap.add_argument("--head-dim", type=int, default=64, choices=[64, 128])
    ap.add_argument("--dtype", default="float16", choices=sorted(DTYPES))
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--repeats", type=int, default=20)
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--backward", action="store_true")
    ap.add_argument("--graph", action="store_true",
                    help="replay a CUDA graph of the call (fixed shapes; no host path per call)")
    ap.add_argument("--causal", action=argparse.BooleanOptionalAction, default=True)
    ap.add_argument("--csv-out", default="results/single_gpu_shapes.csv")
    a = ap.parse_args()
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is not available.")
    rows = []
    for sh in a.shapes:
        sq, sk = parse_shape(sh)
        try:
            rows.append(bench(sq, sk, a))
        except RuntimeError as exc:
            print(f"Skipping {sh}: {exc}")
        torch.cuda.empty_cache()
    print_results(rows)
    if a.csv_out and rows:
        os.makedirs(os.path.dirname(a.csv_out) or ".", exist_ok=True)
        with open(a.csv_out, "w", newline="") as f:
            w = csv.DictWriter(f, fieldnames=list(rows[0].keys()))
            w.writeheader()
            w.writerows(rows)
        print(f"\nCSV saved to: {a.csv_out}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
