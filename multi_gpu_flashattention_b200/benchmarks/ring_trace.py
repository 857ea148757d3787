"""Record a ring engine's per-CTA timeline for one forward call.

    torchrun --nproc-per-node N -m multi_gpu_flashattention_b200.benchmarks.ring_trace \
        [--seq 131072] [--heads 32] [--out DIR] [--backend fused_stepwise|fused_one_launch]

After 3 untraced calls, one traced call writes DIR/summary_rank<r>.json and
DIR/trace_rank0.json (Chrome trace of rank 0). One-launch ring ("fused_one_launch"):
kernel span, CTA busy times, time CTAs waited for received shards, push window.
Per-step engine ("fused_stepwise"): per step the wall span, longest wait for
the KV shard, mean push time per pushing CTA."""
from __future__ import annotations

import argparse
import json
import os

import torch

from ..parallel.layouts import RingLayout
from ..parallel.ring import ENGINES, P_ENGINES, ring_attention_forward
from ..utils.trace import (one_launch_chrome_events, summarize, summarize_one_launch,
                           to_chrome_events, write_chrome_trace)
from . import common


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--seq", type=int, default=131072)
    ap.add_argument("--heads", type=int, default=32)
    ap.add_argument("--layout", default="zigzag")
    ap.add_argument("--out", default="ring_trace")
    ap.add_argument("--backend", default="fused_stepwise",
                    choices=["fused_one_launch", "fused_stepwise"])
    a = ap.parse_args()
    ctx = common.init(need_world_gt1=True)
    lay = RingLayout(a.layout, a.seq, ctx.world, mask="causal")
    L = lay.max_local_len
    g = torch.Generator(device=ctx.device).manual_seed(ctx.rank)
    mk = lambda: (torch.randn(1, L, a.heads, 128, device=ctx.device, generator=g) * 0.5).bfloat16()
    q, k, v = mk(), mk(), mk()
    for _ in range(3):
        ring_attention_forward(q, k, v, lay, causal=True, backend=a.backend, check=True)
    one = a.backend == "fused_one_launch"
    eng = (P_ENGINES if one else ENGINES).get(None, ctx.device, k.numel() * 2)
    eng.set_trace(True)
    torch.cuda.synchronize()
    ctx.barrier()
    ring_attention_forward(q, k, v, lay, causal=True, backend=a.backend, check=True)
    torch.cuda.synchronize()
    eng.set_trace(False)
    tr = eng.last_trace().cpu()
    os.makedirs(a.out, exist_ok=True)
    summ = summarize_one_launch(tr) if one else summarize(tr)
    with open(os.path.join(a.out, f"summary_rank{ctx.rank}.json"), "w") as f:
        json.dump(summ, f, indent=1)
    if ctx.rank == 0:
        ev = one_launch_chrome_events(tr, ctx.rank) if one else to_chrome_events(tr, ctx.rank)
        write_chrome_trace(ev, os.path.join(a.out, "trace_rank0.json"))
        print(json.dumps(summ), flush=True)
    ENGINES.clear()
    P_ENGINES.clear()
    ctx.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
