"""Forward-kernel variant sweep on one GPU (CUDA-event timing, L2 flushed
between launches): the per-query-tile-pair kernel (flash_fwd_sm100.cu) in each
of its pipelines (--variants: 0 whole tiles, 1 half tiles, 2 half tiles with
FMA-pipe exponentials) against the persistent kernel (attn_fwd_persistent.cu)
in each of its softmax variants.

    python -m multi_gpu_flashattention_b200.benchmarks.fwd_tuning [--seq 131072]
        [--heads 32] [--kv-heads 32] [--no-causal] [--reps 5] [--variants 0,1,2]
        [--tunes=0x002,0x302,...]   (--tunes= with no value: stepwise only)

A tune value is the persistent kernel's variant word (attn_fwd_persistent.cuh):
bits 0-7 exponential pairs of every 8 on the FMA pipe (0, 2 or 4), bit 8 packed
f32x2 arithmetic, bit 9 P handed over in two halves. Prints one JSON line per
variant with the median time and attention TFLOP/s. --profile T runs variant T
with its phase counters (bit 10) once and prints the mean clock cycles per key
tile of each softmax and MMA-thread phase; T = -1 profiles the default variant
(packed arithmetic, 0x100). The profiled variants built are the scalar, packed,
packed + split and the tree / speculative combinations of those."""
from __future__ import annotations

import argparse
import json
import statistics

import torch

from .._ext import C
from ..ops.flash import tile_positions

DEFAULT_TUNES = "-1,0x000,0x100,0x200,0x300,0x002,0x102,0x202,0x302,0x004,0x104,0x304"


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--seq", type=int, default=131072)
    ap.add_argument("--heads", type=int, default=32)
    ap.add_argument("--kv-heads", type=int, default=32)
    ap.add_argument("--no-causal", action="store_true")
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--tunes", default=DEFAULT_TUNES)
    ap.add_argument("--variants", default="0,1,2")
    ap.add_argument("--profile", default=None,
                    help="comma-separated tune values to profile by phase instead")
    a = ap.parse_args(argv)
    causal = not a.no_causal
    S, H, Hkv, D = a.seq, a.heads, a.kv_heads, 128
    g = torch.Generator(device="cuda").manual_seed(0)
    q = (torch.randn(1, S, H, D, device="cuda", generator=g) * 0.5).bfloat16()
    k = (torch.randn(1, S, Hkv, D, device="cuda", generator=g) * 0.5).bfloat16()
    v = (torch.randn(1, S, Hkv, D, device="cuda", generator=g) * 0.5).bfloat16()
    o = torch.empty_like(q)
    lse = torch.empty(1, H, S, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    sched = torch.zeros(2, dtype=torch.int32, device="cuda")
    pos = tile_positions(S, "cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    scale = D ** -0.5
    pairs = S * (S + 1) // 2 if causal else S * S
    flops = 4.0 * D * H * pairs

    def stepwise(variant):
        return lambda: C().flash_fwd(q, k, v, o, None, lse, scale, causal, pos, pos, False,
                                     True, st, 2_000_000_000, variant)

    def persistent(tune):
        return lambda: C().flash_fwd_persistent(q, k, v, o, lse, scale, causal, pos, pos, st,
                                                2_000_000_000, sched, tune)

    if a.profile:
        names = ["wait_S", "ld_S", "max", "P_half0", "P_half1", "tiles", "mma_wait_V",
                 "mma_wait_P0h0", "mma_wait_P0h1", "mma_wait_K", "mma_wait_P1h0",
                 "mma_wait_P1h1", "mma_tiles", "mma_loop"]
        for t in a.profile.split(","):
            tv = (0x100 if int(t, 0) < 0 else int(t, 0)) | 0x400
            tr = torch.zeros(512, 16, dtype=torch.int64, device="cuda")
            persistent(tv)()  # warm-up
            tr.zero_()
            flush.fill_(1)
            C().flash_fwd_persistent(q, k, v, o, lse, scale, causal, pos, pos, st,
                                     2_000_000_000, sched, tv, 0, [], tr)
            torch.cuda.synchronize()
            tot = tr.sum(0).double().tolist()
            rec = {"tune": hex(tv), "seq": S}
            for i, nm in enumerate(names):
                if nm in ("tiles", "mma_tiles"):
                    rec[nm] = int(tot[i])
                elif nm == "mma_loop":
                    rec["mma_loop_cycles_per_tile"] = round(tot[i] / max(tot[12], 1), 1)
                elif nm.startswith("mma"):
                    rec[nm] = round(tot[i] / max(tot[12], 1), 1)
                else:
                    rec[nm] = round(tot[i] / max(tot[5], 1), 1)
            print(json.dumps(rec), flush=True)
        return 0

    cases = [("stepwise", int(vr), stepwise(int(vr))) for vr in a.variants.split(",") if vr]
    for t in filter(None, a.tunes.split(",")):
        tv = int(t, 0)
        cases.append(("persistent", tv, persistent(tv)))
    for name, tune, fn in cases:
        for _ in range(2):
            fn()
        times = []
        for i in range(a.reps):
            flush.fill_(i & 0xFF)
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record()
            fn()
            s1.record()
            torch.cuda.synchronize()
            times.append(s0.elapsed_time(s1))
        if int(st.item()) != 0:
            raise SystemExit(f"{name} {tune}: kernel status {int(st.item()):#x}")
        ms = statistics.median(times)
        label = tune if name == "stepwise" else hex(tune) if tune >= 0 else -1
        print(json.dumps({"kernel": name, "variant" if name == "stepwise" else "tune": label,
                          "seq": S, "heads": H, "causal": causal, "ms": round(ms, 3),
                          "tflops": round(flops / ms / 1e9, 1)}), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
