"""Ring-attention forward + backward benchmark with a gradient check.

    torchrun --nproc-per-node N -m multi_gpu_flashattention_b200.benchmarks.ring_train \
        [--seq 524288] [--heads 32] [--kv-heads 8] [--layout striped] [--steps 3]
        [--warmup 2] [--check-seq 32768] [--backend fused]

Inputs and dO are seeded N(0,1)*0.5 bf16 ([1, S, H, 128]). The timed part is
one differentiable ring_attention call plus backward per step (device events,
max over ranks). The check runs the same configuration on --check-seq tokens
and compares each rank's dQ/dK/dV with an fp32 reference computed in query
chunks (exact attention on all-gathered K/V, autograd per chunk).
"""
from __future__ import annotations

import argparse
import json

import torch
import torch.distributed as dist

from ..ops.reference import attention_ref
from ..parallel.api import ring_attention
from ..parallel.layouts import RingLayout
from . import common


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--seq", type=int, default=524288)
    ap.add_argument("--heads", type=int, default=32)
    ap.add_argument("--kv-heads", type=int, default=8)
    ap.add_argument("--layout", default="striped")
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--check-seq", type=int, default=32768)
    ap.add_argument("--backend", default="fused")
    ap.add_argument("--seed", type=int, default=0)
    return ap.parse_args()


def make(ctx, lay, H, Hkv, seed):
    g = torch.Generator(device=ctx.device).manual_seed(seed * 131 + ctx.rank)
    L = lay.max_local_len
    mk = lambda h: (torch.randn(1, L, h, 128, device=ctx.device, generator=g) * 0.5).bfloat16()
    return mk(H), mk(Hkv), mk(Hkv), mk(H)


def chunked_reference(q, k_full, v_full, do, q_pos, k_pos, chunk=1024):
    """fp32 grads of attention(q, K, V) wrt q, K, V, computed over query chunks."""
    kf = k_full.float().requires_grad_()
    vf = v_full.float().requires_grad_()
    dq = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    for a in range(0, q.shape[1], chunk):
        b = min(a + chunk, q.shape[1])
        qc = q[:, a:b].float().requires_grad_()
        o, _ = attention_ref(qc, kf, vf, causal=True, q_pos=q_pos[a:b], k_pos=k_pos)
        o.backward(do[:, a:b].float())
        dq[:, a:b] = qc.grad
    return dq, kf.grad, vf.grad


def check(args, ctx):
    lay = RingLayout(args.layout, args.check_seq, ctx.world, mask="causal")
    q, k, v, do = make(ctx, lay, args.heads, args.kv_heads, args.seed + 1)
    qs, ks, vs = (t.clone().requires_grad_() for t in (q, k, v))
    out = ring_attention(qs, ks, vs, causal=True, layout=lay, backend=args.backend)
    out.backward(do)
    # all-gather K/V (global order) and the dK/dV of every rank for the reference
    L = lay.max_local_len
    kk = [torch.empty_like(k) for _ in range(ctx.world)]
    vv = [torch.empty_like(v) for _ in range(ctx.world)]
    dist.all_gather(kk, k)
    dist.all_gather(vv, v)
    k_full, v_full = lay.unshard(kk), lay.unshard(vv)
    pos = lay.positions(ctx.rank).to(ctx.device)
    all_pos = torch.arange(args.check_seq, device=ctx.device)
    n = lay.local_len(ctx.rank)
    rdq, rdk, rdv = chunked_reference(q[:, :n], k_full, v_full, do[:, :n], pos, all_pos)
    # dK/dV: sum the reference contributions of all ranks' queries
    dist.all_reduce(rdk)
    dist.all_reduce(rdv)
    res = {}
    for name, got, ref in (("dq", qs.grad[:, :n], rdq),
                           ("dk", ks.grad[:, :n], lay.shard(rdk, ctx.rank)[:, :n]),
                           ("dv", vs.grad[:, :n], lay.shard(rdv, ctx.rank)[:, :n])):
        err = (got.float() - ref).abs()
        res[name] = {"max_abs": err.max().item(), "ref_max": ref.abs().max().item(),
                     "rel_l2": ((got.float() - ref).norm() / ref.norm()).item()}
    return res


def main():
    args = parse()
    ctx = common.init()
    P = ctx.world
    res = check(args, ctx) if args.check_seq else None
    lay = RingLayout(args.layout, args.seq, P, mask="causal")
    q, k, v, do = make(ctx, lay, args.heads, args.kv_heads, args.seed)
    qs, ks, vs = (t.requires_grad_() for t in (q, k, v))

    def step():
        out = ring_attention(qs, ks, vs, causal=True, layout=lay, backend=args.backend)
        out.backward(do)
        qs.grad = ks.grad = vs.grad = None

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    ctx.barrier()
    for a, b in ev:
        a.record()
        step()
        b.record()
    torch.cuda.synchronize()
    ms = ctx.max([a.elapsed_time(b) for a, b in ev])
    ms = sum(ms) / len(ms)
    S = args.seq
    fwd_flops = 4.0 * 128 * args.heads * S * (S + 1) / 2
    if ctx.rank == 0:
        print(json.dumps({"seq": S, "heads": args.heads, "kv_heads": args.kv_heads,
                          "layout": args.layout, "gpus": P, "ms_fwd_bwd": round(ms, 3),
                          "tflops_per_gpu_3.5x": round(3.5 * fwd_flops / (ms * 1e-3) / 1e12 / P, 1),
                          "check_seq": args.check_seq, "grad_check": res}), flush=True)
    ctx.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
