"""Ring-attention benchmark driver (the reference's ring/attention/bench programs).

    torchrun --nproc-per-node N -m multi_gpu_flashattention_b200.benchmarks.ring_attention \
        <kv_size_bytes> [warmup=10] [iters=100] [--backend B] [--numerics fp32|bf16]
        [--init legacy|randn] [--layout contiguous|zigzag|striped] [--causal]
        [--heads H] [--kv-heads H] [--head-dim D] [--seed S] [--overlap]

Shapes follow the reference: tokens per rank = kv_size_bytes / (heads * head_dim * 4)
(one fp32 tensor of the shard), so the global length grows with the ranks
(ring/attention/bench/ring_attention_nccl_gpu_bench.cu:180-200).

--numerics fp32 (default; head_dim 64): the fp32 kernels of csrc/kernels/legacy_fp32.cu,
  backends nccl | staged | p2p | ce (p2p / ce: the KV shard moves through
  RingExchange's receive slots by the NVLink push kernel / the copy engine, in the
  sequential order). --init legacy reproduces the reference's inputs (K == V,
  no softmax scale) so `verify_full <dir> N kv_size` checks the dumps;
  --init randn uses the seeded N(0,1) streams and scale 1/sqrt(d)
  (`verify_full <dir> N kv_size --init randn`).
--numerics bf16 (head_dim 128): the sm_100a kernels, backends fused | p2p_unfused |
  ce_unfused | nccl | staged (p2p_unfused: the fused path's NVLink push transport as
  a separate kernel on a second stream; ce_unfused: the copy engine moves the shard
  on a second stream -- the ablations that isolate the fusion).

Environment (as in the reference): ATTENTION_PRINT_SHARDS=1 prints token ranges
and the owner of the shard computed/received at each step of iteration 0;
ATTENTION_DUMP_OUTPUT=1 writes ring_output_rank<r>.bin (raw fp32, normalised,
[tokens x heads x dim]). Timing is on the device, max over ranks per iteration,
mean over iterations; rank 0 prints `<backend> bench: warmup=W iters=I` and
`avg_total=... ms avg_<COMM>=... avg_attn=... avg_merge=... avg_final=...`.
"""
from __future__ import annotations

import argparse
import math
import os

import torch
import torch.distributed as dist

from .._ext import C, sched as _sched
from ..parallel.layouts import RingLayout
from . import common

COMM_NAME = {"nccl": "NCCL", "staged": "MPI", "fused": "P2P", "fused_stepwise": "P2P",
             "fused_one_launch": "P2P",
             "p2p_unfused": "P2P",
             "ce_unfused": "CE", "p2p": "P2P", "ce": "CE"}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("kv_size", type=int, nargs="?")
    ap.add_argument("warmup", type=int, nargs="?", default=10)
    ap.add_argument("iters", type=int, nargs="?", default=100)
    ap.add_argument("--backend", default=None,
                    choices=["fused", "fused_stepwise", "fused_one_launch", "p2p_unfused",
                             "ce_unfused", "nccl", "staged", "p2p", "ce"])
    ap.add_argument("--numerics", default="fp32", choices=["fp32", "bf16"])
    ap.add_argument("--init", default="legacy", choices=["legacy", "randn"])
    ap.add_argument("--layout", default="contiguous",
                    choices=["contiguous", "zigzag", "striped", "scheduler"])
    ap.add_argument("--policy", default="lpt", choices=["dp", "lpt"],
                    help="scheduler layout: row LPT (default) or contiguous-row DP partition")
    ap.add_argument("--dump-format", default="bin", choices=["bin", "npy", "pt"],
                    help="with ATTENTION_DUMP_OUTPUT: raw fp32 (reference format), or .npy / .pt "
                         "with the output and the fp32 LSE")
    ap.add_argument("--json", action="store_true", help="also print one JSON summary line")
    ap.add_argument("--causal", action="store_true")
    ap.add_argument("--heads", type=int, default=1)
    ap.add_argument("--kv-heads", type=int, default=0)
    ap.add_argument("--head-dim", type=int, default=0)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--overlap", action="store_true",
                    help="fp32 backends: move the next shard while computing (the reference's "
                         "*_overlap variants)")
    return ap.parse_args()


# ---------------------------------------------------------------------- inputs
def make_inputs(args, ctx, lay, H, Hkv, D, dtype):
    S = _sched()
    r, dev = ctx.rank, ctx.device
    L = lay.local_len(r)
    if args.init == "legacy":
        # reference formulas, evaluated on the host in fp32 (verify_full.c:69-90)
        n = L * D  # < 2^24, so every value below is an exact fp32 integer / product
        kv = torch.full((n,), r * 1000.0, dtype=torch.float32) + torch.arange(n, dtype=torch.float32)
        q = (torch.full((n,), r * 500.0, dtype=torch.float32)
             + (torch.arange(n) % D).to(torch.float32) * torch.tensor(0.01, dtype=torch.float32)) \
            * torch.tensor(0.001, dtype=torch.float32)
        q = q.view(1, L, 1, D).to(dev)
        kv = kv.view(1, L, 1, D).to(dev)
        return q, kv, kv
    rows = lay.positions(r).tolist()
    out = []
    for stream, heads in ((0, H), (1, Hkv), (2, Hkv)):
        buf = torch.empty(L * heads * D, dtype=torch.float32)
        S.fill_randn_rows(buf.numpy(), args.seed, stream, rows, heads * D)
        out.append(buf.view(1, L, heads, D).to(dev).to(dtype))
    return tuple(out)


# ---------------------------------------------------------------------- shard logs
def log_shards(ctx, lay, L):
    r = ctx.rank
    if lay.kind == "contiguous":
        a, b = r * L, (r + 1) * L
        ctx.log(f"[Rank {r}] Q tokens=[{a},{b}) KV tokens=[{a},{b}) "
                f"global_Q={L * ctx.world} global_KV={L * ctx.world}")
    else:
        d = lay.describe(r)
        ctx.log(f"[Rank {r}] Q tokens={d} KV tokens={d} global_Q={lay.seq} global_KV={lay.seq}")


def tokens(lay, owner):
    d = lay.describe(owner)
    return d


# ---------------------------------------------------------------------- fp32 ring
class Fp32Ring:
    """fp32 partial-attention + merge ring over NCCL or staged host copies."""

    def __init__(self, args, ctx, lay, q, k, v, scale):
        self.args, self.ctx, self.lay = args, ctx, lay
        self.q, self.k, self.v, self.scale = q[0], k[0], v[0], scale
        self.same_kv = k.data_ptr() == v.data_ptr()
        L, H, D = self.q.shape
        dev = ctx.device
        f = dict(dtype=torch.float32, device=dev)
        self.m_run, self.l_run = torch.empty(H, L, **f), torch.empty(H, L, **f)
        self.acc_run = torch.empty(L, H, D, **f)
        self.m_loc, self.l_loc = torch.empty(H, L, **f), torch.empty(H, L, **f)
        self.acc_loc = torch.empty(L, H, D, **f)
        self.out = torch.empty(L, H, D, **f)
        self.bufs = [torch.empty_like(self.k), torch.empty_like(self.v)]
        self.nbufs = [torch.empty_like(self.k), torch.empty_like(self.v)]
        self.causal = args.causal
        P = ctx.world
        self.q_pos = lay.q_positions_for_mask(ctx.rank).to(dev)
        self.k_pos = [lay.k_positions_for_mask(ctx.rank, o).to(dev) for o in range(P)]
        self.ev = [torch.cuda.Event(enable_timing=True) for _ in range(8)]
        if args.backend == "staged":
            self.h_send = [torch.empty(self.k.shape, pin_memory=True) for _ in range(2)]
            self.h_recv = [torch.empty(self.k.shape, pin_memory=True) for _ in range(2)]
        if args.backend in ("p2p", "ce"):
            # KV rotation through RingExchange's two receive slots (K, then V
            # unless K == V), moved by the push kernel or the copy engine
            n = self.k.numel()
            self.kv_bytes = n * 4 * (1 if self.same_kv else 2)
            sms = torch.cuda.get_device_properties(dev).multi_processor_count
            self.ex = C().RingExchange(ctx.rank, P, dev.index,
                                       (self.kv_bytes + 4095) // 4096 * 4096, 2 * sms)
            common.exchange_handles(self.ex, P)
            self.ex_status = torch.zeros(1, dtype=torch.int32, device=dev)
            torch.cuda.synchronize()
        self.comm_stream = torch.cuda.Stream(dev)

    def _slot_kv(self, i):
        b = self.ex.slot(i)[: self.kv_bytes].view(torch.float32)
        n = self.k.numel()
        kk = b[:n].view(self.k.shape)
        return kk, (kk if self.same_kv else b[n: 2 * n].view(self.v.shape))

    def _attn_merge(self, kk, vv, owner, first):
        Cm = C()
        e = self.ev
        e[0].record()
        Cm.legacy_partial(self.q, kk, vv, self.scale, self.q_pos, self.k_pos[owner], self.causal,
                          self.acc_loc, self.m_loc, self.l_loc, False)
        e[1].record()
        if first:
            self.m_run.copy_(self.m_loc)
            self.l_run.copy_(self.l_loc)
            self.acc_run.copy_(self.acc_loc)
        else:
            Cm.legacy_merge(self.m_run, self.l_run, self.acc_run, self.m_loc, self.l_loc,
                            self.acc_loc)
        e[2].record()
        torch.cuda.synchronize()
        return e[0].elapsed_time(e[1]), e[1].elapsed_time(e[2])

    def _exchange(self, cur, nxt):
        P, r = self.ctx.world, self.ctx.rank
        right, left = (r + 1) % P, (r - 1) % P
        n_t = 1 if self.same_kv else 2
        if self.args.backend == "nccl":
            ops = []
            for i in range(n_t):
                ops += [dist.P2POp(dist.isend, cur[i], right), dist.P2POp(dist.irecv, nxt[i], left)]
            return dist.batch_isend_irecv(ops)
        for i in range(n_t):
            self.h_send[i].copy_(cur[i])
        reqs = []
        for i in range(n_t):
            reqs.append(dist.isend(self.h_send[i], right, group=self.ctx.cpu_group))
            reqs.append(dist.irecv(self.h_recv[i], left, group=self.ctx.cpu_group))
        return reqs

    def _finish_exchange(self, reqs, nxt):
        for q in reqs:
            q.wait()
        if self.args.backend == "staged":
            for i in range(1 if self.same_kv else 2):
                nxt[i].copy_(self.h_recv[i])

    def _kv(self, pair):
        return (pair[0], pair[0]) if self.same_kv else (pair[0], pair[1])

    def _run_exchange(self, log_steps):
        """Sequential ring over RingExchange: own shard, then per step one
        transfer into slot (s+1) % 2 and the attention on it. Each push hands its
        slot back only after reading it, and in this order every attention on a
        slot finishes before the push that forwards (and releases) it."""
        ctx, lay, P, r = self.ctx, self.lay, self.ctx.world, self.ctx.rank
        t_comm = t_attn = t_merge = 0.0
        ex, limit = self.ex, 2_000_000_000
        e_tot0, e_tot1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_tot0.record()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record()
        kk, vv = self._slot_kv(0)
        kk.copy_(self.k)
        if not self.same_kv:
            vv.copy_(self.v)
        c1.record()
        torch.cuda.synchronize()
        t_comm += c0.elapsed_time(c1)
        if log_steps:
            ctx.log(f"[Rank {r}] step=own compute_kv_owner={r} KV tokens={tokens(lay, r)}")
        a, m = self._attn_merge(self.k, self.v, r, True)
        t_attn += a
        t_merge += m
        for s in range(P - 1):
            c0.record()
            ex.step(s, self.kv_bytes, self.args.backend, self.ex_status, limit)
            # the left neighbour's transfer into the slot we read next may still
            # be in flight: wait for its arrivals
            ex.wait_received(s, self.args.backend, self.ex_status, limit)
            c1.record()
            torch.cuda.synchronize()
            t_comm += c0.elapsed_time(c1)
            owner = lay.receive_owner(r, s)
            if log_steps:
                ctx.log(f"[Rank {r}] step={s} received_kv_owner={owner} KV tokens={tokens(lay, owner)}")
            a, m = self._attn_merge(*self._slot_kv((s + 1) & 1), owner, False)
            t_attn += a
            t_merge += m
        ex.release(P - 1, self.args.backend, self.ex_status, limit)
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        C().legacy_normalize(self.acc_run, self.l_run, self.out)
        host = self.out.cpu()
        f1.record()
        e_tot1.record()
        torch.cuda.synchronize()
        if int(self.ex_status.item()):
            raise RuntimeError(f"[Rank {r}] transport status {int(self.ex_status.item()):#x}")
        return e_tot0.elapsed_time(e_tot1), t_comm, t_attn, t_merge, f0.elapsed_time(f1), host

    def run(self, log_steps):
        if self.args.backend in ("p2p", "ce"):
            return self._run_exchange(log_steps)
        ctx, lay, P, r = self.ctx, self.lay, self.ctx.world, self.ctx.rank
        t_comm = t_attn = t_merge = 0.0
        e_tot0, e_tot1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_tot0.record()
        pairs = [self.bufs, self.nbufs]
        cur, nxt_i = [self.k, self.v], 0
        if not self.args.overlap:
            # the reference's sequential order: own shard, then receive + compute per step
            if log_steps:
                ctx.log(f"[Rank {r}] step=own compute_kv_owner={r} KV tokens={tokens(lay, r)}")
            a, m = self._attn_merge(*self._kv(cur), r, True)
            t_attn += a
            t_merge += m
            for s in range(P - 1):
                nxt = pairs[nxt_i]
                c0 = torch.cuda.Event(enable_timing=True)
                c1 = torch.cuda.Event(enable_timing=True)
                c0.record()
                self._finish_exchange(self._exchange(cur, nxt), nxt)
                c1.record()
                torch.cuda.synchronize()
                t_comm += c0.elapsed_time(c1)
                owner = lay.receive_owner(r, s)
                if log_steps:
                    ctx.log(f"[Rank {r}] step={s} received_kv_owner={owner} KV tokens={tokens(lay, owner)}")
                a, m = self._attn_merge(*self._kv(nxt), owner, False)
                t_attn += a
                t_merge += m
                cur, nxt_i = nxt, nxt_i ^ 1
        else:
            # the reference's overlap order: move the next shard while computing this one
            owner = r
            for s in range(P - 1):
                nxt = pairs[nxt_i]
                recv_owner = lay.receive_owner(r, s)
                if log_steps:
                    ctx.log(f"[Rank {r}] step={s} compute_kv_owner={owner} KV tokens={tokens(lay, owner)}, "
                            f"receiving_kv_owner={recv_owner} KV tokens={tokens(lay, recv_owner)}")
                c0 = torch.cuda.Event(enable_timing=True)
                c1 = torch.cuda.Event(enable_timing=True)
                self.comm_stream.wait_stream(torch.cuda.current_stream())
                c0.record(self.comm_stream)
                with torch.cuda.stream(self.comm_stream):
                    reqs = self._exchange(cur, nxt)
                a, m = self._attn_merge(*self._kv(cur), owner, s == 0)
                t_attn += a
                t_merge += m
                with torch.cuda.stream(self.comm_stream):
                    self._finish_exchange(reqs, nxt)
                c1.record(self.comm_stream)
                torch.cuda.current_stream().wait_stream(self.comm_stream)
                torch.cuda.synchronize()
                t_comm += c0.elapsed_time(c1)
                cur, nxt_i, owner = nxt, nxt_i ^ 1, recv_owner
            if log_steps:
                ctx.log(f"[Rank {r}] final compute_kv_owner={owner} KV tokens={tokens(lay, owner)}")
            a, m = self._attn_merge(*self._kv(cur), owner, P == 1)
            t_attn += a
            t_merge += m
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        C().legacy_normalize(self.acc_run, self.l_run, self.out)
        host = self.out.cpu()
        f1.record()
        e_tot1.record()
        torch.cuda.synchronize()
        t_final = f0.elapsed_time(f1)
        return e_tot0.elapsed_time(e_tot1), t_comm, t_attn, t_merge, t_final, host


# ---------------------------------------------------------------------- bf16 ring
class Bf16Ring:
    def __init__(self, args, ctx, lay, q, k, v, scale):
        self.args, self.ctx, self.lay = args, ctx, lay
        self.q, self.k, self.v, self.scale = q, k, v, scale
        self.status = torch.zeros(1, dtype=torch.int32, device=ctx.device)

    def run(self, log_steps):
        from ..parallel.ring import ENGINES, P_ENGINES, _meta, ring_attention_forward
        ctx, lay, P, r = self.ctx, self.lay, self.ctx.world, self.ctx.rank
        if log_steps:
            for s in range(P - 1):
                o, ro = lay.compute_owner(r, s), lay.receive_owner(r, s)
                ctx.log(f"[Rank {r}] step={s} compute_kv_owner={o} KV tokens={tokens(lay, o)}, "
                        f"receiving_kv_owner={ro} KV tokens={tokens(lay, ro)}")
            o = lay.compute_owner(r, P - 1)
            ctx.log(f"[Rank {r}] final compute_kv_owner={o} KV tokens={tokens(lay, o)}")
        fused = self.args.backend in ("fused", "fused_stepwise", "fused_one_launch",
                                      "p2p_unfused", "ce_unfused") and P > 1
        if fused:
            from ..parallel.ring import resolve_backend
            one = resolve_backend(self.args.backend) == "fused_one_launch"
            engines = P_ENGINES if one else ENGINES
            eng = engines.get(None, ctx.device, self.k.numel() * self.k.element_size())
            qtp, kvtp, kv_lens = _meta(lay, r, ctx.device)

            def compute_only():
                c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                c0.record()
                eng.forward_compute_only(self.q, self.k, self.v, self.scale, self.args.causal,
                                         qtp if self.args.causal else None,
                                         kvtp if self.args.causal else None, kv_lens, self.status)
                c1.record()
                torch.cuda.synchronize()
                return c0.elapsed_time(c1)
            # the compute-only reference runs before and after the ring and the two
            # are averaged, so clock drift does not land on one side
            before = compute_only()
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record()
        out, lse = ring_attention_forward(self.q, self.k, self.v, lay, causal=self.args.causal,
                                          softmax_scale=self.scale, backend=self.args.backend,
                                          status=self.status,
                                          cpu_group=ctx.cpu_group)
        e1.record()
        host = out[0].float().cpu()
        self.lse = lse[0].cpu()
        e2.record()
        torch.cuda.synchronize()
        total = e0.elapsed_time(e2)
        t_attn = e0.elapsed_time(e1)
        t_comm = 0.0
        if fused:
            t_comp = 0.5 * (before + compute_only())
            t_comm = max(0.0, t_attn - t_comp)  # exposed communication
            t_attn = t_comp
        return total, t_comm, t_attn, 0.0, e1.elapsed_time(e2), host


# ---------------------------------------------------------------------- main
def main():
    args = parse()
    ctx = common.init(need_world_gt1=True)
    P, r, dev = ctx.world, ctx.rank, ctx.device
    if args.backend is None:
        args.backend = "fused" if args.numerics == "bf16" else "nccl"
    D = args.head_dim or (128 if args.numerics == "bf16" else 64)
    H, Hkv = args.heads, args.kv_heads or args.heads
    unit = H * D * 4
    if args.kv_size is None:
        ctx.log0(f"Usage: ring_attention <kv_size_bytes> [warmup>=0] [iters>0]\n"
                 f"kv_size_bytes must be a positive multiple of {unit} bytes.")
        ctx.close()
        return 1
    if args.kv_size <= 0 or args.kv_size % unit != 0 or args.warmup < 0 or args.iters <= 0:
        ctx.log0(f"Invalid arguments: kv_size must be a positive multiple of {unit}, "
                 "warmup >= 0, iters > 0.")
        ctx.close()
        return 1
    fp32_backends = ("nccl", "staged", "p2p", "ce")
    if (args.numerics == "fp32" and (D != 64 or args.backend not in fp32_backends)) or \
            (args.numerics == "bf16" and args.backend in ("p2p", "ce")) or \
            (args.overlap and args.backend in ("p2p", "ce")):
        ctx.log0("fp32 numerics: head_dim 64, backends nccl, staged, p2p or ce (p2p and ce "
                 "run in the sequential order only)")
        ctx.close()
        return 1
    if args.init == "legacy" and (H != 1 or args.layout != "contiguous" or args.causal
                                  or args.numerics != "fp32"):
        ctx.log0("--init legacy is the reference's fp32 single-head, contiguous, non-causal setup")
        ctx.close()
        return 1
    L = args.kv_size // unit
    seq = L * P
    lay = RingLayout(args.layout, seq, P, mask="causal" if args.causal else "full",
                     policy=args.policy)
    props = torch.cuda.get_device_properties(dev)
    lr = int(os.environ.get("LOCAL_RANK", r))
    ctx.log(f"[Rank {r} local_rank {lr}] GPU {dev.index}: {props.name} "
            f"({props.total_memory / 1e6:.0f} MB total)")
    print_shards = os.environ.get("ATTENTION_PRINT_SHARDS") is not None
    if print_shards:
        log_shards(ctx, lay, L)
    ctx.log(f"[Rank {r}] seq_q={L}, seq_k={L}, dim={D}, KV shard={L * H * D * 4 / 1024:.1f} KB")

    scale = 1.0 if args.init == "legacy" else 1.0 / math.sqrt(D)
    dtype = torch.float32 if args.numerics == "fp32" else torch.bfloat16
    q, k, v = make_inputs(args, ctx, lay, H, Hkv, D, dtype)
    ring = (Fp32Ring if args.numerics == "fp32" else Bf16Ring)(args, ctx, lay, q, k, v, scale)

    sums = [0.0] * 5
    host = None
    for it in range(args.warmup + args.iters):
        ctx.barrier()
        res = ring.run(print_shards and it == 0)
        host = res[5]
        mx = ctx.max(list(res[:5]))
        if it >= args.warmup:
            sums = [a + b for a, b in zip(sums, mx)]
    if args.numerics == "bf16":
        st = int(ring.status.item())
        if st:
            raise RuntimeError(f"[Rank {r}] kernel status {st:#x}")
    name = args.backend + ("_overlap" if args.overlap else "")
    comm = COMM_NAME[args.backend]
    if r == 0:
        n = args.iters
        print(f"{name} bench: warmup={args.warmup} iters={args.iters}", flush=True)
        print(f"avg_total={sums[0] / n:.3f} ms avg_{comm}={sums[1] / n:.3f} "
              f"avg_attn={sums[2] / n:.3f} avg_merge={sums[3] / n:.3f} avg_final={sums[4] / n:.3f}",
              flush=True)
    if r == 0 and args.json:
        n = args.iters
        S_tot = lay.seq
        pairs = S_tot * (S_tot + 1) // 2 if args.causal else S_tot * S_tot
        flops = 4.0 * D * H * pairs
        # ring time: the attention ring itself (comm + attention + merge), without
        # the final normalisation / download of the output
        ring_ms = (sums[1] + sums[2] + sums[3]) / n
        import json as _json
        roof = None
        if args.numerics == "bf16":
            # slower of the per-GPU attention FLOPs at the measured sustained bf16
            # peak and the KV bytes each rank sends over NVLink at 770 GB/s
            here = os.path.dirname(os.path.abspath(__file__))
            peaks = os.path.join(here, "..", "..", "MEASURED_PEAKS.json")
            peak = _json.load(open(peaks))["bf16_tflops_sustained"] if os.path.exists(peaks) \
                else 1400.0
            kv_bytes = (P - 1) * 2 * L * Hkv * D * 2
            t_roof = max(flops / P / (peak * 1e12), kv_bytes / 770e9) * 1e3
            roof = t_roof / ring_ms if ring_ms > 0 else None
        print(_json.dumps({"backend": name, "numerics": args.numerics, "ranks": P,
                           "seq": S_tot, "heads": H, "head_dim": D, "causal": args.causal,
                           "layout": args.layout, "avg_total_ms": sums[0] / n,
                           "ring_ms": ring_ms, "avg_comm_ms": sums[1] / n,
                           "avg_attn_ms": sums[2] / n,
                           "tflops_per_gpu": flops / (ring_ms * 1e-3) / 1e12 / P,
                           "comm_fraction": (sums[1] / n) / ring_ms if ring_ms > 0 else None,
                           "roofline_fraction": roof}),
              flush=True)
    if os.environ.get("ATTENTION_DUMP_OUTPUT") is not None:
        lse = getattr(ring, "lse", None)
        if args.dump_format == "bin":
            fname = f"ring_output_rank{r}.bin"
            host.contiguous().numpy().astype("<f4").tofile(fname)
        elif args.dump_format == "npy":
            import numpy as np
            fname = f"ring_output_rank{r}.npy"
            np.save(fname, host.contiguous().numpy().astype("<f4"))
            if lse is not None:
                np.save(f"ring_lse_rank{r}.npy", lse.numpy().astype("<f4"))
        else:
            fname = f"ring_output_rank{r}.pt"
            torch.save({"out": host, "lse": lse, "positions": lay.positions(r)}, fname)
        ctx.log(f"[Rank {r}] output dumped to {fname}")
    ctx.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
