"""Headline benchmark: ring-attention forward at 128K tokens, causal, bf16,
32 heads x head_dim 128, batch 1, zigzag shards, on N GPUs of one node.

    python bench.py [--gpus N] [--steps K] [--warmup W]
                    [--backend fused|p2p_unfused|ce_unfused|nccl|staged]
    torchrun --nproc-per-node N bench.py --gpus N ...      (N > 1)
    python bench.py --impl reference ...                   (the reference's own code path)

Rank 0 prints one JSON line. `value` is the whole-job attention throughput
(TFLOP/s summed over the N GPUs); `ms_per_step` is one ring-attention forward
over the full 128K sequence, timed on the device with CUDA events as the max
over ranks. Inputs are seeded N(0,1)*0.5 (synthetic, no checkpoint needed).
The total sequence is fixed as N grows (strong scaling).
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import re
import statistics
import subprocess
import sys
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "ring-attn ms & TFLOP/s/GPU at 128K causal bf16, 1/2/4/8 B200; exposed comm %"


def parse():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--backend", choices=["fused", "fused_stepwise", "fused_one_launch",
                                          "p2p_unfused", "ce_unfused", "nccl", "staged"],
                    default="fused")
    ap.add_argument("--seq", type=int, default=131072)
    ap.add_argument("--heads", type=int, default=32)
    ap.add_argument("--kv-heads", type=int, default=32)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--layout", default="zigzag")
    ap.add_argument("--no-causal", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--ref-timeout", type=float, default=900.0,
                    help="wall-clock limit (s) for the reference program (--impl reference)")
    return ap.parse_args()


# ---------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region (rank 0)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, devices):
        self.devices = devices
        self.proc = None
        self.path = os.path.join("/tmp", f"mgfa_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-i", ",".join(str(d) for d in self.devices), "-lms", "200"],
                stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for n, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx),
                "power_w_max": max(power) if power else None, "samples": len(sm),
                "reasons": sorted(reasons)}


# ---------------------------------------------------------------------- reference arm
REF_BIN = os.environ.get("MGFA_REF_BIN", os.path.join(ROOT, "baseline", "_ref", "bin"))
REF_HEAD_DIM = 64  # fixed in the reference's benchmarks (ring/attention/bench/*.cu)


def run_child(cmd, env, timeout):
    """Runs cmd in its own process group and returns (output, exit code). The
    group is killed on timeout, and when this process is told to terminate
    (the launcher ending a failed job), so no program outlives its rank."""
    import signal

    child = subprocess.Popen(cmd, env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                             text=True, start_new_session=True)

    def kill_group():
        try:
            os.killpg(child.pid, signal.SIGKILL)
        except ProcessLookupError:
            pass

    def on_term(signum, frame):
        kill_group()
        raise SystemExit(128 + signum)

    old = signal.signal(signal.SIGTERM, on_term)
    try:
        out, _ = child.communicate(timeout=timeout)
        return out, child.returncode
    except subprocess.TimeoutExpired:
        kill_group()
        child.communicate()
        return f"timed out after {timeout} s", -1
    finally:
        signal.signal(signal.SIGTERM, old)


def reference_arm(args):
    """Runs the reference's own NCCL ring-attention benchmark
    (ring/attention/bench/ring_attention_nccl_gpu_bench.cu, built unmodified by
    benchmarks/build_reference.sh against this repository's MPI subset) on the
    same N GPUs and total sequence length, and reports it in the headline's
    units. The reference's kernel computes only fp32, one head, head_dim 64,
    non-causal attention with K=V, so that is the workload it is timed on; its
    own timer (MPI_Wtime from a barrier to the host-normalised output, max over
    ranks, averaged over its timed iterations) gives ms_per_step."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))

    def unavailable(reason):
        if rank == 0:
            print(json.dumps({"impl": "reference", "metric": METRIC, "n_gpus": args.gpus,
                              "unavailable": reason}), flush=True)
        return 0

    if world < 2:
        return unavailable("the reference's ring attention benchmarks need at least 2 ranks "
                           "(they exit with 'Need at least 2 processes.' at world size 1)")
    exe = os.path.join(REF_BIN, "ring_attention_nccl_gpu_bench")
    if not os.path.exists(exe):
        return unavailable("the reference build is missing: benchmarks/build_reference.sh "
                           "builds it from the reference source tree")
    S = args.seq
    if S % world:
        return unavailable(f"seq {S} does not split evenly over {world} ranks")
    seq_k = S // world
    kv_bytes = seq_k * REF_HEAD_DIM * 4
    env = dict(os.environ, MPI_LOCALRANKID=os.environ.get("LOCAL_RANK", str(rank)))
    sampler = ClockSampler(list(range(world))) if rank == 0 else None
    if sampler:
        sampler.start()
    t_wall = time.time()
    out, rc = run_child([exe, str(kv_bytes), str(args.warmup), str(args.steps)], env,
                        args.ref_timeout)
    wall = time.time() - t_wall
    clocks = sampler.stop() if sampler else None
    if rank != 0:
        return 0 if rc == 0 else 1
    m = re.search(r"avg_total=([\d.]+) ms avg_NCCL=([\d.]+) avg_attn=([\d.]+) "
                  r"avg_merge=([\d.]+) avg_final=([\d.]+)", out)
    if rc != 0 or not m:
        tail = " | ".join(out.strip().splitlines()[-3:])
        unavailable(f"the reference benchmark failed (exit {rc}): {tail}"[:400])
        return 1  # a failed rank ends the launcher's other ranks (and their programs)
    total, nccl, attn, merge, final = (float(x) for x in m.groups())
    flops = 4.0 * REF_HEAD_DIM * S * S  # every query row against every key, one head
    tflops = flops / (total * 1e-3) / 1e12
    rec = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(tflops, 4),
        "unit": "TFLOP/s (attention, summed over GPUs)",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(total, 3),
        "tflops_per_gpu": round(tflops / world, 4),
        "exposed_comm_pct": round(100.0 * nccl / total, 2),
        "breakdown_ms": {"nccl": nccl, "attn": attn, "merge": merge, "final": final},
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "fp32",
        "data": "synthetic: the reference's built-in inputs (K=V=rank*1000+i, "
                "Q=(rank*500+(i%64)*0.01)*0.001)",
        "config": {"model": "ring attention fwd, non-causal, 1 head x d64, K=V (the only "
                            "shape the reference's kernel computes)",
                   "global_batch": 1, "seq_len": S,
                   "parallelism": f"cp{world} ring (contiguous shards), NCCL send/recv",
                   "l2": "inputs per rank below L2; the reference does not flush"},
        "timing": "the reference's own: MPI_Wtime from a barrier to the host-normalised "
                  "output, max over ranks (MPI over this repository's TCP-store MPI subset)",
        "program": "ring/attention/bench/ring_attention_nccl_gpu_bench.cu, unmodified, "
                   f"args {kv_bytes} {args.warmup} {args.steps}",
        "clocks": clocks,
        "gpu_launches": 2 * world * args.steps,
        "wall_s": round(wall, 3),
    }
    print(json.dumps(rec), flush=True)
    return 0


# ---------------------------------------------------------------------- ours
def main():
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)

    from multi_gpu_flashattention_b200.parallel.layouts import RingLayout
    from multi_gpu_flashattention_b200.parallel.ring import ENGINES, ring_attention_forward
    from multi_gpu_flashattention_b200.ops.flash import check_status
    import multi_gpu_flashattention_b200 as mgfa

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    causal = not args.no_causal
    S, H, Hkv, D, B = args.seq, args.heads, args.kv_heads, 128, args.batch
    lay = RingLayout(args.layout if world > 1 else "contiguous", S, world,
                     mask="causal" if causal else "full")
    L = lay.max_local_len
    g = torch.Generator(device=dev).manual_seed(args.seed * 1000 + rank)
    q = (torch.randn(B, L, H, D, device=dev, generator=g) * 0.5).bfloat16()
    k = (torch.randn(B, L, Hkv, D, device=dev, generator=g) * 0.5).bfloat16()
    v = (torch.randn(B, L, Hkv, D, device=dev, generator=g) * 0.5).bfloat16()
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)  # > 126 MB L2

    def step():
        return ring_attention_forward(q, k, v, lay, causal=causal, group=group,
                                      backend=args.backend, status=status)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(xs):
        t = torch.tensor(xs, dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    # warm-up (also builds engines / metadata)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    check_status(status, "warm-up")

    # ---------------- device-timed region
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    sampler = ClockSampler([local + i for i in range(world)] if world > 1 else [local]) \
        if rank == 0 else None
    barrier()
    torch.cuda.synchronize()
    if sampler:
        sampler.start()
        time.sleep(0.3)
    barrier()
    wall0 = time.perf_counter()
    for i in range(args.steps):
        flush.fill_(i & 0xFF)  # evict L2 between steps (outside the events)
        starts[i].record()
        step()
        ends[i].record()
    torch.cuda.synchronize()
    barrier()
    wall = time.perf_counter() - wall0
    clocks = sampler.stop() if sampler else None
    check_status(status, "timed steps")
    per_step = max_over_ranks([s.elapsed_time(e) for s, e in zip(starts, ends)])
    ms = sum(per_step) / len(per_step)

    # ---------------- compute-only reference for the exposed-comm fraction
    exposed = None
    from multi_gpu_flashattention_b200.parallel.ring import resolve_backend
    concrete = resolve_backend(args.backend)
    if world > 1 and concrete in ("fused_stepwise", "fused_one_launch", "p2p_unfused",
                                  "ce_unfused"):
        from multi_gpu_flashattention_b200.parallel.ring import P_ENGINES, _meta
        nbytes = k.numel() * k.element_size()
        eng = P_ENGINES.get(group, dev, nbytes) if concrete == "fused_one_launch" else \
            ENGINES.get(group, dev, nbytes)
        qtp, kvtp, kv_lens = _meta(lay, rank, dev)
        def compute_only():
            return eng.forward_compute_only(q, k, v, 1.0 / math.sqrt(D), causal,
                                            qtp if causal else None, kvtp if causal else None,
                                            kv_lens, status)
        for _ in range(2):
            compute_only()
        cs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        ce = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        barrier()
        for i in range(args.steps):
            flush.fill_(i & 0xFF)
            cs[i].record()
            compute_only()
            ce[i].record()
        torch.cuda.synchronize()
        barrier()
        t_c = max_over_ranks([a.elapsed_time(b) for a, b in zip(cs, ce)])
        t_comp = sum(t_c) / len(t_c)
        exposed = max(0.0, (ms - t_comp) / ms * 100.0)

    # ---------------- end to end through the public API (pinned H2D + D2H each step)
    # Every step uploads its q/k/v from pinned host memory and downloads its
    # output; uploads of step i+1 and the download of step i run on copy streams
    # while step i computes (double-buffered device inputs), as an input
    # pipeline would. Timed from the first upload to the last download.
    e2e = None
    if not args.no_e2e:
        hq = q.cpu().pin_memory(); hk = k.cpu().pin_memory(); hv = v.cpu().pin_memory()
        ho = [torch.empty(q.shape, dtype=q.dtype, pin_memory=True) for _ in range(2)]
        dbuf = [(torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)) for _ in range(2)]
        comp = torch.cuda.current_stream()
        up, down = torch.cuda.Stream(), torch.cuda.Stream()

        def e2e_run(n):
            ev_in = [torch.cuda.Event() for _ in range(n)]
            ev_used = [torch.cuda.Event() for _ in range(n)]
            ev_out = [torch.cuda.Event() for _ in range(n)]
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record(up)

            def upload(i):
                with torch.cuda.stream(up):
                    if i >= 2:
                        up.wait_event(ev_used[i - 2])  # buffer i%2 free again
                    for d, h in zip(dbuf[i % 2], (hq, hk, hv)):
                        d.copy_(h, non_blocking=True)
                    ev_in[i].record(up)
            upload(0)
            for i in range(n):
                if i + 1 < n:
                    upload(i + 1)
                comp.wait_event(ev_in[i])
                dq, dk, dv = dbuf[i % 2]
                out = mgfa.ring_attention(dq, dk, dv, causal=causal, group=group, layout=lay,
                                          backend=args.backend)
                ev_used[i].record(comp)
                with torch.cuda.stream(down):
                    down.wait_event(ev_used[i])
                    ho[i % 2].copy_(out, non_blocking=True)
                    out.record_stream(down)
                    ev_out[i].record(down)
            t1.record(down)
            return t0, t1

        e2e_run(2)
        torch.cuda.synchronize()
        barrier()
        t0, t1 = e2e_run(args.steps)
        torch.cuda.synchronize()
        barrier()
        e2e_ms = max_over_ranks([t0.elapsed_time(t1) / args.steps])[0]
        bi = (hq.numel() + hk.numel() + hv.numel()) * hq.element_size()
        bo = ho[0].numel() * ho[0].element_size()
        e2e = (e2e_ms, bi, bo)

    # ---------------- report
    if rank == 0:
        pairs = S * (S + 1) // 2 if causal else S * S
        flops = 4.0 * D * H * B * pairs
        tflops_total = flops / (ms * 1e-3) / 1e12
        peaks_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
        peak = json.load(open(peaks_path))["bf16_tflops_sustained"] if os.path.exists(peaks_path) else 1400.0
        comm_bytes = (world - 1) * 2 * B * L * Hkv * D * 2
        t_roof = max(flops / world / (peak * 1e12), comm_bytes / 770e9) * 1e3
        # the one-launch ring runs one kernel per forward (so does a single GPU);
        # the per-step engines and the baselines one attention kernel per step
        launches_per_step = 1 if concrete == "fused_one_launch" or world == 1 else world
        rec = {
            "metric": METRIC,
            "value": round(tflops_total, 2),
            "unit": "TFLOP/s (attention, summed over GPUs)",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms, 3),
            "tflops_per_gpu": round(tflops_total / world, 2),
            "exposed_comm_pct": None if exposed is None else round(exposed, 2),
            "roofline_fraction": round(t_roof / ms, 3),
            "roofline_note": "max(FLOPs/GPU / measured sustained bf16 peak, KV bytes / 770 GB/s)",
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "baseline_note": "the reference publishes no number for this config (fp32 1-head "
                             "d64 non-causal only, on 2x GTX 1660 Ti)",
            "dtype": "bf16",
            "data": "synthetic: seeded N(0,1)*0.5 q/k/v, no weights (attention op)",
            "impl": "ours",
            "backend": concrete,
            "config": {"model": f"ring attention fwd, causal={causal}, {H} q heads / {Hkv} kv "
                                f"heads x d{D}",
                       "global_batch": B, "seq_len": S,
                       "parallelism": f"cp{world} ring ({lay.kind})",
                       "l2": "flushed between timed steps (256 MB write, outside the events)"},
            "clocks": clocks,
            "gpu_launches": launches_per_step * args.steps,
            "wall_s_timed_region": round(wall, 3),
        }
        if e2e is not None:
            e2e_ms, bi, bo = e2e
            rec["e2e"] = {"value": round(flops / (e2e_ms * 1e-3) / 1e12, 2),
                          "unit": "TFLOP/s (attention, summed over GPUs)",
                          "ms_per_step": round(e2e_ms, 3),
                          "h2d_bytes_per_step": bi, "d2h_bytes_per_step": bo,
                          "path": "multi_gpu_flashattention_b200.ring_attention; every step "
                                  "uploads q/k/v from pinned host memory and downloads the "
                                  "output (copy streams overlap step i+1's upload and step i's "
                                  "download with step i's compute)"}
        print(json.dumps(rec), flush=True)
    if world > 1:
        from multi_gpu_flashattention_b200.parallel.ring import P_ENGINES
        ENGINES.clear()
        P_ENGINES.clear()
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
