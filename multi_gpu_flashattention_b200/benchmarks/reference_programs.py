"""Runs the reference prototype's own benchmark programs, built unmodified by
benchmarks/build_reference.sh (MPI from this repository's MPI subset), and
prints one JSON line per run, so they can be set beside this framework's
numbers from the same box.

    python -m multi_gpu_flashattention_b200.benchmarks.reference_programs \
        --program ring_loop_nccl --gpus 2 --sizes 1M,16M,256M [--warmup 10 --iters 100]

Programs (ring/loop and ring/attention/bench in the reference):
  ring_loop_nccl, ring_loop_cuda_aware, ring_loop_cuda_aware_Isendrecv,
  ring_loop_staged, ring_loop_staged_Isendrecv
      pure ring exchange; their `RESULT backend=... avg_*_ms ... GBps` line
  ring_attention_nccl_gpu_bench, ring_attention_cuda_aware_gpu_bench,
  ring_attention_cuda_aware_Isendrecv_gpu_bench,
  ring_attention_cuda_aware_Isendrecv_overlap_gpu_bench,
  ring_attention_staged_gpu_bench, ring_attention_staged_Isendrecv_gpu_bench,
  ring_attention_staged_Isendrecv_overlap_gpu_bench
      ring attention (fp32, one head, head_dim 64, non-causal, K=V); their
      `avg_total=... ms avg_<comm>=...` line

Each size is the program's own positional argument: bytes of one rank's KV
shard (fp32), a multiple of 256 for the attention programs. The launcher is
`torchrun --no-python` with one rank per GPU on 127.0.0.1. In the MPI subset,
device buffers move by CUDA IPC and copy-engine copies with a shared-memory
mailbox for control, and host buffers through that mailbox or a TCP store, so
the "CUDA-aware" and "staged" timings measure that transport, not an MPI
library's.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
LOOP = ["ring_loop_nccl", "ring_loop_cuda_aware", "ring_loop_cuda_aware_Isendrecv",
        "ring_loop_staged", "ring_loop_staged_Isendrecv"]
ATTN = ["ring_attention_nccl_gpu_bench", "ring_attention_cuda_aware_gpu_bench",
        "ring_attention_cuda_aware_Isendrecv_gpu_bench",
        "ring_attention_cuda_aware_Isendrecv_overlap_gpu_bench",
        "ring_attention_staged_gpu_bench", "ring_attention_staged_Isendrecv_gpu_bench",
        "ring_attention_staged_Isendrecv_overlap_gpu_bench"]

_RESULT = re.compile(r"^RESULT (.*)$", re.M)
_AVG = re.compile(r"avg_total=([\d.]+) ms ((?:avg_[\w-]+=[\d.]+\s*)+)")


def bin_dir() -> str:
    return os.environ.get("MGFA_REF_BIN", os.path.join(ROOT, "baseline", "_ref", "bin"))


def parse_size(text: str) -> int:
    m = re.fullmatch(r"(\d+)([KMG]?)", text.strip(), re.I)
    if not m:
        raise ValueError(f"bad size {text!r}")
    return int(m.group(1)) << {"": 0, "K": 10, "M": 20, "G": 30}[m.group(2).upper()]


def parse_output(program: str, text: str) -> dict:
    """The program's result line as a dict of numbers (and the backend name)."""
    if program in LOOP:
        m = _RESULT.search(text)
        if not m:
            raise ValueError("no RESULT line")
        out = {}
        for kv in m.group(1).split():
            k, v = kv.split("=", 1)
            try:
                out[k] = float(v) if "." in v else int(v)
            except ValueError:
                out[k] = v
        return out
    m = _AVG.search(text)
    if not m:
        raise ValueError("no avg_total line")
    out = {"avg_total_ms": float(m.group(1))}
    for kv in m.group(2).split():
        k, v = kv.split("=", 1)
        out[k.lower().replace("-", "_") + "_ms"] = float(v)
    return out


def run(program: str, gpus: int, size: int, warmup: int, iters: int, port: int,
        timeout: float) -> dict:
    exe = os.path.join(bin_dir(), program)
    rec = {"impl": "reference", "program": program, "n_gpus": gpus, "bytes": size,
           "warmup": warmup, "iters": iters}
    if not os.path.exists(exe):
        rec["unavailable"] = "not built (benchmarks/build_reference.sh)"
        return rec
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={gpus}", "--master-addr", "127.0.0.1", "--master-port", str(port),
           "--no-python", exe, str(size), str(warmup), str(iters)]
    try:
        p = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, cwd=ROOT)
        text, rc = p.stdout + p.stderr, p.returncode
    except subprocess.TimeoutExpired:
        text, rc = f"timed out after {timeout} s", -1
    try:
        if rc != 0:
            raise ValueError(f"exit {rc}")
        rec.update(parse_output(program, text))
        if program in ATTN:
            seq = gpus * size // 256  # tokens in the whole ring (fp32 x 64 per token)
            flops = 4.0 * 64 * seq * seq
            rec["seq_len"] = seq
            rec["tflops_total"] = flops / (rec["avg_total_ms"] * 1e-3) / 1e12
    except ValueError as e:
        tail = " | ".join(text.strip().splitlines()[-3:])
        rec["unavailable"] = f"{e}: {tail}"[:400]
    return rec


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--program", required=True, choices=LOOP + ATTN)
    ap.add_argument("--gpus", type=int, default=2)
    ap.add_argument("--sizes", default="256K")
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--iters", type=int, default=100)
    ap.add_argument("--port", type=int, default=29620)
    ap.add_argument("--timeout", type=float, default=600.0)
    a = ap.parse_args(argv)
    bad = 0
    for i, s in enumerate(a.sizes.split(",")):
        rec = run(a.program, a.gpus, parse_size(s), a.warmup, a.iters, a.port + i, a.timeout)
        bad += "unavailable" in rec
        print(json.dumps(rec), flush=True)
    return 1 if bad else 0


if __name__ == "__main__":
    sys.exit(main())
