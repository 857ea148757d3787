"""bench.py --impl reference: how the reference's NCCL ring-attention benchmark
is launched (one program per rank, per-rank KV bytes for the total sequence,
the driver's warm-up and step counts) and how its `avg_total=... avg_NCCL=...`
line becomes the JSON record. A stand-in program prints that line, so the test
needs no GPU; the real program is exercised by the driver's reference arm."""
import json
import os
import stat
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

FAKE = """#!/bin/sh
echo "args $1 $2 $3 rank $RANK local $MPI_LOCALRANKID" >> "$(dirname "$0")/calls.txt"
if [ "$RANK" = "0" ]; then
  echo "nccl bench: warmup=$2 iters=$3"
  echo "avg_total=2000.000 ms avg_NCCL=100.000 avg_attn=1800.000 avg_merge=50.000 avg_final=50.000"
fi
"""


def _run(tmp_path, nproc, port, extra=()):
    exe = tmp_path / "ring_attention_nccl_gpu_bench"
    exe.write_text(FAKE)
    exe.chmod(exe.stat().st_mode | stat.S_IEXEC)
    env = dict(os.environ, MGFA_REF_BIN=str(tmp_path), OMP_NUM_THREADS="1")
    if nproc == 1:
        cmd = [sys.executable, "bench.py"]
    else:
        cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
               f"--nproc-per-node={nproc}", "--master-addr", "127.0.0.1",
               "--master-port", str(port), "bench.py"]
    cmd += ["--impl", "reference", "--gpus", str(nproc), "--steps", "4", "--warmup", "3",
            *extra]
    p = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    lines = [l for l in p.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, p.stdout + p.stderr
    return json.loads(lines[0]), (tmp_path / "calls.txt")


def test_reference_arm_record(tmp_path):
    rec, calls = _run(tmp_path, 2, 29761)
    S = 131072
    assert rec["impl"] == "reference" and rec["n_gpus"] == 2
    assert rec["ms_per_step"] == 2000.0
    assert abs(rec["value"] - 4.0 * 64 * S * S / 2.0 / 1e12) < 1e-3
    assert rec["exposed_comm_pct"] == 5.0
    assert rec["dtype"] == "fp32" and rec["steps"] == 4 and rec["warmup"] == 3
    kv = S // 2 * 64 * 4
    got = sorted(calls.read_text().splitlines())
    assert got == [f"args {kv} 3 4 rank 0 local 0", f"args {kv} 3 4 rank 1 local 1"]


def test_reference_arm_one_gpu_unavailable(tmp_path):
    rec, calls = _run(tmp_path, 1, 0)
    assert "unavailable" in rec and "at least 2 ranks" in rec["unavailable"]
    assert not calls.exists()


HANG = """#!/bin/sh
if [ "$RANK" = "0" ]; then echo "failing on purpose"; exit 3; fi
sleep 600
"""


def test_failed_rank_ends_the_others(tmp_path):
    """Rank 0's program fails while rank 1's would wait for it forever: the
    launcher ends rank 1 and its program within seconds, not at the timeout."""
    import time
    exe = tmp_path / "ring_attention_nccl_gpu_bench"
    exe.write_text(HANG)
    exe.chmod(exe.stat().st_mode | stat.S_IEXEC)
    env = dict(os.environ, MGFA_REF_BIN=str(tmp_path), OMP_NUM_THREADS="1")
    t0 = time.time()
    p = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                        "--nproc-per-node=2", "--master-addr", "127.0.0.1",
                        "--master-port", "29762", "bench.py", "--impl", "reference",
                        "--gpus", "2", "--steps", "1", "--warmup", "3"],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert time.time() - t0 < 120
    line = [l for l in p.stdout.splitlines() if l.startswith("{")][0]
    assert "failing on purpose" in json.loads(line)["unavailable"]
    ps = subprocess.run(["pgrep", "-f", str(exe)], capture_output=True, text=True)
    assert ps.stdout.strip() == "", "a reference program outlived its rank"
