"""benchmarks.reference_programs: launching the reference's programs (one per
torchrun rank, positional SIZE WARMUP ITERS) and parsing their result lines,
with stand-in programs that print the reference's exact line formats
(ring/loop/ring_loop_cuda_aware.cu:226-231, ring/attention/bench/
ring_attention_cuda_aware_gpu_bench.cu and ring_attention_staged_gpu_bench.cu
avg_total lines)."""
import os
import stat

import pytest

from multi_gpu_flashattention_b200.benchmarks import reference_programs as rp

LOOP_LINE = ("RESULT backend=cuda_aware bytes=$1 ranks=$WORLD_SIZE warmup=$2 iters=$3 "
             "avg_mpi_ms=0.500 avg_total_ms=0.600 total_GBps=1.748 mpi_GBps=2.097")
ATTN_LINES = {
    "ring_attention_cuda_aware_gpu_bench":
        "avg_total=10.000 ms avg_CUDA-aware=1.000 avg_attn=8.000 avg_merge=0.500 avg_final=0.500",
    "ring_attention_staged_gpu_bench":
        "avg_total=12.000 ms avg_D2H=1.000 avg_MPI=1.000 avg_H2D=1.000 avg_attn=8.000 "
        "avg_merge=0.500 avg_final=0.500",
}


def _fake(tmp_path, name, line):
    exe = tmp_path / name
    exe.write_text(f'#!/bin/sh\nif [ "$RANK" = "0" ]; then echo "{line}"; fi\n')
    exe.chmod(exe.stat().st_mode | stat.S_IEXEC)


def test_parse_sizes():
    assert rp.parse_size("256K") == 262144 and rp.parse_size("16M") == 16 << 20
    assert rp.parse_size("1000") == 1000
    with pytest.raises(ValueError):
        rp.parse_size("12Q")


def test_loop_program(tmp_path, monkeypatch):
    _fake(tmp_path, "ring_loop_cuda_aware", LOOP_LINE)
    monkeypatch.setenv("MGFA_REF_BIN", str(tmp_path))
    rec = rp.run("ring_loop_cuda_aware", 2, 1 << 20, 3, 7, 29781, 120)
    assert rec["backend"] == "cuda_aware" and rec["bytes"] == 1 << 20
    assert rec["ranks"] == 2 and rec["warmup"] == 3 and rec["iters"] == 7
    assert rec["avg_total_ms"] == 0.6 and rec["mpi_GBps"] == 2.097


@pytest.mark.parametrize("name", list(ATTN_LINES))
def test_attention_program(tmp_path, monkeypatch, name):
    _fake(tmp_path, name, ATTN_LINES[name])
    monkeypatch.setenv("MGFA_REF_BIN", str(tmp_path))
    rec = rp.run(name, 2, 262144, 1, 2, 29782, 120)
    assert rec["seq_len"] == 2048
    assert rec["avg_attn_ms"] == 8.0
    if "staged" in name:
        assert rec["avg_total_ms"] == 12.0 and rec["avg_h2d_ms"] == 1.0
    else:
        assert rec["avg_total_ms"] == 10.0 and rec["avg_cuda_aware_ms"] == 1.0
    want = 4.0 * 64 * 2048 * 2048 / (rec["avg_total_ms"] * 1e-3) / 1e12
    assert abs(rec["tflops_total"] - want) < 1e-9


def test_missing_program(tmp_path, monkeypatch):
    monkeypatch.setenv("MGFA_REF_BIN", str(tmp_path))
    rec = rp.run("ring_loop_nccl", 2, 1024, 1, 1, 29783, 60)
    assert "unavailable" in rec


def test_build_script_reports_a_missing_reference_tree(tmp_path):
    """benchmarks/build_reference.sh exits 2 (the callers' 'skip' signal) when
    no reference tree is found, and builds nothing."""
    import subprocess
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, REF_SRC=str(tmp_path / "absent"), OUT=str(tmp_path / "out"))
    for args in ([], ["--cpu-only"], ["--print-src"]):
        p = subprocess.run(["bash", "benchmarks/build_reference.sh"] + args, cwd=root, env=env,
                           capture_output=True, text=True, timeout=120)
        assert p.returncode == 2, (args, p.stdout, p.stderr)
    assert not (tmp_path / "out").exists()
