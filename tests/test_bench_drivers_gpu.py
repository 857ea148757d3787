"""The Python benchmark drivers (benchmarks.ring_attention, benchmarks.ring_loop)
under torchrun on 2+ GPUs: their output lines, and the fp32 dumps through the
reference checker."""
import os
import socket
import subprocess
import sys

import pytest

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _module(mod, args, cwd, env=None, nproc=2):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={nproc}", "--master-addr=127.0.0.1", f"--master-port={_port()}",
           "-m", mod] + [str(a) for a in args]
    e = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    e.update(env or {})
    p = subprocess.run(cmd, capture_output=True, text=True, cwd=cwd, env=e, timeout=600)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-3000:]
    return p.stdout


@pytest.mark.parametrize("backend", ["nccl", "staged", "p2p"])
def test_python_ring_attention_fp32_dumps_pass_verify_full(tmp_path, backend):
    size = 1024 * 64 * 4
    out = _module("multi_gpu_flashattention_b200.benchmarks.ring_attention",
                  [size, 1, 2, "--backend", backend], tmp_path,
                  env={"ATTENTION_DUMP_OUTPUT": "1", "ATTENTION_PRINT_SHARDS": "1"})
    assert f"{backend} bench: warmup=1 iters=2" in out and "avg_total=" in out
    vf = os.path.join(ROOT, "build", "bin", "verify_full")
    if not os.path.exists(vf):
        pytest.skip("verify_full not built")
    p = subprocess.run([vf, str(tmp_path), "2", str(size)], capture_output=True, text=True,
                       timeout=300)
    assert p.returncode == 0 and "ALL PASS" in p.stdout, p.stdout[-2000:]


def test_python_ring_attention_bf16_json():
    import json
    size = 2048 * 4 * 128 * 4
    out = _module("multi_gpu_flashattention_b200.benchmarks.ring_attention",
                  [size, 1, 2, "--numerics", "bf16", "--init", "randn", "--causal",
                   "--layout", "zigzag", "--heads", 4, "--backend", "fused", "--json"], ROOT)
    rec = json.loads([l for l in out.splitlines() if l.startswith("{")][-1])
    assert rec["ranks"] == 2 and rec["tflops_per_gpu"] > 0 and rec["ring_ms"] > 0


@pytest.mark.parametrize("backend", ["p2p", "ce", "nccl", "staged"])
def test_python_ring_loop_result_line(backend):
    out = _module("multi_gpu_flashattention_b200.benchmarks.ring_loop",
                  [1 << 20, 2, 3, "--backend", backend], ROOT)
    line = [l for l in out.splitlines() if l.startswith("RESULT")]
    assert len(line) == 1 and f"backend={backend}" in line[0]
