"""Legacy CPU-compute ring (one-shot driver, --cpu mode) on gloo ranks, and the
C++ host attention against a float64 PyTorch reference."""
import os
import subprocess

import numpy as np
import pytest
import torch

from dist_utils import run_ranks

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _ref_attention(q, k, v, scale):
    s = (q.double() @ k.double().T) * scale
    return torch.softmax(s, dim=-1) @ v.double()


def test_cpu_attention_partial_merge_normalize():
    from multi_gpu_flashattention_b200._ext import sched
    S = sched()
    g = torch.Generator().manual_seed(0)
    sq, sk, d = 77, 130, 64
    q = torch.randn(sq, d, generator=g)
    k1, v1 = torch.randn(sk, d, generator=g), torch.randn(sk, d, generator=g)
    k2, v2 = torch.randn(50, d, generator=g), torch.randn(50, d, generator=g)
    m = torch.full((sq,), -torch.finfo(torch.float32).max)
    l, acc = torch.zeros(sq), torch.zeros(sq, d)
    ml, ll, al = torch.empty(sq), torch.empty(sq), torch.empty(sq, d)
    for k, v in ((k1, v1), (k2, v2)):
        S.cpu_attention_partial(q.numpy(), k.numpy(), v.numpy(), sq, k.shape[0], d, 0.125,
                                al.numpy(), ml.numpy(), ll.numpy(), 3)
        S.cpu_merge_online_softmax(m.numpy(), l.numpy(), acc.numpy(), ml.numpy(), ll.numpy(),
                                   al.numpy(), sq, d)
    S.cpu_normalize(acc.numpy(), l.numpy(), sq, d)
    ref = _ref_attention(q, torch.cat([k1, k2]), torch.cat([v1, v2]), 0.125)
    torch.testing.assert_close(acc.double(), ref, rtol=1e-4, atol=1e-5)
    s = (q.double() @ torch.cat([k1, k2]).double().T) * 0.125
    torch.testing.assert_close(m.double(), s.max(-1).values, rtol=1e-5, atol=1e-5)


def test_cpu_attention_rejects_short_buffer():
    from multi_gpu_flashattention_b200._ext import sched
    S = sched()
    a = np.zeros(10, dtype=np.float32)
    with pytest.raises(ValueError):
        S.cpu_attention_partial(a, a, a, 4, 4, 4, 1.0, a, a, a)


def _oneshot_rank(rank, world, out_dir, seq):
    from multi_gpu_flashattention_b200.benchmarks import common, ring_oneshot
    args = ring_oneshot.parse(["--cpu", "--attention", "cpu", "--backend", "staged",
                               "--seq", str(seq), "--out-dir", out_dir])
    ctx = common.Ctx(rank, world, torch.device("cpu"), None)
    ring_oneshot.run(ctx, args)


@pytest.mark.parametrize("world", [2, 3])
def test_oneshot_cpu_ring_matches_full_attention(tmp_path, world):
    from multi_gpu_flashattention_b200.benchmarks.ring_oneshot import legacy_inputs
    seq, dim = 128, 64
    run_ranks(_oneshot_rank, world, str(tmp_path), seq)
    kv_all = torch.cat([legacy_inputs(r, seq, dim)[1] for r in range(world)])
    for r in range(world):
        got = torch.from_numpy(np.fromfile(tmp_path / f"ring_output_rank{r}.bin", dtype="<f4"))
        q = legacy_inputs(r, seq, dim)[0]
        ref = _ref_attention(q, kv_all, kv_all, 1.0).float().view(-1)
        err = (got - ref).abs().max().item()
        assert err < 0.05, (r, err)


def test_oneshot_dumps_pass_verify_full(tmp_path):
    """The reference's checker rule (verify_full) accepts the one-shot dumps."""
    exe = os.path.join(ROOT, "build", "bin", "verify_full")
    if not os.path.exists(exe):
        exe = str(tmp_path / "verify_full")
        src = [os.path.join(ROOT, "csrc/bench/verify_full.cpp")] + [
            os.path.join(ROOT, "csrc/sched", f)
            for f in ("scheduler.cpp", "workload.cpp", "shard_plan.cpp")]
        subprocess.check_call(["g++", "-O2", "-std=c++17", "-pthread", "-o", exe] + src)
    seq, world = 1024, 2
    out = tmp_path / "dumps"
    out.mkdir()
    run_ranks(_oneshot_rank, world, str(out), seq)
    p = subprocess.run([exe, str(out), str(world), str(seq * 64 * 4)], capture_output=True,
                       text=True)
    assert p.returncode == 0, p.stdout + p.stderr
    assert "ALL PASS" in p.stdout


def _probe_rank(rank, world, which):
    import torch
    from multi_gpu_flashattention_b200.benchmarks import probes
    lines = []
    if which == "ring_test":
        got = probes.ring_test(rank, world, log=lines.append)
        left = (rank - 1) % world
        assert got.tolist() == [left * 100.0 + i for i in range(4)]
        assert lines[-1] == f"[Rank {rank}] recv_buf = [{', '.join(str(left * 100 + i) for i in range(4))}]"
    else:
        got = probes.ring_cuda(rank, world, torch.device("cpu"), log=lines.append)
        left = (rank - 1) % world
        assert got[:4].tolist() == [left * 1000.0 + i for i in range(4)]
        assert got[-1].item() == left * 1000.0 + 128 * 8 * 64 - 1
        assert "first 4 values" in lines[-1]


@pytest.mark.parametrize("which,world", [("ring_test", 3), ("ring_cuda", 2)])
def test_transport_probes(which, world):
    run_ranks(_probe_rank, world, which)


def test_native_and_python_oneshot_dumps_identical(tmp_path):
    """The native one-shot ring (build/bin/ring_oneshot --cpu) and the Python
    driver run the same host attention on the same inputs: their dumps agree
    bit for bit."""
    import sys
    exe = os.path.join(ROOT, "build", "bin", "ring_oneshot")
    if not os.path.exists(exe):
        pytest.skip("ring_oneshot not built (make cuda-tools)")
    seq, world = 256, 3
    py_dir, nat_dir = tmp_path / "py", tmp_path / "native"
    py_dir.mkdir()
    nat_dir.mkdir()
    run_ranks(_oneshot_rank, world, str(py_dir), seq)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1", "--master-port", "29798",
           "--no-python", exe, "--attention", "cpu", "--cpu", "--seq", str(seq), "--out-dir",
           str(nat_dir)]
    p = subprocess.run(cmd, capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert p.returncode == 0, p.stdout + p.stderr
    for r in range(world):
        a = (py_dir / f"ring_output_rank{r}.bin").read_bytes()
        b = (nat_dir / f"ring_output_rank{r}.bin").read_bytes()
        assert len(a) == seq * 64 * 4 and a == b, r
