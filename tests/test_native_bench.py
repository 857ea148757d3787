"""Native benchmark executables (build/bin/ring_loop_bench, ring_attention_bench)
launched by torchrun --no-python: argument handling on the host, and on 2+ GPUs
the RESULT lines, the reference checker on fp32 dumps and the bf16 dumps
against the fp32 oracle."""
import os
import re
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "build", "bin")


def _exe(name):
    p = os.path.join(BIN, name)
    if not os.path.exists(p):
        pytest.skip(f"{name} not built (make cuda-tools)")
    return p


def test_usage_and_bad_arguments():
    for name in ("ring_loop_bench", "ring_attention_bench"):
        exe = _exe(name)
        p = subprocess.run([exe, "--no-such-flag"], capture_output=True, text=True, timeout=60)
        assert p.returncode == 1 and "Usage:" in p.stdout


@pytest.mark.parametrize("nproc", [2, 3])
def test_oneshot_native_host_ring(tmp_path, nproc):
    """build/bin/ring_oneshot --cpu: the CPU-attention legacy ring on host
    memory only (staged transport through the MPI subset), the reference's
    per-step lines, and dumps that pass verify_full."""
    exe = _exe("ring_oneshot")
    out = _torchrun(exe, ["--attention", "cpu", "--cpu", "--seq", "384", "--out-dir",
                          str(tmp_path)], nproc, tmp_path)
    for r in range(nproc):
        assert f"[Rank {r}] step 0: attention on own KV" in out
        for s in range(1, nproc):
            assert f"[Rank {r}] step {s}: KV from rank {(r - s) % nproc} | MPI=" in out
        assert f"[Rank {r}] output dumped to ring_output_rank{r}.bin" in out
    v = subprocess.run([_exe("verify_full"), str(tmp_path), str(nproc), str(384 * 64 * 4)],
                       capture_output=True, text=True, timeout=300)
    assert v.returncode == 0 and "Overall: ALL PASS" in v.stdout, v.stdout


def test_oneshot_native_arguments():
    exe = _exe("ring_oneshot")
    p = subprocess.run([exe, "--backend", "bogus"], capture_output=True, text=True, timeout=60)
    assert p.returncode == 1 and "Usage:" in p.stdout
    p = subprocess.run([exe, "--cpu", "--attention", "gpu"], capture_output=True, text=True,
                       timeout=60)
    assert p.returncode == 1
    p = subprocess.run([exe, "--attention", "cpu", "--cpu"], capture_output=True, text=True,
                       timeout=60, env={k: v for k, v in os.environ.items() if k != "WORLD_SIZE"})
    assert p.returncode == 1 and "Need at least 2 processes" in p.stdout


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _torchrun(exe, args, nproc, cwd, env=None, timeout=300):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={nproc}", "--master-addr=127.0.0.1", f"--master-port={_port()}",
           "--no-python", exe] + [str(a) for a in args]
    e = dict(os.environ)
    e.update(env or {})
    p = subprocess.run(cmd, capture_output=True, text=True, cwd=cwd, env=e, timeout=timeout)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-3000:]
    return p.stdout


def _world():
    return min(torch.cuda.device_count(), 4)


@pytest.mark.gpu
@pytest.mark.multigpu
@pytest.mark.parametrize("backend", ["p2p", "ce", "nccl", "staged"])
def test_ring_loop_bench(tmp_path, backend):
    out = _torchrun(_exe("ring_loop_bench"), [1 << 20, 2, 3, "--backend", backend], _world(),
                    tmp_path)
    line = [l for l in out.splitlines() if l.startswith("RESULT")]
    assert len(line) == 1 and f"backend={backend}" in line[0] and f"ranks={_world()}" in line[0]


@pytest.mark.gpu
@pytest.mark.multigpu
def test_ring_loop_bench_payload_mode(tmp_path):
    out = _torchrun(_exe("ring_loop_bench"), [0, 1, 2, "--payload-tokens", 256], _world(), tmp_path)
    assert f"bytes={256 * 8 * 128 * 4}" in out


@pytest.mark.gpu
@pytest.mark.multigpu
@pytest.mark.parametrize("extra", [["--backend", "nccl"], ["--backend", "staged"],
                                   ["--backend", "nccl", "--overlap"], ["--backend", "p2p"],
                                   ["--backend", "ce"]])
def test_ring_attention_bench_fp32_passes_verify_full(tmp_path, extra):
    size = 1024 * 64 * 4
    out = _torchrun(_exe("ring_attention_bench"), [size, 1, 2] + extra, _world(), tmp_path,
                    env={"ATTENTION_DUMP_OUTPUT": "1", "ATTENTION_PRINT_SHARDS": "1"})
    assert "avg_total=" in out
    assert "kv_owner=" in out  # ATTENTION_PRINT_SHARDS step lines
    vf = os.path.join(BIN, "verify_full")
    if not os.path.exists(vf):
        pytest.skip("verify_full not built")
    p = subprocess.run([vf, str(tmp_path), str(_world()), str(size)], capture_output=True,
                       text=True, timeout=300)
    assert p.returncode == 0 and "ALL PASS" in p.stdout, p.stdout[-2000:]


@pytest.mark.gpu
@pytest.mark.multigpu
@pytest.mark.parametrize("backend,layout", [("fused", "zigzag"), ("nccl", "zigzag"),
                                            ("staged", "contiguous")])
def test_ring_attention_bench_bf16_dumps(tmp_path, backend, layout):
    from multi_gpu_flashattention_b200._ext import sched
    from multi_gpu_flashattention_b200.ops.reference import attention_ref
    from multi_gpu_flashattention_b200.parallel.layouts import RingLayout
    P, H, D, L = _world(), 2, 128, 1024
    size = L * H * D * 4
    _torchrun(_exe("ring_attention_bench"),
              [size, 1, 2, "--numerics", "bf16", "--init", "randn", "--backend", backend,
               "--layout", layout, "--causal", "--heads", H, "--seed", 3, "--json"],
              P, tmp_path, env={"ATTENTION_DUMP_OUTPUT": "1"})
    seq = L * P
    S = sched()
    full = []
    for stream in (0, 1, 2):
        buf = np.empty(seq * H * D, dtype=np.float32)
        S.fill_randn_rows(buf, 3, stream, list(range(seq)), H * D)
        full.append(torch.from_numpy(buf).view(1, seq, H, D).bfloat16())
    ref, _ = attention_ref(*full, causal=True)
    lay = RingLayout(layout, seq, P)
    for r in range(P):
        got = torch.from_numpy(np.fromfile(tmp_path / f"ring_output_rank{r}.bin", dtype="<f4"))
        got = got.view(-1, H, D)[: lay.local_len(r)]
        exp = lay.shard(ref, r)[0, : lay.local_len(r)]
        err = (got - exp).abs().max().item()
        assert err < 2e-2, (r, err)


@pytest.mark.parametrize("layout,world,causal", [("contiguous", 2, False), ("contiguous", 3, True),
                                                 ("zigzag", 2, True), ("zigzag", 4, True),
                                                 ("striped", 3, True), ("scheduler", 4, True),
                                                 ("scheduler", 3, False)])
def test_native_layout_tables_match_python(layout, world, causal):
    """The native benchmark's kernel tables (tile positions per owner, mask
    positions, lengths) equal the Python layer's for every layout."""
    import json
    from multi_gpu_flashattention_b200.parallel.layouts import RingLayout
    exe = _exe("ring_attention_bench")
    H, D, L = 2, 64, 768
    args = [exe, str(L * H * D * 4), "--print-tables", str(world), "--layout", layout,
            "--heads", str(H), "--head-dim", str(D)] + (["--causal"] if causal else [])
    p = subprocess.run(args, capture_output=True, text=True, timeout=60)
    assert p.returncode == 0, p.stdout + p.stderr
    rows = [json.loads(l) for l in p.stdout.splitlines()]
    lay = RingLayout(layout, L * world, world, mask="causal" if causal else "full")
    assert len(rows) == world
    for r, row in enumerate(rows):
        assert row["L"] == lay.max_local_len and row["local_len"] == lay.local_len(r)
        assert row["q_tile_pos"] == lay.q_tile_pos(r, "cpu").tolist()
        assert row["kv_tile_pos"] == lay.kv_tile_pos_by_owner(r, "cpu").tolist()
        assert row["q_positions"] == lay.q_positions_for_mask(r).tolist()
        assert row["k_positions"] == [lay.k_positions_for_mask(r, o).tolist()
                                      for o in range(world)]


@pytest.mark.gpu
@pytest.mark.multigpu
@pytest.mark.parametrize("extra", [["--backend", "nccl"], ["--backend", "staged"],
                                   ["--backend", "nccl", "--overlap"], ["--backend", "p2p"]])
def test_fp32_randn_seq4096_two_ranks(tmp_path, extra):
    """fp32 N(0,1) q/k/v (seed 0), 1 head x d64, 4096 tokens over 2 ranks in
    contiguous 2048-token shards, scale 1/8, non-causal: every rank's dump within
    1e-4 (max abs) of the full single-device fp32 reference."""
    import re
    size = 2048 * 64 * 4
    _torchrun(_exe("ring_attention_bench"),
              [size, 1, 2, "--init", "randn", "--seed", 0] + extra, 2, tmp_path,
              env={"ATTENTION_DUMP_OUTPUT": "1"})
    vf = os.path.join(BIN, "verify_full")
    if not os.path.exists(vf):
        pytest.skip("verify_full not built")
    p = subprocess.run([vf, str(tmp_path), "2", str(size), "--init", "randn", "--seed", "0"],
                       capture_output=True, text=True, timeout=300)
    assert p.returncode == 0 and "ALL PASS" in p.stdout, p.stdout[-2000:]
    errs = [float(x) for x in re.findall(r"Max absolute error:\s*([0-9.eE+-]+)", p.stdout)]
    assert len(errs) == 2 and max(errs) <= 1e-4, errs


def test_check_peer_runs():
    p = subprocess.run([_exe("check_peer")], capture_output=True, text=True, timeout=60)
    assert p.returncode == 0
    for line in p.stdout.splitlines():
        assert re.fullmatch(r"GPU \d+ -> GPU \d+: (YES|NO)", line), line


@pytest.mark.gpu
@pytest.mark.multigpu
def test_check_peer_lists_every_pair():
    n = torch.cuda.device_count()
    p = subprocess.run([_exe("check_peer")], capture_output=True, text=True, timeout=60)
    lines = p.stdout.splitlines()
    assert len(lines) == n * (n - 1)
    assert lines[0] == "GPU 0 -> GPU 1: YES"


@pytest.mark.parametrize("nproc", [2, 3])
def test_dist_layer_under_torchrun(tmp_path, nproc):
    """The native tools' process-group layer on CPU: torchrun's store, barriers,
    all-gather, MAX reductions, host send/recv around the ring."""
    out = _torchrun(_exe("dist_selftest"), [], nproc, tmp_path, timeout=120)
    assert out.count("dist selftest ok") == nproc


def test_dist_layer_with_rank0_hosting_the_store():
    exe = _exe("dist_selftest")
    port = _port()
    env = dict(os.environ, WORLD_SIZE="2", MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    env.pop("TORCHELASTIC_USE_AGENT_STORE", None)
    procs = [subprocess.Popen([exe], env=dict(env, RANK=str(r), LOCAL_RANK=str(r)),
                              stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)
             for r in range(2)]
    outs = [p.communicate(timeout=120) for p in procs]
    assert all(p.returncode == 0 for p in procs), outs
    assert all("dist selftest ok" in o for o, _ in outs)
