"""examples/train_ring_lm.py on 2 gloo ranks (fp32 `torch` ring backend): the
loss starts near ln(vocab) and falls as the model learns the synthetic
pattern, through the public model, layout and ring-attention API."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_train_example_learns():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", "29793",
           os.path.join(ROOT, "examples", "train_ring_lm.py"), "--seq", "512", "--layers", "2",
           "--d-model", "64", "--heads", "4", "--kv-heads", "2", "--head-dim", "16",
           "--steps", "25", "--lr", "3e-3", "--vocab", "128"]
    p = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=300,
                       env=dict(os.environ, OMP_NUM_THREADS="1", CUDA_VISIBLE_DEVICES=""))
    assert p.returncode == 0, p.stdout + p.stderr
    rec = json.loads([l for l in p.stdout.splitlines() if l.startswith("{")][-1])
    assert rec["world"] == 2 and rec["backend"] == "torch"
    assert abs(rec["first_loss"] - rec["uniform_loss"]) < 0.5
    assert rec["last_loss"] < 0.6 * rec["first_loss"]


def _train(tmp_path, port, extra):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(port),
           os.path.join(ROOT, "examples", "train_ring_lm.py"), "--seq", "256", "--layers", "2",
           "--d-model", "64", "--heads", "4", "--kv-heads", "2", "--head-dim", "16",
           "--lr", "3e-3", "--vocab", "128"] + extra
    p = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=300,
                       env=dict(os.environ, OMP_NUM_THREADS="1", CUDA_VISIBLE_DEVICES=""))
    assert p.returncode == 0, p.stdout + p.stderr
    return [l for l in p.stdout.splitlines() if l.startswith("step")]


def test_checkpoint_resume_continues_exactly(tmp_path):
    """Four steps, a checkpoint, four resumed steps: the same step lines (and
    losses) as eight uninterrupted steps."""
    ck = str(tmp_path / "ck.pt")
    full = _train(tmp_path, 29794, ["--steps", "8"])
    first = _train(tmp_path, 29795, ["--steps", "4", "--save", ck])
    second = _train(tmp_path, 29796, ["--steps", "4", "--resume", ck])
    assert first + second == full


def test_quickstart_example_matches_single_device():
    """examples/ring_attention_quickstart.py on 3 gloo ranks: the gathered
    output and query gradient match attention over the whole sequence."""
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=3",
           "--master-addr", "127.0.0.1", "--master-port", "29797",
           os.path.join(ROOT, "examples", "ring_attention_quickstart.py"), "--seq", "384",
           "--heads", "4", "--kv-heads", "2", "--head-dim", "32"]
    p = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=300,
                       env=dict(os.environ, OMP_NUM_THREADS="1", CUDA_VISIBLE_DEVICES=""))
    assert p.returncode == 0, p.stdout + p.stderr
    line = [l for l in p.stdout.splitlines() if l.startswith("world=3")][0]
    vals = dict(kv.split("=") for kv in line.split() if kv.startswith("max"))
    assert float(vals["max|out-ref|"]) < 1e-5 and float(vals["max|dq-ref|"]) < 1e-5
