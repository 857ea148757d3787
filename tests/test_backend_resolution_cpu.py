"""Backend names of the ring API (host only): "fused" is the per-step fused ring
unless MGFA_RING_ENGINE selects the one-launch ring, None picks the fused ring
on CUDA and the fp32 torch ring elsewhere, and every listed backend resolves to
itself."""
import pytest

from multi_gpu_flashattention_b200.parallel import ring


def test_default_fused_is_the_per_step_ring(monkeypatch):
    monkeypatch.setattr(ring, "RING_ENGINE", "stepwise")
    assert ring.resolve_backend("fused") == "fused_stepwise"
    assert ring.resolve_backend(None) == "fused_stepwise"
    assert ring.resolve_backend(None, is_cuda=False) == "torch"


def test_engine_variable_selects_the_one_launch_ring(monkeypatch):
    monkeypatch.setattr(ring, "RING_ENGINE", "one_launch")
    assert ring.resolve_backend("fused") == "fused_one_launch"
    assert ring.resolve_backend(None) == "fused_one_launch"


@pytest.mark.parametrize("name", [b for b in ring.BACKENDS if b != "fused"])
def test_concrete_backends_resolve_to_themselves(name, monkeypatch):
    for engine in ("stepwise", "one_launch"):
        monkeypatch.setattr(ring, "RING_ENGINE", engine)
        assert ring.resolve_backend(name) == name
