"""Failure detection on CPU ranks (gloo): the failure is made on the host --
a rank that raises, leaves, or goes silent -- and the others must end with an
error instead of hanging."""
import time

import pytest
import torch

from dist_utils import run_ranks


def _raising_rank(rank, world):
    from multi_gpu_flashattention_b200.parallel.layouts import RingLayout
    from multi_gpu_flashattention_b200.parallel.ring import ring_attention_forward
    lay = RingLayout("contiguous", 256, world, mask="full")
    q = torch.randn(1, 128, 1, 16)
    if rank == 1:
        raise RuntimeError("injected failure on rank 1")
    ring_attention_forward(q, q, q, lay, backend="torch")  # rank 0 waits for rank 1


def test_rank_exception_ends_peers_with_error():
    t0 = time.monotonic()
    with pytest.raises(AssertionError) as e:
        run_ranks(_raising_rank, 2, pg_timeout=5, timeout=90)
    assert "injected failure on rank 1" in str(e.value)
    assert time.monotonic() - t0 < 90


def _finish(rank, store, key):
    """Rank 0 marks that it has seen the failure; every rank's process stays
    until then and tears its process group down locally."""
    import torch.distributed as dist
    if rank == 0:
        store.set(key, "1")
    else:
        store.wait([key])
    dist.destroy_process_group()


def _leaving_rank(rank, world):
    import torch.distributed as dist
    from multi_gpu_flashattention_b200.parallel.health import PeerLostError, RingHealth
    h = RingHealth()
    h.step(0, timeout_s=20)          # both ranks take call 0
    if rank == 1:
        h.leave()                    # leaves between calls, nothing in flight
    else:
        h.beat(1)
        with pytest.raises(PeerLostError, match="rank 1 left"):
            h.check(1, timeout_s=20)
    _finish(rank, dist.distributed_c10d._get_default_store(), "test/leave_seen")


def test_health_detects_departed_rank():
    run_ranks(_leaving_rank, 2, final_barrier=False)


def _silent_rank(rank, world):
    import torch.distributed as dist
    from multi_gpu_flashattention_b200.parallel.health import PeerLostError, RingHealth
    h = RingHealth()
    h.step(0, timeout_s=20)
    if rank == 0:                    # rank 1 never announces call 1
        h.beat(1)
        t0 = time.monotonic()
        with pytest.raises(PeerLostError, match="did not reach call 1"):
            h.check(1, timeout_s=1.0)
        assert time.monotonic() - t0 < 3
    _finish(rank, dist.distributed_c10d._get_default_store(), "test/silence_seen")


def test_health_times_out_on_silent_rank():
    run_ranks(_silent_rank, 2, final_barrier=False)


def _gated_ring(rank, world):
    """A rank leaves after the first call; the other learns it at its next
    call's gate, before any transfer is started."""
    from multi_gpu_flashattention_b200 import ring_attention
    from multi_gpu_flashattention_b200.parallel.health import PeerLostError, RingHealth
    from multi_gpu_flashattention_b200.parallel.layouts import RingLayout
    lay = RingLayout("zigzag", 256, world, mask="causal")
    h = RingHealth()
    q = torch.randn(1, lay.max_local_len, 2, 16, requires_grad=True)
    import torch.distributed as dist
    store = dist.distributed_c10d._get_default_store()
    out = ring_attention(q, q, q, causal=True, layout=lay, backend="torch", health=h)
    out.sum().backward()  # forward and backward each pass the gate (calls 0 and 1)
    if rank == 1:
        h.leave()
    else:
        t0 = time.monotonic()
        with pytest.raises(PeerLostError, match="left"):
            ring_attention(q, q, q, causal=True, layout=lay, backend="torch", health=h)
        assert time.monotonic() - t0 < 10
    _finish(rank, store, "test/gate_seen")


def test_health_gate_stops_the_next_call():
    run_ranks(_gated_ring, 2, final_barrier=False)
