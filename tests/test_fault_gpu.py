"""Failure paths on the GPU without faulting it: bounded waits that expire on a
flag nothing sets, a dropped transport signal, and a rank that leaves between
calls. Multi-GPU cases run as child processes with NVLS off."""
import pytest
import torch

from dist_utils import run_ranks

pytestmark = pytest.mark.gpu


def test_bounded_wait_expires_with_status_and_context_survives():
    from multi_gpu_flashattention_b200._ext import C
    from multi_gpu_flashattention_b200.ops.flash import check_status, flash_attn_fwd
    q = (torch.randn(1, 256, 1, 128, device="cuda") * 0.5).bfloat16()
    status = C().fwd_timeout_probe(q, q, q, 200_000_000)  # 0.2 s limit
    torch.cuda.synchronize()
    word = int(status.item())
    assert word & 0xFF == 2, f"expected a peer-flag timeout, got {word:#x}"
    assert (word >> 8) & 0xFF == 8  # the TMA producer's wait
    # the context is still usable
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    o, _ = flash_attn_fwd(q, q, q, status=st)
    check_status(st)
    assert torch.isfinite(o.float()).all()


def test_public_call_raises_error_of_an_earlier_kernel():
    """A kernel whose bounded wait expires while reporting into the public API's
    status word (the device's StatusMonitor) makes a later public call raise
    KernelStatusError before it launches anything; the word is re-armed and
    the next call runs clean."""
    from multi_gpu_flashattention_b200._ext import C
    from multi_gpu_flashattention_b200.ops.flash import (KernelStatusError, check_errors,
                                                         flash_attn_fwd, status_monitor)
    q = (torch.randn(1, 256, 1, 128, device="cuda") * 0.5).bfloat16()
    check_errors()
    mon = status_monitor(q.device)
    C().fwd_timeout_probe(q, q, q, 200_000_000, mon.word)  # records a peer-flag timeout
    flash_attn_fwd(q, q, q)  # runs behind it; its read-back carries the sticky word
    torch.cuda.synchronize()  # (a user's loss.item() or the like)
    with pytest.raises(KernelStatusError, match="peer flag wait timed out"):
        flash_attn_fwd(q, q, q)
    o, _ = flash_attn_fwd(q, q, q)
    check_errors()
    assert torch.isfinite(o.float()).all()


def _drop_signal_public(rank, world, backend):
    """A dropped push signal surfaces through mgfa.ring_attention() itself (no
    check=True, no status argument): the receiving rank's next public call
    raises, and reset_ring() re-arms the ring on both ranks. Both fused engines:
    the per-step ring (one chunk of step 0 never signalled) and the one-launch
    ring (one part of kv head 0's step-0 unit never signalled)."""
    import multi_gpu_flashattention_b200 as mgfa
    from multi_gpu_flashattention_b200.ops.flash import KernelStatusError, check_errors
    from multi_gpu_flashattention_b200.parallel.ring import ENGINES, P_ENGINES, reset_ring
    dev = torch.device("cuda", rank)
    g = torch.Generator(device=dev).manual_seed(rank)
    q = (torch.randn(1, 512, 2, 128, device=dev, generator=g) * 0.5).bfloat16()
    out_ok = mgfa.ring_attention(q, q, q, backend=backend)
    check_errors()
    one = backend == "fused_one_launch"
    eng = (P_ENGINES if one else ENGINES).get(None, dev, q.numel() * 2)
    drop = (lambda on: eng.set_drop_signal(on)) if one else \
        (lambda on: eng.set_drop_signal_step(0 if on else -1))
    if rank == 0:
        drop(True)
    mgfa.ring_attention(q, q, q, backend=backend)
    drop(False)
    torch.cuda.synchronize()
    if rank == 1:
        with pytest.raises(KernelStatusError, match="peer flag wait timed out"):
            mgfa.ring_attention(q, q, q, backend=backend)
    else:
        check_errors()  # the sending side finished its work
    reset_ring()
    out = mgfa.ring_attention(q, q, q, backend=backend)
    check_errors()
    torch.testing.assert_close(out, out_ok, rtol=0, atol=0)


@pytest.mark.multigpu
@pytest.mark.parametrize("backend", ["fused", pytest.param("fused_one_launch", marks=pytest.mark.xfail(
    reason="one-launch ring: intermittent wrong second query tile on a fresh ring "
           "(the error itself is raised; the re-armed ring's output is what fails)",
    strict=False))])
def test_dropped_signal_raises_through_public_ring_attention(backend):
    run_ranks(_drop_signal_public, 2, backend, backend="nccl",
              env={"NCCL_NVLS_ENABLE": "0", "MGFA_WAIT_LIMIT_NS": "300000000"})


def _drop_signal(rank, world):
    from multi_gpu_flashattention_b200.ops.flash import KernelStatusError
    from multi_gpu_flashattention_b200.parallel.layouts import RingLayout
    from multi_gpu_flashattention_b200.parallel.ring import ENGINES, ring_attention_forward
    dev = torch.device("cuda", rank)
    lay = RingLayout("contiguous", 1024, world, mask="full")
    g = torch.Generator(device=dev).manual_seed(rank)
    q = (torch.randn(1, 512, 2, 128, device=dev, generator=g) * 0.5).bfloat16()
    out_ok, _ = ring_attention_forward(q, q, q, lay, backend="fused_stepwise", check=True)
    eng = ENGINES.get(None, dev, q.numel() * 2)
    if rank == 0:
        eng.set_drop_signal_step(0)  # rank 1 never hears about one chunk of step 0
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    if rank == 1:
        with pytest.raises(KernelStatusError, match="peer flag wait timed out"):
            ring_attention_forward(q, q, q, lay, backend="fused_stepwise", status=st,
                                   wait_limit_ns=300_000_000, check=True)
    else:
        ring_attention_forward(q, q, q, lay, backend="fused_stepwise", status=st,
                               wait_limit_ns=300_000_000, check=True)
    # recover: every rank idle, flags re-armed, then a clean call matches the first
    eng.set_drop_signal_step(-1)
    torch.cuda.synchronize()
    torch.distributed.barrier()
    eng.reset()
    torch.cuda.synchronize()
    torch.distributed.barrier()
    out, _ = ring_attention_forward(q, q, q, lay, backend="fused_stepwise", check=True)
    torch.testing.assert_close(out, out_ok, rtol=0, atol=0)


@pytest.mark.multigpu
def test_dropped_signal_times_out_and_ring_recovers():
    run_ranks(_drop_signal, 2, backend="nccl", env={"NCCL_NVLS_ENABLE": "0"})


def _leave_between_calls(rank, world):
    from multi_gpu_flashattention_b200.parallel.health import PeerLostError, RingHealth
    from multi_gpu_flashattention_b200.parallel.layouts import RingLayout
    from multi_gpu_flashattention_b200.parallel.ring import ring_attention_forward
    dev = torch.device("cuda", rank)
    lay = RingLayout("contiguous", 1024, world, mask="full")
    q = (torch.randn(1, 512, 1, 128, device=dev) * 0.5).bfloat16()
    import torch.distributed as dist
    store = dist.distributed_c10d._get_default_store()
    h = RingHealth()
    h.step(0)
    ring_attention_forward(q, q, q, lay, backend="fused", check=True)
    torch.cuda.synchronize()  # nothing of ours in flight past this point
    if rank == 1:
        h.leave()
        store.wait(["test/leave_seen"])  # the process stays until rank 0 saw it
    else:
        h.beat(1)
        with pytest.raises(PeerLostError):
            h.check(1, timeout_s=20)  # rank 0 learns it on the host and launches nothing
        store.set("test/leave_seen", "1")
    dist.destroy_process_group()


@pytest.mark.multigpu
def test_rank_leaving_between_calls_is_detected_before_launch():
    run_ranks(_leave_between_calls, 2, backend="nccl", final_barrier=False,
              env={"NCCL_NVLS_ENABLE": "0"})
