"""Ring attention on 2+ GPUs (one process per GPU, NCCL for bootstrap/baselines):
fused in-kernel transport and the NCCL baseline against exact fp32 attention."""
import pytest
import torch

from dist_utils import run_ranks

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _case(rank, world, kind, causal, backend, seq, hq, hkv, iters):
    from multi_gpu_flashattention_b200.ops.reference import attention_ref
    from multi_gpu_flashattention_b200.parallel.layouts import RingLayout
    from multi_gpu_flashattention_b200.parallel.ring import ring_attention_forward
    dev = torch.device("cuda", rank)
    g = torch.Generator(device=dev).manual_seed(99)
    q = (torch.randn(1, seq, hq, 128, device=dev, generator=g) * 0.5).bfloat16()
    k = (torch.randn(1, seq, hkv, 128, device=dev, generator=g) * 0.5).bfloat16()
    v = (torch.randn(1, seq, hkv, 128, device=dev, generator=g) * 0.5).bfloat16()
    lay = RingLayout(kind, seq, world, mask="causal" if causal else "full")
    ql, kl, vl = lay.shard(q, rank), lay.shard(k, rank), lay.shard(v, rank)
    ref, ref_lse = attention_ref(q, k, v, causal=causal)
    n = lay.local_len(rank)
    exp = lay.shard(ref, rank)[:, :n]
    k0, v0 = kl.clone(), vl.clone()
    for _ in range(iters):  # repeated calls reuse the slots and flags
        out, lse = ring_attention_forward(ql, kl, vl, lay, causal=causal, backend=backend,
                                          check=True)
        assert torch.equal(kl, k0) and torch.equal(vl, v0), "inputs must not be written"
        err = (out[:, :n].float() - exp).abs()
        assert err.max().item() < 2e-2, (rank, err.max().item())
        assert err.mean().item() < 2e-3, (rank, err.mean().item())
    exp_lse = lay.shard(ref_lse.transpose(1, 2), rank)[:, :n].transpose(1, 2)
    torch.testing.assert_close(lse[:, :, :n], exp_lse, rtol=0, atol=2e-3)


# The one-launch ring (backend "fused_one_launch", opt-in) has an open defect: on
# a fresh or re-armed engine, whose push warps start together with the compute,
# the second query tile of an item is intermittently wrong (no status raised).
# Its result checks are expected failures until that is fixed.
ONE_LAUNCH = pytest.param("fused_one_launch", marks=pytest.mark.xfail(
    reason="one-launch ring: intermittent wrong second query tile on a fresh ring",
    strict=False))


def _rearmed_case(rank, world, push_ctas):
    """Re-arm the one-launch ring before every call (its push warps then start
    with the compute) and count calls whose output has a wrong query tile."""
    from multi_gpu_flashattention_b200.ops.reference import attention_ref
    from multi_gpu_flashattention_b200.parallel.layouts import RingLayout
    from multi_gpu_flashattention_b200.parallel.ring import (P_ENGINES, reset_ring,
                                                             ring_attention_forward)
    dev = torch.device("cuda", rank)
    seq = 512 * world
    g = torch.Generator(device=dev).manual_seed(5)
    q = (torch.randn(1, seq, 2, 128, device=dev, generator=g) * 0.5).bfloat16()
    k = (torch.randn(1, seq, 2, 128, device=dev, generator=g) * 0.5).bfloat16()
    v = (torch.randn(1, seq, 2, 128, device=dev, generator=g) * 0.5).bfloat16()
    lay = RingLayout("contiguous", seq, world, mask="full")
    ql, kl, vl = lay.shard(q, rank), lay.shard(k, rank), lay.shard(v, rank)
    exp = lay.shard(attention_ref(q, k, v)[0], rank)
    P_ENGINES.get(None, dev, kl.numel() * kl.element_size()).set_push_ctas(push_ctas)
    # candidates for a wrong row: attention over the rank's own shard only, over
    # the other shards only, and exact (all keys)
    own = slice(rank * 512, rank * 512 + 512)
    mask_own = torch.zeros(seq, dtype=torch.bool, device=dev)
    mask_own[own] = True

    def nearest(row, h, got):
        qrow = q[0, rank * 512 + row, h].float()
        kk, vv = k[0, :, h].float(), v[0, :, h].float()
        sc = (kk @ qrow) * 128 ** -0.5
        cands = {"exact": torch.ones_like(mask_own), "own_shard_only": mask_own,
                 "other_shards_only": ~mask_own}
        dist = {}
        for name, m in cands.items():
            pr = torch.softmax(sc.masked_fill(~m, float("-inf")), 0)
            dist[name] = round((got - pr @ vv).abs().max().item(), 4)
        return dist

    bad = []
    for it in range(10):
        reset_ring()
        out, _ = ring_attention_forward(ql, kl, vl, lay, causal=False,
                                        backend="fused_one_launch", check=True)
        err = (out.float() - exp).abs()
        rows = (err.amax(dim=(0, 2, 3)) > 2e-2).nonzero().flatten().tolist()
        tiles = sorted({int(r) // 128 for r in rows})
        if tiles:
            r0 = int(rows[0])
            h0 = int(err[0, r0].amax(dim=1).argmax())
            bad.append((it, tiles, {"row": r0, "head": h0,
                                    "distance_to": nearest(r0, h0, out[0, r0, h0].float())}))
    P_ENGINES.get(None, dev, kl.numel() * kl.element_size()).set_push_ctas(0)
    assert not bad, f"rank {rank}: calls with wrong query tiles {bad}"


@pytest.mark.parametrize("push_ctas", [0, 8])
@pytest.mark.xfail(reason="one-launch ring: intermittent wrong second query tile on a fresh "
                          "ring (push_ctas=8 separates pushing and computing CTAs)",
                   strict=False)
def test_one_launch_rearmed_calls(push_ctas):
    run_ranks(_rearmed_case, min(_world(), 2), push_ctas, backend="nccl")


def _world():
    # every visible GPU, up to MGFA_TEST_MAX_WORLD (default 8), so an 8-GPU run
    # tests the ring at P = 8
    import os
    return min(torch.cuda.device_count(), int(os.environ.get("MGFA_TEST_MAX_WORLD", "8")))


@pytest.mark.parametrize("backend", ["fused", "fused_stepwise", ONE_LAUNCH, "p2p_unfused",
                                     "ce_unfused", "nccl"])
@pytest.mark.parametrize("kind,causal", [("zigzag", True), ("striped", True),
                                         ("contiguous", False), ("contiguous", True)])
def test_ring_forward_matches_reference(backend, kind, causal):
    run_ranks(_case, _world(), kind, causal, backend, 4096, 4, 2, 3, backend="nccl")


def test_ring_forward_cumulative_arrival_counts():
    """Arrival counters that keep growing (cumulative targets): repeated calls
    stay correct with dependent launch on."""
    run_ranks(_case, _world(), "zigzag", True, "fused_stepwise", 4096, 4, 2, 4, backend="nccl",
              env={"MGFA_CUMULATIVE_ARRIVALS": "1"})


@pytest.mark.parametrize("backend", ["fused_one_launch", "fused_stepwise"])
def test_ring_forward_scheduler_layout_fused(backend):
    run_ranks(_case, _world(), "scheduler", True, backend, 4096, 2, 2, 2, backend="nccl")


def test_ring_forward_one_launch_gqa_batch_and_many_calls():
    """The one-launch ring with GQA (8 query heads on 2 kv heads), ragged
    striped shards and six calls in a row (slots, arrivals, tags and the call
    credit are reused every call)."""
    run_ranks(_case, _world(), "striped", True, "fused_one_launch", 5000, 8, 2, 6, backend="nccl")


def _bwd_case(rank, world, kind, causal, bwd_backend="nccl", head_dim=128,
              dtype=torch.bfloat16):
    from multi_gpu_flashattention_b200.ops.reference import attention_ref
    from multi_gpu_flashattention_b200.parallel.layouts import RingLayout
    from multi_gpu_flashattention_b200.parallel.ring import ring_attention_forward
    from multi_gpu_flashattention_b200.parallel.ring_bwd import ring_attention_backward
    dev = torch.device("cuda", rank)
    seq, hq, hkv = 2048, 4, 2
    g = torch.Generator(device=dev).manual_seed(5)
    mk = lambda h: (torch.randn(1, seq, h, head_dim, device=dev, generator=g) * 0.5).to(dtype)
    q, k, v, do = mk(hq), mk(hkv), mk(hkv), mk(hq)
    lay = RingLayout(kind, seq, world, mask="causal" if causal else "full")
    ql, kl, vl, dol = (lay.shard(t, rank) for t in (q, k, v, do))
    k0, v0 = kl.clone(), vl.clone()
    out, lse = ring_attention_forward(ql, kl, vl, lay, causal=causal, backend="fused", check=True)
    assert out.dtype == dtype
    if head_dim != 128 or dtype != torch.bfloat16:
        ref, _ = attention_ref(q, k, v, causal=causal)
        m = lay.local_len(rank)
        err = (out[:, :m].float() - lay.shard(ref, rank)[:, :m]).abs().max().item()
        assert err < 2e-2, (rank, "out", err)
    dq, dk, dv = ring_attention_backward(dol, ql, kl, vl, out, lse, lay, causal=causal,
                                         backend=bwd_backend)
    # no backend writes the caller's k / v (autograd saved them)
    assert torch.equal(kl, k0) and torch.equal(vl, v0), rank
    rq, rk, rv = ring_attention_backward(dol, ql, kl, vl, out, lse, lay, causal=causal,
                                         backend="torch")
    n = lay.local_len(rank)
    for name, a, b in (("dq", dq, rq), ("dk", dk, rk), ("dv", dv, rv)):
        a, b = a[:, :n].float(), b[:, :n].float()
        err = (a - b).abs().max().item()
        assert err <= 3e-2 * b.abs().max().item() + 1e-3, (rank, name, err)


@pytest.mark.parametrize("bwd_backend", ["fused", "nccl"])
@pytest.mark.parametrize("kind,causal", [("zigzag", True), ("contiguous", False),
                                         ("striped", True)])
def test_ring_backward_matches_reference(kind, causal, bwd_backend):
    run_ranks(_bwd_case, _world(), kind, causal, bwd_backend, backend="nccl")


@pytest.mark.parametrize("head_dim,dtype", [(64, torch.bfloat16), (64, torch.float16),
                                           (128, torch.float16)])
def test_ring_fused_head_dim_and_dtype(head_dim, dtype):
    run_ranks(_bwd_case, _world(), "zigzag", True, "fused", head_dim, dtype, backend="nccl")


def _bwd_repeat_case(rank, world):
    """Repeated fused backward calls reuse slots, home buffer and flags."""
    from multi_gpu_flashattention_b200.parallel.layouts import RingLayout
    from multi_gpu_flashattention_b200.parallel.ring import ring_attention_forward
    from multi_gpu_flashattention_b200.parallel.ring_bwd import ring_attention_backward
    dev = torch.device("cuda", rank)
    lay = RingLayout("zigzag", 4096, world, mask="causal")
    g = torch.Generator(device=dev).manual_seed(17 + rank)
    mk = lambda h: (torch.randn(1, lay.max_local_len, h, 128, device=dev, generator=g) * 0.5).bfloat16()
    q, k, v, do = mk(4), mk(2), mk(2), mk(4)
    out, lse = ring_attention_forward(q, k, v, lay, causal=True, backend="fused", check=True)
    ref = ring_attention_backward(do, q, k, v, out, lse, lay, causal=True, backend="fused")
    for _ in range(3):
        got = ring_attention_backward(do, q, k, v, out, lse, lay, causal=True, backend="fused")
        for a, b in zip(got, ref):
            torch.testing.assert_close(a, b, rtol=0, atol=0)


def test_ring_backward_fused_repeated_calls():
    run_ranks(_bwd_repeat_case, _world(), backend="nccl")


def _trace_case(rank, world):
    from multi_gpu_flashattention_b200.parallel.layouts import RingLayout
    from multi_gpu_flashattention_b200.parallel.ring import ENGINES, ring_attention_forward
    from multi_gpu_flashattention_b200.utils.trace import summarize, to_chrome_events
    dev = torch.device("cuda", rank)
    lay = RingLayout("zigzag", 4096, world, mask="causal")
    q = (torch.randn(1, lay.max_local_len, 2, 128, device=dev) * 0.5).bfloat16()
    ring_attention_forward(q, q, q, lay, causal=True, backend="fused_stepwise", check=True)
    eng = ENGINES.get(None, dev, q.numel() * 2)
    eng.set_trace(True)
    ring_attention_forward(q, q, q, lay, causal=True, backend="fused_stepwise", check=True)
    eng.set_trace(False)
    tr = eng.last_trace()
    assert tr.shape[0] == world and tr.shape[2] == 8
    assert (tr[..., 6] >= tr[..., 1]).all() and (tr[..., 6] > 0).all()
    pushed = tr[: world - 1, :, 4] > 0
    assert pushed.all(), "every CTA of a pushing step records its push"
    assert (tr[world - 1, :, 4] == 0).all(), "the last step pushes nothing"
    ev = to_chrome_events(tr, rank)
    assert any(e["name"] == "push" for e in ev)
    assert len(summarize(tr)["steps"]) == world


def test_ring_forward_trace_records_timeline():
    run_ranks(_trace_case, _world(), backend="nccl")


def _trace_case_one_launch(rank, world):
    from multi_gpu_flashattention_b200.parallel.layouts import RingLayout
    from multi_gpu_flashattention_b200.parallel.ring import P_ENGINES, ring_attention_forward
    dev = torch.device("cuda", rank)
    lay = RingLayout("zigzag", 8192, world, mask="causal")
    q = (torch.randn(1, lay.max_local_len, 4, 128, device=dev) * 0.5).bfloat16()
    ring_attention_forward(q, q, q, lay, causal=True, backend="fused_one_launch", check=True)
    eng = P_ENGINES.get(None, dev, q.numel() * 2)
    eng.set_trace(True)
    ring_attention_forward(q, q, q, lay, causal=True, backend="fused_one_launch", check=True)
    eng.set_trace(False)
    tr = eng.last_trace().cpu()
    assert tr.shape == (eng.grid(), 8)
    assert (tr[:, 2] >= tr[:, 1]).all() and (tr[:, 1] > 0).all()
    assert int(tr[:, 3].sum()) == 4 * ((lay.max_local_len + 255) // 256), "every item ran once"
    pushed = tr[:, 6] > 0
    assert pushed.sum() >= min(eng.grid(), 128), "push warps record their push window"
    assert (tr[pushed, 7] >= tr[pushed, 6]).all()


def test_ring_forward_one_launch_trace():
    run_ranks(_trace_case_one_launch, _world(), backend="nccl")


def _poison_case(rank, world, backend):
    """NaN-poisoned receive slots must never leak into the output (no read races
    ahead of its data), and every slot carries the right owner tag."""
    from multi_gpu_flashattention_b200.parallel.layouts import RingLayout
    from multi_gpu_flashattention_b200.parallel.ring import (ENGINES, P_ENGINES,
                                                             ring_attention_forward)
    dev = torch.device("cuda", rank)
    lay = RingLayout("zigzag", 8192, world, mask="causal")
    g = torch.Generator(device=dev).manual_seed(rank)
    q = (torch.randn(1, lay.max_local_len, 4, 128, device=dev, generator=g) * 0.5).bfloat16()
    ref, _ = ring_attention_forward(q, q, q, lay, causal=True, backend=backend, check=True)
    engines = P_ENGINES if backend == "fused_one_launch" else ENGINES
    eng = engines.get(None, dev, q.numel() * 2)
    for _ in range(3):
        torch.cuda.synchronize()
        torch.distributed.barrier()
        eng.poison_slots()
        torch.cuda.synchronize()
        torch.distributed.barrier()
        out, _ = ring_attention_forward(q, q, q, lay, causal=True, backend=backend, check=True)
        assert torch.isfinite(out.float()).all()
        torch.testing.assert_close(out, ref, rtol=0, atol=0)


@pytest.mark.parametrize("ring_backend", [ONE_LAUNCH, "fused_stepwise"])
def test_ring_forward_poisoned_slots_and_tags(ring_backend):
    run_ranks(_poison_case, _world(), ring_backend, backend="nccl")


def _oneshot_case(rank, world, attention, backend, out_dir):
    import numpy as np
    import torch.distributed as dist
    from multi_gpu_flashattention_b200.benchmarks import common, ring_oneshot
    torch.cuda.set_device(rank)
    ctx = common.Ctx(rank, world, torch.device("cuda", rank), dist.new_group(backend="gloo"))
    args = ring_oneshot.parse(["--attention", attention, "--backend", backend, "--seq", "1024",
                               "--out-dir", out_dir])
    ring_oneshot.run(ctx, args)
    seq, dim = 1024, 64
    kv = torch.cat([ring_oneshot.legacy_inputs(r, seq, dim)[1] for r in range(world)]).double()
    q = ring_oneshot.legacy_inputs(rank, seq, dim)[0].double()
    ref = torch.softmax(q @ kv.T, dim=-1) @ kv
    got = torch.from_numpy(np.fromfile(f"{out_dir}/ring_output_rank{rank}.bin", dtype="<f4"))
    err = (got.double() - ref.view(-1)).abs().max().item()
    assert err < 0.05, (rank, attention, backend, err)


@pytest.mark.parametrize("attention,backend", [("gpu", "staged"), ("gpu", "nccl"),
                                               ("gpu", "p2p"), ("cpu", "nccl")])
def test_oneshot_legacy_ring(tmp_path, attention, backend):
    run_ranks(_oneshot_case, _world(), attention, backend, str(tmp_path), backend="nccl")
