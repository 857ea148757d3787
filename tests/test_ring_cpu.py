"""Ring protocol, layouts and LSE merging on CPU ranks (gloo) against exact attention."""
import pytest
import torch

from dist_utils import run_ranks


def _ring_case(rank, world, kind, causal, seq, heads, kv_heads):
    from multi_gpu_flashattention_b200.ops.reference import attention_ref
    from multi_gpu_flashattention_b200.parallel.layouts import RingLayout
    from multi_gpu_flashattention_b200.parallel.ring import ring_attention_forward
    g = torch.Generator().manual_seed(1234)
    q = torch.randn(1, seq, heads, 16, generator=g)
    k = torch.randn(1, seq, kv_heads, 16, generator=g)
    v = torch.randn(1, seq, kv_heads, 16, generator=g)
    lay = RingLayout(kind, seq, world, block=32, mask="causal" if causal else "full")
    ql, kl, vl = lay.shard(q, rank), lay.shard(k, rank), lay.shard(v, rank)
    out, lse = ring_attention_forward(ql, kl, vl, lay, causal=causal, backend="torch")
    ref, ref_lse = attention_ref(q, k, v, causal=causal)
    n = lay.local_len(rank)
    exp = lay.shard(ref, rank)[:, :n]
    torch.testing.assert_close(out[:, :n], exp, rtol=1e-5, atol=1e-5)
    exp_lse = lay.shard(ref_lse.transpose(1, 2), rank)[:, :n].transpose(1, 2)
    torch.testing.assert_close(lse[:, :, :n], exp_lse, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("kind", ["contiguous", "zigzag", "striped", "scheduler"])
@pytest.mark.parametrize("causal", [True, False])
def test_ring_torch_backend_world2(kind, causal):
    run_ranks(_ring_case, 2, kind, causal, 256, 2, 1)


@pytest.mark.parametrize("kind", ["zigzag", "striped", "scheduler"])
def test_ring_torch_backend_world4_causal_gqa(kind):
    run_ranks(_ring_case, 4, kind, True, 512, 4, 2)


def _host_group_case(rank, world):
    import torch.distributed as dist
    from multi_gpu_flashattention_b200.parallel.ring import _host_group
    # a gloo default group carries host buffers itself
    assert _host_group(None) is None
    sub = dist.new_group([0, 1], backend="gloo")
    assert _host_group(sub) is sub


def test_staged_transport_host_group_selection():
    from dist_utils import run_ranks
    run_ranks(_host_group_case, 2)
