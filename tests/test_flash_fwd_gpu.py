"""sm_100a tcgen05 attention forward against the fp32 PyTorch oracle."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _C():
    from multi_gpu_flashattention_b200._ext import C
    return C()


def _inputs(B, Sq, Sk, Hq, Hkv, seed=0, scale=0.5):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = (torch.randn(B, Sq, Hq, 128, device="cuda", generator=g) * scale).bfloat16()
    k = (torch.randn(B, Sk, Hkv, 128, device="cuda", generator=g) * scale).bfloat16()
    v = (torch.randn(B, Sk, Hkv, 128, device="cuda", generator=g) * scale).bfloat16()
    return q, k, v


def test_umma_probe_matches_matmul():
    torch.manual_seed(0)
    a = torch.randn(128, 64, device="cuda").bfloat16()
    b = torch.randn(128, 64, device="cuda").bfloat16()
    v = torch.randn(64, 128, device="cuda").bfloat16()
    c1, c2, status = _C().umma_probe(a, b, v)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref1 = a.float() @ b.float().t()
    ref2 = a.float() @ v.float()
    torch.testing.assert_close(c1, ref1, rtol=1e-3, atol=1e-3)
    torch.testing.assert_close(c2, ref2, rtol=1e-3, atol=1e-3)


def _check(o, lse, q, k, v, causal, q_pos=None, k_pos=None):
    from multi_gpu_flashattention_b200.ops.reference import attention_ref
    ref_o, ref_lse = attention_ref(q, k, v, causal=causal, q_pos=q_pos, k_pos=k_pos)
    err = (o.float() - ref_o).abs()
    assert err.max().item() < 2e-2, f"max err {err.max().item()}"
    assert err.mean().item() < 2e-3, f"mean err {err.mean().item()}"
    finite = torch.isfinite(ref_lse)
    assert torch.equal(finite, torch.isfinite(lse))
    torch.testing.assert_close(lse[finite], ref_lse[finite], rtol=0, atol=2e-3)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("B,S,Hq,Hkv", [(1, 256, 2, 2), (2, 512, 4, 1), (1, 384, 2, 2),
                                        (1, 1024, 1, 1)])
def test_flash_fwd_self_attention(B, S, Hq, Hkv, causal):
    from multi_gpu_flashattention_b200.ops.flash import check_status, flash_attn_fwd
    q, k, v = _inputs(B, S, S, Hq, Hkv)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    o, lse = flash_attn_fwd(q, k, v, causal=causal, status=status)
    check_status(status)
    _check(o, lse, q, k, v, causal)


def test_flash_fwd_ragged_lengths():
    from multi_gpu_flashattention_b200.ops.flash import check_status, flash_attn_fwd
    q, k, v = _inputs(1, 200, 333, 2, 2, seed=3)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    o, lse = flash_attn_fwd(q, k, v, causal=False, status=status)
    check_status(status)
    _check(o, lse, q, k, v, False)


def test_flash_fwd_tile_positions_mask():
    """Causal mask driven by non-contiguous tile positions (zigzag-like shard)."""
    from multi_gpu_flashattention_b200.ops.flash import check_status, flash_attn_fwd
    q, k, v = _inputs(1, 256, 512, 2, 2, seed=5)
    # query tiles live at global 128 and 640; key tiles at 0, 128, 512, 768
    # (shards always list their tiles in increasing global position)
    qtp = torch.tensor([128, 640], dtype=torch.int32, device="cuda")
    ktp = torch.tensor([0, 128, 512, 768], dtype=torch.int32, device="cuda")
    q_pos = torch.cat([torch.arange(128) + 128, torch.arange(128) + 640]).cuda()
    k_pos = torch.cat([torch.arange(128) + t for t in (0, 128, 512, 768)]).cuda()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    o, lse = flash_attn_fwd(q, k, v, causal=True, q_tile_pos=qtp, kv_tile_pos=ktp, status=status)
    check_status(status)
    _check(o, lse, q, k, v, True, q_pos=q_pos, k_pos=k_pos)


@pytest.mark.parametrize("causal", [False, True])
def test_flash_fwd_merge_two_shards(causal):
    """Two passes over halves of the keys merged in-kernel equal one full pass."""
    from multi_gpu_flashattention_b200.ops.flash import (check_status, flash_attn_fwd_step,
                                                         tile_positions)
    B, S, H = 1, 512, 2
    q, k, v = _inputs(B, S, S, H, H, seed=7)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    o_state = torch.empty(B, S, H, 128, device="cuda", dtype=torch.float32)
    lse = torch.empty(B, H, S, device="cuda", dtype=torch.float32)
    out = torch.empty_like(q)
    qtp = tile_positions(S, "cuda")
    halves = [(slice(256, 512), 256), (slice(0, 256), 0)]  # later half first
    for i, (sl, start) in enumerate(halves):
        ktp = tile_positions(256, "cuda", start=start)
        flash_attn_fwd_step(q, k[:, sl].contiguous(), v[:, sl].contiguous(), o_state, lse,
                            causal=causal, q_tile_pos=qtp, kv_tile_pos=ktp, merge=i > 0,
                            final_out=i == len(halves) - 1, out=out, status=st)
    check_status(st)
    _check(out, lse, q, k, v, causal)
