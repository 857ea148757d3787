"""Argument checks of the CUDA entry points fail cleanly (a Python exception
with a readable message, no crash) when given host tensors, and the public
ring_attention runs on the host with the fp32 `torch` backend and no process
group."""
import pytest
import torch


def _qkv(dtype=torch.bfloat16, S=256, H=2, D=128):
    g = torch.Generator().manual_seed(0)
    return [(torch.randn(1, S, H, D, generator=g) * 0.5).to(dtype) for _ in range(3)]


def test_flash_fwd_rejects_host_tensors():
    from multi_gpu_flashattention_b200.ops.flash import flash_attn_fwd
    q, k, v = _qkv()
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        flash_attn_fwd(q, k, v, causal=False, status=torch.zeros(1, dtype=torch.int32))


def test_flash_bwd_rejects_host_tensors():
    from multi_gpu_flashattention_b200.ops.flash import flash_attn_bwd
    q, k, v = _qkv()
    lse = torch.zeros(1, 2, 256)
    with pytest.raises(RuntimeError, match="CUDA"):
        flash_attn_bwd(q.clone(), q, k, v, q.clone(), lse, causal=False,
                       status=torch.zeros(1, dtype=torch.int32))


@pytest.mark.parametrize("causal", [False, True])
def test_ring_attention_on_host_matches_oracle(causal):
    import multi_gpu_flashattention_b200 as mgfa
    from multi_gpu_flashattention_b200.ops.reference import attention_ref
    q, k, v = _qkv(torch.float32, S=192, H=4, D=32)
    out = mgfa.ring_attention(q, k, v, causal=causal, backend="torch")
    ref, _ = attention_ref(q, k, v, causal=causal)
    torch.testing.assert_close(out.float(), ref, rtol=1e-4, atol=1e-5)
