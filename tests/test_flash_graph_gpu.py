"""CUDA-graph replays of the single-GPU attention (GraphedAttention) against
eager calls and the fp32 oracle."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(seed, B=1, S=512, H=2, D=128, dtype=torch.bfloat16):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return [(torch.randn(B, S, H, D, device="cuda", generator=g) * 0.5).to(dtype)
            for _ in range(4)]


@pytest.mark.parametrize("causal", [False, True])
def test_graph_replay_matches_eager(causal):
    from multi_gpu_flashattention_b200.ops.flash import check_status, flash_attn_bwd, flash_attn_fwd
    from multi_gpu_flashattention_b200.ops.graphs import GraphedAttention
    q0, k0, v0, _ = _inputs(0)
    g = GraphedAttention(q0, k0, v0, causal=causal, backward=True)
    for seed in (1, 2):  # new inputs each replay
        q, k, v, do = _inputs(seed)
        out, lse = g.forward(q, k, v)
        dq, dk, dv = g.backward(do)
        torch.cuda.synchronize()
        check_status(g.status)
        ro, rl = flash_attn_fwd(q, k, v, causal=causal)
        rq, rk, rv = flash_attn_bwd(do, q, k, v, ro, rl, causal=causal)
        torch.testing.assert_close(out, ro, rtol=0, atol=0)
        torch.testing.assert_close(lse, rl, rtol=0, atol=0)
        for a, b in ((dq, rq), (dk, rk), (dv, rv)):
            torch.testing.assert_close(a, b, rtol=0, atol=0)


def test_graph_forward_matches_oracle_d64_fp16():
    from multi_gpu_flashattention_b200.ops.graphs import GraphedAttention
    from multi_gpu_flashattention_b200.ops.reference import attention_ref
    q, k, v, _ = _inputs(3, S=384, H=4, D=64, dtype=torch.float16)
    g = GraphedAttention(q, k, v, causal=True)
    out, lse = g(q, k, v)
    ref, ref_lse = attention_ref(q, k, v, causal=True)
    assert (out.float() - ref).abs().max().item() < 2e-2
    torch.testing.assert_close(lse, ref_lse, rtol=0, atol=2e-3)
