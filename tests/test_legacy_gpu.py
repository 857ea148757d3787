"""fp32 legacy-numerics kernels against the fp32 PyTorch oracle."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_legacy_partial_merge_normalize():
    from multi_gpu_flashattention_b200._ext import C
    from multi_gpu_flashattention_b200.ops.reference import attention_ref
    torch.manual_seed(0)
    S, H = 300, 2
    q = torch.randn(S, H, 64, device="cuda")
    k = torch.randn(2 * S, H, 64, device="cuda")
    v = torch.randn(2 * S, H, 64, device="cuda")
    scale = 0.125
    acc = torch.empty(S, H, 64, device="cuda")
    m = torch.empty(H, S, device="cuda")
    l = torch.empty(H, S, device="cuda")
    acc2, m2, l2 = torch.empty_like(acc), torch.empty_like(m), torch.empty_like(l)
    C().legacy_partial(q, k[:S].contiguous(), v[:S].contiguous(), scale, None, None, False,
                       acc, m, l, False)
    C().legacy_partial(q, k[S:].contiguous(), v[S:].contiguous(), scale, None, None, False,
                       acc2, m2, l2, False)
    C().legacy_merge(m, l, acc, m2, l2, acc2)
    out = torch.empty_like(acc)
    lse = torch.empty_like(m)
    C().legacy_normalize(acc, l, out, lse, m)
    ref_o, ref_lse = attention_ref(q[None], k[None], v[None], softmax_scale=scale)
    torch.testing.assert_close(out, ref_o[0], rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(lse, ref_lse[0], rtol=1e-5, atol=1e-5)


def test_legacy_partial_in_place_merge_causal():
    from multi_gpu_flashattention_b200._ext import C
    from multi_gpu_flashattention_b200.ops.reference import attention_ref
    torch.manual_seed(1)
    S, H = 256, 1
    q = torch.randn(S, H, 64, device="cuda")
    k = torch.randn(S, H, 64, device="cuda")
    v = torch.randn(S, H, 64, device="cuda")
    pos = torch.arange(S, device="cuda")
    acc = torch.empty(S, H, 64, device="cuda")
    m = torch.empty(H, S, device="cuda")
    l = torch.empty(H, S, device="cuda")
    # later keys first, then earlier keys merged in place
    C().legacy_partial(q, k[128:].contiguous(), v[128:].contiguous(), 0.125, pos, pos[128:].contiguous(),
                       True, acc, m, l, False)
    C().legacy_partial(q, k[:128].contiguous(), v[:128].contiguous(), 0.125, pos, pos[:128].contiguous(),
                       True, acc, m, l, True)
    out = torch.empty_like(acc)
    C().legacy_normalize(acc, l, out)
    ref_o, _ = attention_ref(q[None], k[None], v[None], causal=True, softmax_scale=0.125)
    torch.testing.assert_close(out, ref_o[0], rtol=1e-4, atol=1e-5)
