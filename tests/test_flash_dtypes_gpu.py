"""head_dim 64 / 128 and bf16 / fp16 variants of the sm_100a forward and backward
kernels against the fp32 PyTorch oracle."""
import pytest
import torch

pytestmark = pytest.mark.gpu

DTYPES = {"bf16": torch.bfloat16, "fp16": torch.float16}


def _inputs(B, Sq, Sk, Hq, Hkv, D, dtype, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    mk = lambda S, H: (torch.randn(B, S, H, D, device="cuda", generator=g) * 0.5).to(dtype)
    return mk(Sq, Hq), mk(Sk, Hkv), mk(Sk, Hkv), mk(Sq, Hq)


def _close(got, ref, name, tol=2e-2):
    err = (got.float() - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= tol * scale + 1e-3, f"{name}: max err {err} vs max |ref| {scale}"
    rel = ((got.float() - ref).norm() / ref.norm()).item()
    assert rel < tol / 2, f"{name}: relative l2 error {rel}"


@pytest.mark.parametrize("dt", ["bf16", "fp16"])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("B,Sq,Sk,Hq,Hkv", [(1, 256, 256, 2, 2), (2, 384, 384, 4, 1),
                                             (1, 200, 333, 2, 2)])
def test_forward_backward_variants(B, Sq, Sk, Hq, Hkv, causal, D, dt):
    if causal and Sq != Sk:
        pytest.skip("causal needs matching lengths here")
    from multi_gpu_flashattention_b200.ops.flash import (check_status, flash_attn_bwd,
                                                         flash_attn_fwd)
    from multi_gpu_flashattention_b200.ops.reference import attention_ref
    dtype = DTYPES[dt]
    q, k, v, do = _inputs(B, Sq, Sk, Hq, Hkv, D, dtype)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    out, lse = flash_attn_fwd(q, k, v, causal=causal, status=st)
    check_status(st)
    assert out.dtype == dtype and out.shape == q.shape
    qf, kf, vf = (t.float().requires_grad_() for t in (q, k, v))
    ro, rlse = attention_ref(qf, kf, vf, causal=causal)
    err = (out.float() - ro).abs()
    assert err.max().item() < 2e-2 and err.mean().item() < 2e-3, err.max().item()
    torch.testing.assert_close(lse, rlse, rtol=0, atol=2e-3)

    dq, dk, dv = flash_attn_bwd(do, q, k, v, out, lse, causal=causal, status=st)
    check_status(st)
    rq, rk, rv = torch.autograd.grad(ro, (qf, kf, vf), do.float())
    _close(dq, rq, "dq")
    _close(dk, rk, "dk")
    _close(dv, rv, "dv")


@pytest.mark.parametrize("dt", ["bf16", "fp16"])
def test_autograd_d64(dt):
    from multi_gpu_flashattention_b200.ops.flash import flash_attn
    from multi_gpu_flashattention_b200.ops.reference import attention_ref
    q, k, v, do = _inputs(1, 512, 512, 4, 2, 64, DTYPES[dt], seed=3)
    qs, ks, vs = (t.clone().requires_grad_() for t in (q, k, v))
    flash_attn(qs, ks, vs, causal=True).backward(do)
    qf, kf, vf = (t.float().requires_grad_() for t in (q, k, v))
    ro, _ = attention_ref(qf, kf, vf, causal=True)
    rq, rk, rv = torch.autograd.grad(ro, (qf, kf, vf), do.float())
    _close(qs.grad, rq, "dq")
    _close(ks.grad, rk, "dk")
    _close(vs.grad, rv, "dv")


def test_mixed_dtypes_rejected():
    from multi_gpu_flashattention_b200.ops.flash import flash_attn_fwd
    q, k, v, _ = _inputs(1, 128, 128, 1, 1, 64, torch.bfloat16)
    with pytest.raises(RuntimeError):
        flash_attn_fwd(q, k.half(), v, causal=False)
    with pytest.raises(RuntimeError):
        flash_attn_fwd(q[..., :32].contiguous(), k[..., :32].contiguous(),
                       v[..., :32].contiguous())
