"""sm_100a attention backward (dK/dV and dQ kernels) against fp32 autograd."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(B, Sq, Sk, Hq, Hkv, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    mk = lambda S, H: (torch.randn(B, S, H, 128, device="cuda", generator=g) * 0.5).bfloat16()
    return mk(Sq, Hq), mk(Sk, Hkv), mk(Sk, Hkv), mk(Sq, Hq)


def _ref_grads(q, k, v, do, causal, q_pos=None, k_pos=None):
    from multi_gpu_flashattention_b200.ops.reference import attention_ref
    qf, kf, vf = (t.float().requires_grad_() for t in (q, k, v))
    o, _ = attention_ref(qf, kf, vf, causal=causal, q_pos=q_pos, k_pos=k_pos)
    return torch.autograd.grad(o, (qf, kf, vf), do.float())


def _close(got, ref, name):
    err = (got.float() - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= 2e-2 * scale + 1e-3, f"{name}: max err {err} vs max |ref| {scale}"
    rel = (got.float() - ref).norm() / ref.norm()
    assert rel.item() < 1e-2, f"{name}: relative l2 error {rel.item()}"


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("B,S,Hq,Hkv", [(1, 256, 2, 2), (2, 384, 4, 2), (1, 512, 4, 1)])
def test_flash_bwd_matches_autograd(B, S, Hq, Hkv, causal):
    from multi_gpu_flashattention_b200.ops.flash import (check_status, flash_attn_bwd,
                                                         flash_attn_fwd)
    q, k, v, do = _inputs(B, S, S, Hq, Hkv)
    out, lse = flash_attn_fwd(q, k, v, causal=causal)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    dq, dk, dv = flash_attn_bwd(do, q, k, v, out, lse, causal=causal, status=st)
    check_status(st)
    rq, rk, rv = _ref_grads(q, k, v, do, causal)
    _close(dq, rq, "dq")
    _close(dk, rk, "dk")
    _close(dv, rv, "dv")


def test_flash_bwd_ragged_noncausal():
    from multi_gpu_flashattention_b200.ops.flash import flash_attn_bwd, flash_attn_fwd
    q, k, v, do = _inputs(1, 200, 333, 2, 2, seed=4)
    out, lse = flash_attn_fwd(q, k, v)
    dq, dk, dv = flash_attn_bwd(do, q, k, v, out, lse)
    rq, rk, rv = _ref_grads(q, k, v, do, False)
    _close(dq, rq, "dq")
    _close(dk, rk, "dk")
    _close(dv, rv, "dv")


def test_flash_attn_autograd_function():
    from multi_gpu_flashattention_b200.ops.flash import flash_attn
    q, k, v, do = _inputs(1, 256, 256, 2, 2, seed=9)
    qs, ks, vs = (t.clone().requires_grad_() for t in (q, k, v))
    out = flash_attn(qs, ks, vs, causal=True)
    out.backward(do)
    rq, rk, rv = _ref_grads(q, k, v, do, True)
    _close(qs.grad, rq, "dq")
    _close(ks.grad, rk, "dk")
    _close(vs.grad, rv, "dv")


def test_flash_bwd_accumulate_split_keys():
    """Two key halves with accumulate=True give the full gradients (ring building block)."""
    from multi_gpu_flashattention_b200.ops.flash import (flash_attn_bwd, flash_attn_fwd,
                                                         tile_positions)
    q, k, v, do = _inputs(1, 512, 512, 2, 2, seed=11)
    out, lse = flash_attn_fwd(q, k, v, causal=True)
    dq = torch.empty(q.shape, dtype=torch.float32, device="cuda")
    dk = torch.zeros(k.shape, dtype=torch.float32, device="cuda")
    dv = torch.zeros(v.shape, dtype=torch.float32, device="cuda")
    qtp = tile_positions(512, "cuda")
    for i, (lo, hi) in enumerate([(256, 512), (0, 256)]):
        flash_attn_bwd(do, q, k[:, lo:hi].contiguous(), v[:, lo:hi].contiguous(), out, lse,
                       causal=True, q_tile_pos=qtp, kv_tile_pos=tile_positions(256, "cuda", lo),
                       dq=dq, dk=dk[:, lo:hi], dv=dv[:, lo:hi], accumulate=i > 0)
    # dq accumulates over both halves; the second half's dk/dv add to zeros
    rq, rk, rv = _ref_grads(q, k, v, do, True)
    _close(dq, rq, "dq")
    _close(dk, rk, "dk")
    _close(dv, rv, "dv")
