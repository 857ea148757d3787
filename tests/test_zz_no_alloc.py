"""Allocation-free backward entry point (mgfa_attn_bwd_noalloc), called through
its exported C symbol, against the regular backward entry point and the fp32
autograd oracle.

The entry point serves callers that cannot allocate device memory (a host
runtime or memory-pool framework that owns every allocation and only passes in
input and output buffers). Its scratch is a static device array in the library,
and its kernels' status word is read back through
mgfa_attn_bwd_noalloc_status into caller-owned host memory.
This file is named so that pytest collects it last."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    import multi_gpu_flashattention_b200._C as ext  # loads torch's libraries first
    lib = ctypes.CDLL(ext.__file__)
    fn = lib.mgfa_attn_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 9 + [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_int,
                                                                  ctypes.c_void_p]
    status = lib.mgfa_attn_bwd_noalloc_status
    status.restype = ctypes.c_int
    status.argtypes = [ctypes.POINTER(ctypes.c_uint), ctypes.c_void_p]
    return fn, status


def _close(got, ref, name):
    # same criterion as the backward tests against the fp32 oracle
    err = (got.float() - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= 2e-2 * scale + 1e-3, f"{name}: max err {err} vs max |ref| {scale}"
    rel = (got.float() - ref).norm() / max(ref.norm().item(), 1e-30)
    assert rel.item() < 1e-2, f"{name}: relative l2 error {rel.item()}"


def _oracle_grads(q, k, v, do, causal):
    from multi_gpu_flashattention_b200.ops.reference import attention_ref
    qf, kf, vf = (t.float().requires_grad_() for t in (q, k, v))
    o, _ = attention_ref(qf, kf, vf, causal=causal)
    return torch.autograd.grad(o, (qf, kf, vf), do.float())


# (batch, seqlen_q, seqlen_k, heads_q, heads_kv, causal): tile-aligned, a ragged
# length, and causal cases with seqlen_q != seqlen_k on both sides (query i sees
# keys 0..i, so the causal tile positions and the scratch layout differ between
# the query and key sides)
SHAPES = [
    (1, 384, 384, 4, 2, True),
    (1, 384, 384, 4, 2, False),
    (1, 333, 333, 2, 1, True),
    (2, 200, 333, 4, 2, True),
    (1, 333, 200, 2, 2, True),
]


@pytest.mark.parametrize("B,Sq,Sk,Hq,Hkv,causal", SHAPES)
def test_noalloc_backward_matches_regular_entry_point_and_oracle(B, Sq, Sk, Hq, Hkv, causal):
    from multi_gpu_flashattention_b200.ops.flash import flash_attn_bwd, flash_attn_fwd
    fn, status_fn = _lib()
    g = torch.Generator(device="cuda").manual_seed(21 + Sq + Sk)
    mk = lambda S, H: (torch.randn(B, S, H, 128, device="cuda", generator=g) * 0.5).bfloat16()
    q, k, v, do = mk(Sq, Hq), mk(Sk, Hkv), mk(Sk, Hkv), mk(Sq, Hq)
    out, lse = flash_attn_fwd(q, k, v, causal=causal)
    rq, rk, rv = flash_attn_bwd(do, q, k, v, out, lse, causal=causal)
    oq, ok, ov = _oracle_grads(q, k, v, do, causal)
    scale = 128 ** -0.5
    stream = torch.cuda.current_stream().cuda_stream
    results = []
    for _ in range(2):  # two calls in a row share (and reuse) the static scratch
        dq = torch.full(q.shape, float("nan"), device="cuda")
        dk = torch.full(k.shape, float("nan"), device="cuda")
        dv = torch.full(v.shape, float("nan"), device="cuda")
        rc = fn(do.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                lse.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, Sq, Sk, Hq, Hkv,
                scale, int(causal), stream)
        assert rc == 0
        word = ctypes.c_uint(0xFFFFFFFF)
        assert status_fn(ctypes.byref(word), stream) == 0
        torch.cuda.synchronize()
        assert word.value == 0, f"kernel status {word.value:#x}"
        for got, reg, ref, name in ((dq, rq, oq, "dq"), (dk, rk, ok, "dk"), (dv, rv, ov, "dv")):
            _close(got, reg, name + " vs regular entry point")
            _close(got, ref, name + " vs fp32 oracle")
        results.append((dq, dk, dv))
    for a, b in zip(*results):
        torch.testing.assert_close(a, b, rtol=0, atol=0)


def test_noalloc_rejects_oversized_problem():
    fn, _ = _lib()
    x = torch.empty(16, device="cuda")
    # 64 query heads x 1M tokens needs far more scratch than the static array
    rc = fn(*[x.data_ptr()] * 9, 1, 1 << 20, 1 << 20, 64, 64, 0.1, 1,
            torch.cuda.current_stream().cuda_stream)
    assert rc == 2
