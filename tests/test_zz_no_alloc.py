"""Allocation-free backward entry point (mgfa_attn_bwd_noalloc), called through
its exported C symbol, against the regular backward entry point.

The entry point serves callers that cannot allocate device memory (a host
runtime or memory-pool framework that owns every allocation and only passes in
input and output buffers). Its scratch is a static device array in the library.
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
    return fn


def _close(got, ref, name):
    # same criterion as the backward tests against the fp32 oracle
    err = (got.float() - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= 2e-2 * scale + 1e-3, f"{name}: max err {err} vs max |ref| {scale}"
    rel = (got.float() - ref).norm() / max(ref.norm().item(), 1e-30)
    assert rel.item() < 1e-2, f"{name}: relative l2 error {rel.item()}"


@pytest.mark.parametrize("causal", [True, False])
def test_noalloc_backward_matches_regular_entry_point(causal):
    from multi_gpu_flashattention_b200.ops.flash import flash_attn_bwd, flash_attn_fwd
    fn = _lib()
    B, S, Hq, Hkv = 1, 384, 4, 2
    g = torch.Generator(device="cuda").manual_seed(21)
    mk = lambda H: (torch.randn(B, S, H, 128, device="cuda", generator=g) * 0.5).bfloat16()
    q, k, v, do = mk(Hq), mk(Hkv), mk(Hkv), mk(Hq)
    out, lse = flash_attn_fwd(q, k, v, causal=causal)
    rq, rk, rv = flash_attn_bwd(do, q, k, v, out, lse, causal=causal)
    scale = 128 ** -0.5
    stream = torch.cuda.current_stream().cuda_stream
    results = []
    for _ in range(2):  # two calls in a row share (and reuse) the static scratch
        dq = torch.full(q.shape, float("nan"), device="cuda")
        dk = torch.full(k.shape, float("nan"), device="cuda")
        dv = torch.full(v.shape, float("nan"), device="cuda")
        rc = fn(do.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                lse.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, S, S, Hq, Hkv,
                scale, int(causal), stream)
        assert rc == 0
        torch.cuda.synchronize()
        _close(dq, rq, "dq")
        _close(dk, rk, "dk")
        _close(dv, rv, "dv")
        results.append((dq, dk, dv))
    for a, b in zip(*results):
        torch.testing.assert_close(a, b, rtol=0, atol=0)


def test_noalloc_rejects_oversized_problem():
    fn = _lib()
    x = torch.empty(16, device="cuda")
    # 64 query heads x 1M tokens needs far more scratch than the static array
    rc = fn(*[x.data_ptr()] * 9, 1, 1 << 20, 1 << 20, 64, 64, 0.1, 1,
            torch.cuda.current_stream().cuda_stream)
    assert rc == 2
