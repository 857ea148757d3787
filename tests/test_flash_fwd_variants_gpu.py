"""Every pipeline of the per-step sm_100a forward kernel (flash_fwd_sm100.cu:
whole 128-key tiles with packed or scalar softmax arithmetic, half tiles) against
the fp32 PyTorch oracle: causal and full masks, GQA, ragged lengths, tile
positions of a zigzag-like shard, head_dim 64, fp16, the in-kernel merge with
a running state, and scores whose row max keeps growing (O rescaled in TMEM at
many steps)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

VARIANTS = [0, 1, 2]


def _C():
    from multi_gpu_flashattention_b200._ext import C
    return C()


def _inputs(B, Sq, Sk, Hq, Hkv, D=128, dtype=torch.bfloat16, seed=0, scale=0.5):
    g = torch.Generator(device="cuda").manual_seed(seed)
    mk = lambda S, H: (torch.randn(B, S, H, D, device="cuda", generator=g) * scale).to(dtype)
    return mk(Sq, Hq), mk(Sk, Hkv), mk(Sk, Hkv)


def _check(o, lse, q, k, v, causal, q_pos=None, k_pos=None, tol=2e-2):
    from multi_gpu_flashattention_b200.ops.reference import attention_ref
    ref_o, ref_lse = attention_ref(q, k, v, causal=causal, q_pos=q_pos, k_pos=k_pos)
    err = (o.float() - ref_o).abs()
    assert err.max().item() < tol, f"max err {err.max().item()}"
    assert err.mean().item() < tol / 10, f"mean err {err.mean().item()}"
    finite = torch.isfinite(ref_lse)
    assert torch.equal(finite, torch.isfinite(lse))
    torch.testing.assert_close(lse[finite], ref_lse[finite], rtol=0, atol=2e-3)


def _fwd(q, k, v, causal, variant, qtp=None, ktp=None, o_state=None, lse=None, merge=False,
         final_out=True, out=None):
    from multi_gpu_flashattention_b200.ops.flash import check_status, tile_positions
    if causal and qtp is None:
        qtp = tile_positions(q.shape[1], "cuda")
    if causal and ktp is None:
        ktp = tile_positions(k.shape[1], "cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    o = out if out is not None else (torch.full_like(q, float("nan")) if final_out else None)
    if lse is None:
        lse = torch.empty(q.shape[0], q.shape[2], q.shape[1], device="cuda")
    _C().flash_fwd(q, k, v, o, o_state, lse, q.shape[-1] ** -0.5, causal, qtp, ktp, merge,
                   final_out, st, 2_000_000_000, variant)
    check_status(st)
    return o, lse


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("B,S,Hq,Hkv", [(1, 256, 2, 2), (2, 640, 4, 1), (1, 1024, 3, 3)])
def test_self_attention(B, S, Hq, Hkv, causal, variant):
    q, k, v = _inputs(B, S, S, Hq, Hkv)
    o, lse = _fwd(q, k, v, causal, variant)
    _check(o, lse, q, k, v, causal)


@pytest.mark.parametrize("variant", VARIANTS)
def test_ragged(variant):
    q, k, v = _inputs(1, 200, 333, 2, 2, seed=3)
    o, lse = _fwd(q, k, v, False, variant)
    _check(o, lse, q, k, v, False)
    q, k, v = _inputs(1, 333, 333, 2, 1, seed=4)
    o, lse = _fwd(q, k, v, True, variant)
    _check(o, lse, q, k, v, True)


@pytest.mark.parametrize("variant", VARIANTS)
def test_tile_positions_mask(variant):
    q, k, v = _inputs(1, 256, 512, 2, 2, seed=5)
    qtp = torch.tensor([128, 640], dtype=torch.int32, device="cuda")
    ktp = torch.tensor([0, 128, 512, 768], dtype=torch.int32, device="cuda")
    q_pos = torch.cat([torch.arange(128) + 128, torch.arange(128) + 640]).cuda()
    k_pos = torch.cat([torch.arange(128) + t for t in (0, 128, 512, 768)]).cuda()
    o, lse = _fwd(q, k, v, True, variant, qtp=qtp, ktp=ktp)
    _check(o, lse, q, k, v, True, q_pos=q_pos, k_pos=k_pos)


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("D,dtype", [(64, torch.bfloat16), (128, torch.float16),
                                     (64, torch.float16)])
def test_head_dims_and_dtypes(D, dtype, variant):
    q, k, v = _inputs(1, 512, 512, 4, 2, D=D, dtype=dtype, seed=6)
    for causal in (False, True):
        o, lse = _fwd(q, k, v, causal, variant)
        _check(o, lse, q, k, v, causal)


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("causal", [False, True])
def test_merge_two_shards(causal, variant):
    from multi_gpu_flashattention_b200.ops.flash import tile_positions
    B, S, H = 1, 512, 2
    q, k, v = _inputs(B, S, S, H, H, seed=7)
    o_state = torch.empty(B, S, H, 128, device="cuda", dtype=torch.float32)
    lse = torch.empty(B, H, S, device="cuda", dtype=torch.float32)
    out = torch.empty_like(q)
    qtp = tile_positions(S, "cuda")
    halves = [(slice(256, 512), 256), (slice(0, 256), 0)]
    for i, (sl, start) in enumerate(halves):
        ktp = tile_positions(256, "cuda", start=start)
        last = i == len(halves) - 1
        _fwd(q, k[:, sl].contiguous(), v[:, sl].contiguous(), causal, variant, qtp=qtp, ktp=ktp,
             o_state=o_state, lse=lse, merge=i > 0, final_out=last, out=out if last else None)
    _check(out, lse, q, k, v, causal)


@pytest.mark.parametrize("variant", VARIANTS)
def test_growing_row_max_rescales(variant):
    """Keys scaled up along the sequence: every few key tiles a row's max grows
    by more than 2^8 and O is rescaled in TMEM between PV steps."""
    q, k, v = _inputs(1, 512, 2048, 2, 2, seed=8, scale=1.0)
    ramp = torch.linspace(0.2, 6.0, 2048, device="cuda").view(1, -1, 1, 1)
    k = (k.float() * ramp).bfloat16()
    o, lse = _fwd(q, k, v, False, variant)
    _check(o, lse, q, k, v, False, tol=3e-2)


def test_variants_agree_closely():
    """The pipelines differ only in the order of the additions and the exponential
    method: outputs within bf16 rounding of each other."""
    q, k, v = _inputs(2, 1024, 1024, 4, 2, seed=9)
    outs = [_fwd(q, k, v, True, var)[0].float() for var in VARIANTS]
    for o in outs[1:]:
        assert (o - outs[0]).abs().max().item() < 1.6e-2
