"""Persistent sm_100a attention forward (attn_fwd_persistent.cu) against the fp32
PyTorch oracle: self-attention shapes, GQA, ragged lengths, non-contiguous tile
positions, every exponential variant, small grids (many items per CTA, so the
dynamic scheduler and the per-item TMEM hand-over run many times), several KV
segments accumulated in one launch, and repeated launches on one counter pair."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _C():
    from multi_gpu_flashattention_b200._ext import C
    return C()


def _inputs(B, Sq, Sk, Hq, Hkv, D=128, dtype=torch.bfloat16, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    mk = lambda S, H: (torch.randn(B, S, H, D, device="cuda", generator=g) * 0.5).to(dtype)
    return mk(Sq, Hq), mk(Sk, Hkv), mk(Sk, Hkv)


def _check(o, lse, q, k, v, causal, q_pos=None, k_pos=None):
    from multi_gpu_flashattention_b200.ops.reference import attention_ref
    ref_o, ref_lse = attention_ref(q, k, v, causal=causal, q_pos=q_pos, k_pos=k_pos)
    err = (o.float() - ref_o).abs()
    assert err.max().item() < 2e-2, f"max err {err.max().item()}"
    assert err.mean().item() < 2e-3, f"mean err {err.mean().item()}"
    finite = torch.isfinite(ref_lse)
    assert torch.equal(finite, torch.isfinite(lse))
    torch.testing.assert_close(lse[finite], ref_lse[finite], rtol=0, atol=2e-3)


def _run(q, k, v, causal, qtp=None, ktp=None, tune=-1, grid=0, seg_lens=(), calls=1):
    from multi_gpu_flashattention_b200.ops.flash import check_status, tile_positions
    if causal and qtp is None:
        qtp = tile_positions(q.shape[1], "cuda")
    if causal and ktp is None:
        ktp = tile_positions(k.shape[1], "cuda")
    sched = torch.zeros(2, dtype=torch.int32, device="cuda")
    outs = []
    for _ in range(calls):
        st = torch.zeros(1, dtype=torch.int32, device="cuda")
        o = torch.full_like(q, float("nan"))
        lse = torch.empty(q.shape[0], q.shape[2], q.shape[1], device="cuda")
        _C().flash_fwd_persistent(q, k, v, o, lse, q.shape[-1] ** -0.5, causal, qtp, ktp, st,
                                  2_000_000_000, sched, tune, grid, list(seg_lens))
        check_status(st)
        outs.append((o, lse))
    torch.cuda.synchronize()
    assert sched.tolist() == [0, 0], "the last CTA re-arms the work counters"
    return outs


# softmax variants: polynomial pairs of 8 (0, 2, 4) x scalar / packed x whole /
# split P hand-over x chained / tree row max x exact / speculative max x P-store
# wait in place / hidden
TUNES = [-1, 0x000, 0x002, 0x004, 0x100, 0x200, 0x302, 0x304, 0xb00, 0xb02, 0x1b00, 0x1b02,
         0x2b00, 0x3b00, 0x3b02]


@pytest.mark.parametrize("tune", TUNES)
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("B,S,Hq,Hkv", [(1, 256, 2, 2), (2, 640, 4, 1), (1, 1024, 3, 3)])
def test_self_attention(B, S, Hq, Hkv, causal, tune):
    q, k, v = _inputs(B, S, S, Hq, Hkv)
    (o, lse), = _run(q, k, v, causal, tune=tune)
    _check(o, lse, q, k, v, causal)


@pytest.mark.parametrize("grid", [1, 3, 7])
def test_small_grid_many_items_per_cta(grid):
    q, k, v = _inputs(2, 1408, 1408, 4, 2, seed=2)  # 11 query tiles: an odd last pair
    outs = _run(q, k, v, True, grid=grid, calls=2)
    for o, lse in outs:
        _check(o, lse, q, k, v, True)
    torch.testing.assert_close(outs[0][0], outs[1][0], rtol=0, atol=0)


@pytest.mark.parametrize("grid", [1, 2])
def test_items_without_visible_keys_between_others(grid):
    """Causal query pairs that see no key at all (no MMA, but an O hand-over
    phase) alternate with pairs that do, in one or two CTAs, so every CTA runs
    both kinds back to back: the output of the visible pairs must be exact and
    the others zero with an LSE of -inf."""
    q, k, v = _inputs(1, 1024, 256, 2, 2, seed=11)
    starts = [0, 128, 640, 768, 128, 256, 1024, 1152]  # pairs: none, both, none, both
    qtp = torch.tensor(starts, dtype=torch.int32, device="cuda")
    ktp = torch.tensor([512, 640], dtype=torch.int32, device="cuda")
    q_pos = torch.cat([torch.arange(128) + s0 for s0 in starts]).cuda()
    k_pos = torch.cat([torch.arange(128) + s0 for s0 in (512, 640)]).cuda()
    outs = _run(q, k, v, True, qtp=qtp, ktp=ktp, grid=grid, calls=3)
    for o, lse in outs:
        _check(o, lse, q, k, v, True, q_pos=q_pos, k_pos=k_pos)


def test_ragged_lengths_noncausal():
    q, k, v = _inputs(1, 200, 333, 2, 2, seed=3)
    (o, lse), = _run(q, k, v, False)
    _check(o, lse, q, k, v, False)


def test_ragged_causal():
    q, k, v = _inputs(1, 333, 333, 2, 1, seed=4)
    (o, lse), = _run(q, k, v, True)
    _check(o, lse, q, k, v, True)


def test_tile_positions_mask():
    """Causal mask from non-contiguous tile positions (zigzag-like shard)."""
    q, k, v = _inputs(1, 256, 512, 2, 2, seed=5)
    qtp = torch.tensor([128, 640], dtype=torch.int32, device="cuda")
    ktp = torch.tensor([0, 128, 512, 768], dtype=torch.int32, device="cuda")
    q_pos = torch.cat([torch.arange(128) + 128, torch.arange(128) + 640]).cuda()
    k_pos = torch.cat([torch.arange(128) + t for t in (0, 128, 512, 768)]).cuda()
    (o, lse), = _run(q, k, v, True, qtp=qtp, ktp=ktp)
    _check(o, lse, q, k, v, True, q_pos=q_pos, k_pos=k_pos)


@pytest.mark.parametrize("D,dtype", [(64, torch.bfloat16), (128, torch.float16),
                                     (64, torch.float16)])
def test_head_dims_and_dtypes(D, dtype):
    q, k, v = _inputs(1, 512, 512, 4, 2, D=D, dtype=dtype, seed=6)
    for causal in (False, True):
        (o, lse), = _run(q, k, v, causal)
        _check(o, lse, q, k, v, causal)


@pytest.mark.parametrize("causal", [False, True])
def test_segments_accumulate_in_one_launch(causal):
    """Three segments over the same buffer at different positions (the ring's
    compute pattern on one GPU): the result is attention over their union,
    with the softmax state carried across segments on chip."""
    from multi_gpu_flashattention_b200.ops.flash import tile_positions
    L = 384
    q, k, v = _inputs(1, 2 * L, L, 2, 2, seed=8)
    # queries at [0, 2L) of a 3L sequence whose keys are k at [2L,3L), [0,L), [L,2L)
    starts, lens = [2 * L, 0, L], [L, L, 256]
    ktp = torch.stack([tile_positions(L, "cuda", start=s0) for s0 in starts]).contiguous()
    qtp = tile_positions(2 * L, "cuda")
    (o, lse), = _run(q, k, v, causal, qtp=qtp, ktp=ktp, seg_lens=lens)
    k_all = torch.cat([k[:, :n] for n in lens], dim=1)
    v_all = torch.cat([v[:, :n] for n in lens], dim=1)
    k_pos = torch.cat([torch.arange(n) + s0 for s0, n in zip(starts, lens)]).cuda()
    _check(o, lse, q, k_all, v_all, causal, q_pos=torch.arange(2 * L).cuda(), k_pos=k_pos)


def test_public_flash_attn_fwd_uses_it_on_its_own_stream(monkeypatch):
    """flash_attn_fwd with the persistent kernel selected, on two streams: each
    stream gets its own counter pair."""
    from multi_gpu_flashattention_b200.ops import flash
    from multi_gpu_flashattention_b200.ops.flash import check_errors, flash_attn_fwd, sched_counters
    monkeypatch.setattr(flash, "FWD_KERNEL", "persistent")
    q, k, v = _inputs(1, 1024, 1024, 8, 8, seed=9)
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    s1.wait_stream(torch.cuda.current_stream())
    s2.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s1):
        o1, l1 = flash_attn_fwd(q, k, v, causal=True)
        c1 = sched_counters("cuda")
    with torch.cuda.stream(s2):
        o2, l2 = flash_attn_fwd(q, k, v, causal=True)
        c2 = sched_counters("cuda")
    torch.cuda.synchronize()
    check_errors()
    assert c1.data_ptr() != c2.data_ptr()
    _check(o1, l1, q, k, v, True)
    torch.testing.assert_close(o1, o2, rtol=0, atol=0)
