"""RingAttentionBlock on gloo ranks equals the unsharded block (forward and grads)."""
import torch

from dist_utils import run_ranks


def _block_case(rank, world, kind):
    import torch.distributed as dist
    from multi_gpu_flashattention_b200.models import RingAttentionBlock
    from multi_gpu_flashattention_b200.parallel.layouts import RingLayout
    torch.manual_seed(0)
    blk = RingAttentionBlock(d_model=32, n_heads=4, n_kv_heads=2, head_dim=16, mlp_mult=2)
    S = 256
    x = torch.randn(1, S, 32)
    lay = RingLayout(kind, S, world, block=32, mask="causal")
    # reference: the same block on one "rank" with a contiguous single-shard layout
    ref_lay = RingLayout("contiguous", S, 1, mask="causal")
    xr = x.clone().requires_grad_()
    y_ref = blk(xr, ref_lay, 0, group=_solo_group(), backend="torch")
    y_ref.square().sum().backward()
    g_ref = {n: p.grad.clone() for n, p in blk.named_parameters()}
    blk.zero_grad()
    xl = lay.shard(x, rank).requires_grad_()
    y = blk(xl, lay, rank, backend="torch")
    n = lay.local_len(rank)
    torch.testing.assert_close(y[:, :n], lay.shard(y_ref.detach(), rank)[:, :n], rtol=1e-4, atol=1e-5)
    y[:, :n].square().sum().backward()
    for name, p in blk.named_parameters():
        dist.all_reduce(p.grad)
        torch.testing.assert_close(p.grad, g_ref[name], rtol=1e-3, atol=1e-4)


_SOLO = {}


def _solo_group():
    import torch.distributed as dist
    r = dist.get_rank()
    if r not in _SOLO:
        groups = [dist.new_group([i]) for i in range(dist.get_world_size())]
        _SOLO[r] = groups[r]
    return _SOLO[r]


def test_block_matches_unsharded_zigzag():
    run_ranks(_block_case, 2, "zigzag")


def test_block_matches_unsharded_striped():
    run_ranks(_block_case, 2, "striped")


def _lm_case(rank, world, kind):
    import torch.distributed as dist
    from multi_gpu_flashattention_b200.models import RingTransformerLM, shard_targets
    from multi_gpu_flashattention_b200.parallel.layouts import RingLayout
    torch.manual_seed(0)
    model = RingTransformerLM(vocab=50, d_model=32, n_layers=2, n_heads=4, n_kv_heads=2,
                              head_dim=16, mlp_mult=2)
    S = 192
    ids = torch.randint(0, 50, (2, S), generator=torch.Generator().manual_seed(1))
    # reference: the unsharded model (one-rank layout on a solo group)
    ref_lay = RingLayout("contiguous", S, 1, mask="causal")
    loss_ref = model.loss(ids, shard_targets(ids, ref_lay, 0), ref_lay, 0, group=_solo_group(),
                          backend="torch")
    loss_ref.backward()
    g_ref = {n: p.grad.clone() for n, p in model.named_parameters()}
    model.zero_grad()
    lay = RingLayout(kind, S, world, block=32, mask="causal")
    loss = model.loss(lay.shard(ids, rank), shard_targets(ids, lay, rank), lay, rank,
                      backend="torch")
    total = loss.detach().clone()
    dist.all_reduce(total)
    torch.testing.assert_close(total, loss_ref.detach(), rtol=1e-4, atol=1e-5)
    loss.backward()
    for name, p in model.named_parameters():
        dist.all_reduce(p.grad)
        torch.testing.assert_close(p.grad, g_ref[name], rtol=1e-3, atol=1e-5)


def test_lm_loss_and_grads_match_unsharded_zigzag():
    run_ranks(_lm_case, 2, "zigzag")


def test_lm_loss_and_grads_match_unsharded_contiguous_3_ranks():
    run_ranks(_lm_case, 3, "contiguous")
