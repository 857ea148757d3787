"""Property checks of the shard layouts on random sizes (hypothesis): every
layout partitions the sequence, shard/unshard round-trips, tile position
tables are non-decreasing (the kernels rely on visible key tiles forming a
prefix), and the per-(rank, owner) causal work adds up to the whole causal
triangle (full mask: the whole square). Zigzag chunks that are not whole
128-token tiles are refused with a clear error when tile tables are asked for."""
import pytest
import torch
from hypothesis import given, settings, strategies as st

from multi_gpu_flashattention_b200.parallel.layouts import RingLayout


@st.composite
def layouts(draw):
    kind = draw(st.sampled_from(["contiguous", "zigzag", "striped", "scheduler"]))
    world = draw(st.integers(1, 8))
    mask = draw(st.sampled_from(["causal", "full"]))
    if kind == "zigzag":
        seq = 2 * world * draw(st.integers(1, 40)) * 8
    elif kind == "striped":
        seq = world * draw(st.integers(1, 300))
    elif kind == "scheduler":
        seq = 128 * draw(st.integers(world, 24))
    else:
        seq = draw(st.integers(world, 5000))
    policy = draw(st.sampled_from(["dp", "lpt"]))
    return RingLayout(kind, seq, world, mask=mask, policy=policy)


@settings(max_examples=80, deadline=None)
@given(layouts())
def test_partition_and_round_trip(lay):
    allpos = torch.cat([lay.positions(r) for r in range(lay.world)])
    assert torch.equal(allpos.sort().values, torch.arange(lay.seq))
    assert sum(lay.local_len(r) for r in range(lay.world)) == lay.seq
    x = torch.arange(lay.seq, dtype=torch.float32).view(1, -1, 1)
    shards = [lay.shard(x, r) for r in range(lay.world)]
    assert all(s.shape[1] == lay.max_local_len for s in shards)
    for r, s in enumerate(shards):  # a shard holds its own global positions, in order
        n = lay.local_len(r)
        assert torch.equal(s[0, :n, 0].long(), lay.positions(r))
    torch.testing.assert_close(lay.unshard(shards), x)


@settings(max_examples=60, deadline=None)
@given(layouts())
def test_tile_tables_monotone_and_work_complete(lay):
    if lay.kind == "zigzag" and lay.world > 1 and (lay.seq // (2 * lay.world)) % 128:
        # a zigzag chunk that is not whole 128-token tiles has no tile table
        with pytest.raises(ValueError, match="multiples of 128"):
            lay.q_tile_pos(0, "cpu")
        return
    for r in range(lay.world):
        qt = lay.q_tile_pos(r, "cpu").tolist()
        assert qt == sorted(qt)
        for o in range(lay.world):
            kt = lay.kv_tile_pos(r, o, "cpu").tolist()
            assert kt == sorted(kt)
    S = lay.seq
    total = sum(lay.step_work(r, o) for r in range(lay.world) for o in range(lay.world))
    assert total == (S * (S + 1) // 2 if lay.mask == "causal" else S * S)


@settings(max_examples=40, deadline=None)
@given(st.integers(1, 8), st.integers(0, 7), st.integers(0, 7))
def test_ring_owners(world, rank, step):
    lay = RingLayout("contiguous", 128 * world, world)
    rank, step = rank % world, step % world
    assert lay.compute_owner(rank, step) == (rank - step) % world
    assert lay.receive_owner(rank, step) == (rank - step - 1) % world


@pytest.mark.parametrize("kind,seq,world", [("zigzag", 100, 4), ("striped", 10, 4)])
def test_unsplittable_sizes_are_rejected(kind, seq, world):
    with pytest.raises(Exception):
        RingLayout(kind, seq, world)


@settings(max_examples=60, deadline=None)
@given(layouts())
def test_step_work_equals_brute_force(lay):
    """Each (rank, owner) pair's visible (query, key) count equals a direct
    count over the two shards' global positions."""
    if lay.seq > 2048:
        return
    for r in range(lay.world):
        qp = lay.positions(r)
        for o in range(lay.world):
            kp = lay.positions(o)
            want = int((kp[None, :] <= qp[:, None]).sum()) if lay.mask == "causal" \
                else qp.numel() * kp.numel()
            assert lay.step_work(r, o) == want
