"""Race checks of the ring transports' flag protocols (executable model in
multi_gpu_flashattention_b200/utils/protocol_model.py), under seeded random
interleavings of every rank's activities."""
import pytest

from multi_gpu_flashattention_b200.utils.protocol_model import ProtocolViolation, check


@pytest.mark.parametrize("kind", ["fused", "push", "ce"])
@pytest.mark.parametrize("world", [2, 3, 5, 8])
@pytest.mark.parametrize("small_grid", [False, True])
def test_engine_protocols_are_race_free(kind, world, small_grid):
    check(world, kind, calls=3, seeds=12, small_grid=small_grid)


@pytest.mark.parametrize("world", [2, 3, 4, 5, 8])
def test_backward_engine_protocol_is_race_free(world):
    check(world, "backward", calls=3, seeds=15)


@pytest.mark.parametrize("world", [2, 3, 4, 5])
def test_exchange_protocol_is_race_free(world):
    check(world, "exchange", calls=3, seeds=20)


def test_engine_without_chain_guard_races_on_small_grids():
    """Dependent launches chained deeper than one step let step t+3 read the
    slot it shares with step t before step t resets its arrival count."""
    with pytest.raises(ProtocolViolation):
        check(5, "fused", calls=2, seeds=200, small_grid=True, chain_guard=False)


def test_exchange_without_slot0_release_races():
    """Without the step-0 release, a step-1 push can overwrite a rank's own
    shard while its step-0 push still reads it (P >= 3)."""
    with pytest.raises(ProtocolViolation, match="store began while"):
        check(3, "exchange", calls=2, seeds=200, release_slot0=False)


def test_reading_the_received_slot_needs_its_arrivals():
    with pytest.raises(ProtocolViolation):
        check(2, "exchange", calls=2, seeds=200, wait_received=False)


def test_two_ranks_are_safe_without_the_guards():
    """The races above need a third rank (slot 0) or a deep chain (P >= 5):
    two-rank runs could not have shown them."""
    check(2, "exchange", calls=3, seeds=50, release_slot0=False)
    check(4, "fused", calls=3, seeds=50, small_grid=True, chain_guard=False)


@pytest.mark.parametrize("world", [5, 8])
def test_cumulative_arrival_counts_make_deep_chains_safe(world):
    """The full fix of the chain hazard, checked before it is built: arrival
    counters that are never reset, with cumulative targets, stay race-free with
    dependent launch on for every grid size."""
    check(world, "fused", calls=3, seeds=30, small_grid=True, chain_guard=False,
          cumulative=True)


@pytest.mark.parametrize("mutation", ["credit", "release"])
@pytest.mark.parametrize("world", [2, 4])
def test_checker_catches_broken_variants(mutation, world):
    """Sensitivity of the model: a credit target one too low, or a slot handed
    back before its reads end, is caught."""
    with pytest.raises(ProtocolViolation, match="store began while"):
        check(world, "fused", calls=3, seeds=200, mutation=mutation)


@pytest.mark.parametrize("world,rank", [(2, 0), (3, 2), (5, 1), (8, 7)])
def test_native_engine_flag_arithmetic_matches_the_model(world, rank):
    """RingEngine.plan() replays the native engine's host counters (the code its
    run() takes every flag value from); the rows equal the model's."""
    from multi_gpu_flashattention_b200.utils.protocol_model import engine_plan
    try:
        from multi_gpu_flashattention_b200._ext import C
        eng = C().RingEngine
    except Exception as e:  # pragma: no cover - extension not built
        pytest.skip(f"extension not built: {e}")
    assert [list(r) for r in eng.plan(world, rank, 4)] == engine_plan(world, rank, 4)


@pytest.mark.parametrize("world,rank", [(2, 1), (4, 0), (8, 3)])
def test_native_backward_engine_flag_arithmetic_matches_the_model(world, rank):
    from multi_gpu_flashattention_b200.utils.protocol_model import backward_plan
    try:
        from multi_gpu_flashattention_b200._ext import C
        eng = C().RingBwdEngine
    except Exception as e:  # pragma: no cover - extension not built
        pytest.skip(f"extension not built: {e}")
    assert [list(r) for r in eng.plan(world, rank, 3)] == backward_plan(world, rank, 3)


@pytest.mark.parametrize("world", [2, 3, 5, 8])
def test_one_launch_ring_is_race_free(world):
    from multi_gpu_flashattention_b200.utils.protocol_model import check_one_launch
    check_one_launch(world, chunks=2, workers=2, calls=3, seeds=40)


@pytest.mark.parametrize("mutation", ["no_credit", "no_final_wait"])
def test_one_launch_checker_catches_broken_variants(mutation):
    from multi_gpu_flashattention_b200.utils.protocol_model import (ProtocolViolation,
                                                                    check_one_launch)
    with pytest.raises(ProtocolViolation):
        check_one_launch(3, chunks=2, workers=2, calls=3, seeds=200, mutation=mutation)


@pytest.mark.parametrize("world,rank", [(2, 1), (5, 3), (8, 0)])
def test_native_one_launch_engine_flags_match_the_model(world, rank):
    from multi_gpu_flashattention_b200._ext import C
    from multi_gpu_flashattention_b200.utils.protocol_model import one_launch_plan
    assert [list(r) for r in C().RingEngineP.plan(world, rank, 4)] == \
        one_launch_plan(world, rank, 4)
