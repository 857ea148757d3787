"""The in-CTA pipeline model of the persistent attention forward
(utils/cta_pipeline_model.py): the kernel's barrier protocol runs race- and
deadlock-free under seeded random interleavings of its warps, TMA loads and
tensor-core work, and each broken variant of it is caught."""
import random

import pytest

from multi_gpu_flashattention_b200.utils.cta_pipeline_model import PipelineViolation, check


def _items(rng, lo=0):
    return [rng.randrange(lo, 7) for _ in range(rng.randrange(1, 6))]


@pytest.mark.parametrize("split", [False, True])
def test_protocol_is_race_free(split):
    for seed in range(150):
        rng = random.Random(seed)
        check(_items(rng), seed, split=split, rescale_every=rng.choice([0, 1, 2, 3]))


def test_items_without_key_tiles_between_others():
    for seed in range(150):
        check([3, 0, 2, 0, 0, 4, 0], seed, rescale_every=2)


@pytest.mark.parametrize("mutation", ["no_k_empty", "s_before_pv", "early_o_empty",
                                      "p_count_3", "no_q_empty", "t0_no_o_empty"])
def test_each_broken_variant_is_caught(mutation):
    caught = 0
    for seed in range(200):
        rng = random.Random(seed)
        items = [rng.randrange(0 if mutation == "t0_no_o_empty" else 1, 7)
                 for _ in range(rng.randrange(2, 6))]
        try:
            check(items, seed, mutation=mutation, rescale_every=2)
        except PipelineViolation:
            caught += 1
    assert caught > 0, f"{mutation} was never caught"
