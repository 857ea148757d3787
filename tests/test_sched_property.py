"""Property checks of the workload model and schedulers on random inputs
(hypothesis): the closed-form active count equals brute force, heap LPT equals
scan LPT, one move / swap repair never raises the makespan, and the contiguous
DP partition is optimal against exhaustive search on small row sets."""
import itertools

from hypothesis import given, settings, strategies as st

from multi_gpu_flashattention_b200._ext import sched as _load_sched

sched = _load_sched()


@settings(max_examples=300, deadline=None)
@given(st.sampled_from(["causal", "full"]), st.integers(0, 300), st.integers(0, 120),
       st.integers(0, 300), st.integers(0, 120))
def test_count_active_closed_form(mask, qb, qn, kb, kn):
    assert sched.count_active(mask, qb, qb + qn, kb, kb + kn) == \
        sched.count_active_bruteforce(mask, qb, qb + qn, kb, kb + kn)


@settings(max_examples=100, deadline=None)
@given(st.lists(st.floats(0.0, 100.0, allow_nan=False), min_size=0, max_size=80),
       st.integers(1, 12))
def test_lpt_heap_equals_scan(costs, g):
    a, b = sched.assign_lpt(costs, g, "scan"), sched.assign_lpt(costs, g, "heap")
    assert a.task_to_gpu == b.task_to_gpu and a.makespan() == b.makespan()


@settings(max_examples=100, deadline=None)
@given(st.lists(st.floats(0.0, 100.0, allow_nan=False), min_size=1, max_size=40),
       st.integers(1, 8), st.booleans())
def test_repairs_never_raise_the_makespan(costs, g, quirk):
    a = sched.assign_lpt(costs, g, "scan")
    moved, m = sched.rebalance_move_once(costs, a)
    assert m.makespan() <= a.makespan() + 1e-9
    swapped, s = sched.rebalance_swap_once(costs, a, reference_partner_quirk=quirk)
    assert s.makespan() <= a.makespan() + 1e-9
    for x in (m, s):  # every task still on one gpu, loads consistent
        assert sorted(set(x.task_to_gpu)) <= list(range(g))
        loads = [0.0] * g
        for t, gpu in enumerate(x.task_to_gpu):
            loads[gpu] += costs[t]
        assert abs(max(loads) - x.makespan()) <= 1e-6 * max(1.0, x.makespan())


@settings(max_examples=60, deadline=None)
@given(st.integers(1, 9), st.sampled_from([64, 100, 128]), st.sampled_from(["causal", "full"]),
       st.integers(1, 4))
def test_contiguous_dp_is_optimal(nrows, block, mask, g):
    shape = sched.WorkloadShape(nrows * block, nrows * block, block, block)
    tasks = sched.build_block_tasks(shape, mask, sched.CostModel(0.0, 1.0))
    rows = sched.build_row_tasks(shape, tasks)
    dp = sched.partition_rows_contiguous(rows, g)
    if g > len(rows):
        assert not dp.ok
        return
    costs = [r.total_cost for r in rows]
    best = min(max(sum(costs[a:b]) for a, b in zip((0,) + cuts, cuts + (len(costs),)))
               for cuts in itertools.combinations(range(1, len(costs)), g - 1))
    assert dp.ok and abs(dp.makespan() - best) <= 1e-9 * max(1.0, best)
