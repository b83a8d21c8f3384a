"""The prefill sweep's group planner (slotstream_b200.sweep.plan_sweep) against the plans the reference's own
planner produced (engine/sweep.py:34-58, fixture sweep_plan.npz made by make_golden.py), plus its invariants."""
import numpy as np
import pytest

from conftest import GOLDEN
from slotstream_b200.sweep import EXPERTS, plan_sweep


def test_plans_match_reference_planner():
    g = np.load(GOLDEN / "sweep_plan.npz")
    for c in range(int(g["n_cases"])):
        p = plan_sweep(g[f"ids_{c}"], g[f"res_{c}"], int(g[f"gs_{c}"]))
        np.testing.assert_array_equal(p.order, g[f"order_{c}"])
        got = np.array([[x.row_lo, x.row_hi, int(x.resident), x.experts.size] for x in p.groups],
                       dtype=np.int64).reshape(-1, 4)
        np.testing.assert_array_equal(got, g[f"groups_{c}"])
        ex = np.concatenate([x.experts for x in p.groups]) if p.groups else np.zeros(0, np.int32)
        np.testing.assert_array_equal(ex, g[f"experts_{c}"])


@pytest.mark.parametrize("gs", [1, 5, 32])
def test_plan_invariants(gs):
    rng = np.random.default_rng(gs)
    ids = (rng.zipf(1.2, 5000) % EXPERTS).astype(np.int32)
    res = rng.random(EXPERTS) < 0.5
    p = plan_sweep(ids, res, gs)
    assert np.array_equal(np.sort(p.order), np.arange(ids.size))
    pos = 0
    seen_staged = False
    for grp in p.groups:
        assert 1 <= grp.experts.size <= gs and np.all(np.diff(grp.experts) > 0)
        assert grp.row_lo == pos and grp.row_hi > grp.row_lo
        rows = p.order[grp.row_lo:grp.row_hi]
        assert set(ids[rows].tolist()) == set(grp.experts.tolist())
        assert np.all(res[grp.experts] == grp.resident)       # never mixes resident and staged experts
        assert np.all(np.diff(rows[ids[rows] == grp.experts[0]]) > 0)   # rows of an expert keep their order
        seen_staged |= not grp.resident
        assert not (seen_staged and grp.resident)              # resident groups first
        pos = grp.row_hi
    assert pos == ids.size


def test_plan_rejects_bad_inputs():
    res = np.zeros(EXPERTS, dtype=bool)
    with pytest.raises(ValueError):
        plan_sweep(np.zeros(3, np.int64), res)
    with pytest.raises(ValueError):
        plan_sweep(np.array([512], np.int32), res)
    with pytest.raises(ValueError):
        plan_sweep(np.array([-1], np.int32), res)
    with pytest.raises(ValueError):
        plan_sweep(np.zeros(3, np.int32), np.zeros(10, bool))
    with pytest.raises(ValueError):
        plan_sweep(np.zeros(3, np.int32), res, 0)
    assert plan_sweep(np.zeros(0, np.int32), res).groups == []


def test_count_planner_gives_the_row_planner_groups():
    """plan_groups (per-expert counts, what the device path reads back) == plan_sweep's groups."""
    from slotstream_b200.sweep import plan_groups
    rng = np.random.default_rng(3)
    for trial in range(100):
        n = int(rng.integers(0, 5000))
        ids = ((rng.zipf(1.2, n) % EXPERTS) if trial % 2 else rng.integers(0, EXPERTS, n)).astype(np.int32)
        res = rng.random(EXPERTS) < rng.random()
        gs = int(rng.integers(1, 40))
        a = plan_sweep(ids, res, gs).groups
        b = plan_groups(np.bincount(ids, minlength=EXPERTS), res, gs).groups
        assert len(a) == len(b)
        for x, y in zip(a, b):
            assert np.array_equal(x.experts, y.experts) and (x.resident, x.row_lo, x.row_hi) == (
                y.resident, y.row_lo, y.row_hi)
