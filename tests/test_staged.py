"""The host-staged experts' placement (tsb_staged_rebalance: the reference's rebalance, src/qwen35/q36_engine.cu:
3215-3265) against the oracle's restatement on random and tied scores, and its argument checks.  Host code only."""
import numpy as np
import pytest

import tinystrata_b200 as T
from oracle import oracle as O


def state(rng, E, S, tie_levels=None):
    score = (rng.integers(0, tie_levels, E) if tie_levels else rng.exponential(3.0, E)).astype(np.float64)
    exp_in_slot = rng.permutation(E)[:S].astype(np.int32)
    slot_of = np.full(E, -1, np.int32)
    slot_of[exp_in_slot] = np.arange(S, dtype=np.int32)
    return score, slot_of, exp_in_slot


@pytest.mark.parametrize("E,S,swaps,ties", [(64, 24, 64, None), (256, 40, 8, None), (256, 40, 1000, 3),
                                            (32, 31, 5, 2), (128, 1, 4, None), (64, 0, 8, None), (64, 64, 8, None)])
def test_rebalance_matches_the_restatement(E, S, swaps, ties):
    rng = np.random.default_rng(E * 1000 + S + swaps)
    for _ in range(5):
        score, slot_of, exp_in_slot = state(rng, E, S, ties)
        s2, so2, ex2 = score.copy(), slot_of.copy(), exp_in_slot.copy()
        me, ms = T.staged_rebalance(score, slot_of, exp_in_slot, swaps)
        want = O.staged_rebalance(s2, so2, ex2, swaps)
        assert list(zip(me.tolist(), ms.tolist())) == want
        assert np.array_equal(slot_of, so2) and np.array_equal(exp_in_slot, ex2)
        assert np.array_equal(score, s2)
        assert len(me) <= swaps
        if 0 < S < E:   # after the moves the slots hold distinct experts and slot_of agrees
            assert len(set(exp_in_slot.tolist())) == S
            assert all(slot_of[x] == s for s, x in enumerate(exp_in_slot))


def test_rebalance_takes_the_most_used():
    E, S = 16, 4
    score = np.zeros(E)
    score[[9, 10, 11, 12]] = [5, 4, 3, 2]
    slot_of = np.full(E, -1, np.int32)
    exp_in_slot = np.arange(S, dtype=np.int32)
    slot_of[:S] = np.arange(S)
    score[1] = 3.5   # a resident that stays (it outranks experts 11 and 12)
    me, ms = T.staged_rebalance(score, slot_of, exp_in_slot, 8)
    assert sorted(exp_in_slot.tolist()) == [1, 9, 10, 11]
    assert me.tolist() == [9, 10, 11] and slot_of[1] == 1
    assert np.allclose(score[[9, 1]], [2.5, 1.75])   # aged


def test_rebalance_rejects_an_inconsistent_table():
    score = np.ones(8)
    slot_of = np.full(8, -1, np.int32)
    exp_in_slot = np.array([2, 3], np.int32)
    slot_of[2] = 0   # expert 3's entry is missing
    with pytest.raises(T.TsbError):
        T.staged_rebalance(score, slot_of, exp_in_slot, 4)
