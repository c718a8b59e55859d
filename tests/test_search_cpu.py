"""Resident BF16 search: the oracle against the reference's own known answers
(ops/bf16_parity.py:109-165, ops/bf16_bench.py:14-45) and the host-side rules
of ``ennx_b200.search`` (validation, failure tolerance, acquisition names).
No GPU is used."""
import json
import math
import os

import numpy as np
import pytest

import oracle.search as S
from ennx_b200 import search as P

LEAVES = [(17, 0, 257, 1.0e-6), (19, 257, 516, 1.0e-3), (23, 773, 257, 0.25)]


def _golden_base(golden_dir):
    data = json.load(open(os.path.join(golden_dir, "bf16_parity.json")))
    case = next(c for c in data["cases"] if len(c["base"]) == 1030)
    return np.array(case["base"], np.uint16)


def test_oracle_reproduces_reference_scenario(golden_dir):
    """check_search (ops/bf16_parity.py:109-165): weights 1, 0.5, 2; capacity
    8, two arms; three rounds of rewards with the reference's asserted
    acceptances, incumbent, history length and final trust-region length."""
    base = _golden_base(golden_dir)
    blocks = [leaf + (w,) for leaf, w in zip(LEAVES, (1.0, 0.5, 2.0))]
    o = S.SearchOracle(base, blocks, -0.75, 8, max_pending=2, base_variance=0.04)
    p = o.ask_round(2, 4, 1, 3, beta=1.3, draw_seed=23)
    assert len(p) == 2 and o.batch.shape == (2, 1030)
    assert np.isfinite(S.np.frombuffer((o.batch.astype(np.uint32) << 16).astype(np.uint32).tobytes(),
                                       np.float32)).all()
    o.tell_round(p, [1.0, 0.5], [0.01, 0.09])
    assert o.sync() == [True, False]
    assert o.h_best == 1.0 and math.isclose(o.h_best_variance, 0.01, rel_tol=1e-6) and o.h_history == 3
    p = o.ask_round(2, 4, 1, 5, beta=1.3, draw_seed=29)
    o.tell_device(p, [1.5, 0.25], [0.02, 0.03])
    assert o.sync() == [True, False]
    assert o.h_best == 1.5 and math.isclose(o.h_best_variance, 0.02, rel_tol=1e-6) and o.h_history == 5
    p = o.ask_round(2, 4, 1, 7, beta=1.3, draw_seed=31)
    o.tell_device(p, [2.0, 0.75])
    assert o.sync() == [True, False]
    assert o.h_best == 2.0 and math.isclose(o.h_length, 1.6, rel_tol=1e-12) and o.h_history == 7


def test_oracle_reproduces_reference_bench_state():
    """ops/bf16_bench.py:14-45 at a reduced dimension: 18 Thompson rounds of one
    arm with rewards 1..18 end with [True], best 18 and a full history of 8."""
    n = 4096
    o = S.SearchOracle(np.zeros(n, np.uint16), [(71, 0, n, 0.01, 1.0 / n)], 0.0, 8)
    for r in range(18):
        p = o.ask_round(1, 8, 8, r, acquisition_kind=1, draw_seed=r)
        o.tell_round(p, [float(r + 1)])
    assert o.sync() == [True]
    assert o.h_best == 18.0 and o.h_history == 8


def test_oracle_incumbent_row_is_the_accepted_trial():
    rng = np.random.default_rng(0)
    n = 300
    base = (rng.standard_normal(n).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    o = S.SearchOracle(base, [(5, 0, 100, 0.1, 1.0), (6, 100, 200, 0.01, 2.0)], 0.0, 3, max_pending=2)
    p = o.ask_round(2, 3, 1, 11)
    rows = o.rows.copy()
    o.tell_round(p, [-1.0, 1.0])
    assert o.sync() == [False, True]
    assert np.array_equal(o.rows[0], rows[p[1][1]])           # incumbent <- accepted trial
    assert np.array_equal(o.rows[2], rows[p[0][1]])           # history slot 2 <- first trial
    assert np.array_equal(o.rows[3], rows[p[1][1]])           # history slot 3 <- second trial
    assert o.hist_slots == [1, 2, 3]


def test_oracle_restart_resets_history_and_copies_incumbent():
    n = 64
    o = S.SearchOracle(np.full(n, 0x3F80, np.uint16), [(9, 0, n, 0.05, 1.0)], 0.0, 4, length_init=0.02,
                       length_min=0.015)
    # tolerance = ceil(max(4 / arms, dimensions / arms)): with one dimension,
    # the fourth failure halves the length below length_min -> restart
    o.dimensions = 1
    for r in range(4):
        p = o.ask_round(1, 2, 1, r)
        o.tell_round(p, [-5.0])
        assert o.sync() == [False]
        assert o.h_restarts == (1 if r == 3 else 0)
    assert o.h_history == 1 and o.h_length == 0.02
    assert np.array_equal(o.rows[1], o.rows[0])


def test_seed_and_draw_are_deterministic():
    assert S.round_seed(0, 0) == S.trial_hash(0, 0, 0) | (S.trial_hash(0, 0, 0x9E3779B9) << 32)
    d = np.array([S.draw_normal(23, i) for i in range(20000)])
    assert abs(d.mean()) < 0.03 and abs(d.std() - 1.0) < 0.03
    assert S.draw_normal(23, 5) == S.draw_normal(23, 5) != S.draw_normal(24, 5)


def test_acquisition_neighbour_order_and_kinds():
    dist = np.array([3.0, 1.0, 1.0, 2.0], np.float32)
    outcomes = [0.0, 1.0, 2.0, 3.0]
    variances = [0.0] * 4
    # two nearest: observations 1 and 2 (tie -> lower index first)
    ucb = S.acquisition(dist, outcomes, variances, 2, 0, 0.7, 0.05, 1.0, 1.0, 0.0)
    w = 1.0 / (1e-9 + 0.7 * 1.0 + 0.05)
    mean, se = (w * 1.0 + w * 2.0) / (2 * w), math.sqrt(1.0 / (2 * w))
    assert math.isclose(ucb, mean + se, rel_tol=1e-6)
    assert math.isclose(S.acquisition(dist, outcomes, variances, 2, 2, 0.7, 0.05, 1.0, 9.0, 0.0), mean + se,
                        rel_tol=1e-6)
    assert math.isclose(S.acquisition(dist, outcomes, variances, 2, 1, 0.7, 0.05, 1.0, 9.0, -0.5),
                        mean - 0.5 * se, rel_tol=1e-6)


def test_host_rules_of_the_search_mirror():
    assert P._failure_tolerance(1_000_000, 1) == 1_000_000
    assert P._failure_tolerance(2, 8) == 1 and P._failure_tolerance(3, 2) == 2
    assert P._acquisition(" Thompson ") == 1
    with pytest.raises(ValueError, match="unknown acquisition 'ei'"):
        P._acquisition("ei")

    class B:
        def __init__(self, offset, length):
            self.offset, self.length = offset, length

    check = P.SearchState._check_search
    with pytest.raises(ValueError, match="BF16 base value and variance are invalid"):
        check(4, float("nan"), 0.0, [B(0, 4)], 8, 1)
    with pytest.raises(ValueError, match="BF16 base value and variance are invalid"):
        check(4, 0.0, -1.0, [B(0, 4)], 8, 1)
    with pytest.raises(ValueError, match=r"BF16 history capacity must be in 1..=128"):
        check(4, 0.0, 0.0, [B(0, 4)], 129, 1)
    with pytest.raises(ValueError, match=r"BF16 pending capacity must be in 1..=32"):
        check(4, 0.0, 0.0, [B(0, 4)], 8, 33)
    with pytest.raises(ValueError, match="BF16 blocks must form a contiguous layout"):
        check(4, 0.0, 0.0, [B(1, 3)], 8, 1)
    with pytest.raises(ValueError, match="BF16 blocks cover 3 weights, expected 4"):
        check(4, 0.0, 0.0, [B(0, 3)], 8, 1)


def test_oracle_full_history_reuses_the_oldest_slot():
    """tell_history (cuda/kernels/src/lib.rs:446-472): at capacity the oldest
    history slot is evicted and receives the new trial row."""
    n = 128
    o = S.SearchOracle(np.full(n, 0x3F80, np.uint16), [(4, 0, n, 0.05, 1.0)], 0.0, 3)
    slots = []
    for r in range(4):
        p = o.ask_round(1, 2, 1, r)
        trial = o.rows[p[0][1]].copy()
        o.tell_round(p, [float(r + 1)])
        assert o.sync() == [True]
        slots.append(list(o.hist_slots))
        assert np.array_equal(o.rows[o.hist_slots[-1]], trial) and np.array_equal(o.rows[0], trial)
    assert slots == [[1, 2], [1, 2, 3], [2, 3, 1], [3, 1, 2]]
    assert o.outcomes == [2.0, 3.0, 4.0]


def _host_only_search(capacity=3, pending=2):
    """A SearchState with its host bookkeeping only (no device handle): the
    rules of bf16_search.rs:470-540 that run before any device call."""
    s = object.__new__(P.SearchState)
    s._capacity, s._pending_capacity, s._slots = capacity, pending, capacity + pending + 1
    s._pending, s._exports, s._next_id, s._device_index = [], 0, 0, 0
    return s


def test_search_host_rules_without_a_device():
    s = _host_only_search()
    assert s._free_slots(2) == [4, 5]
    s._pending = [(0, 4)]
    assert s._free_slots(1) == [5]
    with pytest.raises(ValueError, match="not enough free BF16 model slots"):
        s._free_slots(2)
    with pytest.raises(ValueError, match="duplicate trial"):
        s._check_trials([(0, 4), (0, 4)])
    with pytest.raises(ValueError, match="does not match an outstanding ask"):
        s._check_trials([(1, 5)])
    s._exports = 1
    with pytest.raises(ValueError, match="release live JAX proposals"):
        s._ensure_idle()
    with pytest.raises(ValueError, match="release live JAX proposals"):
        s.ask(1, 2, 1, 0)
    s._exports = 0
    with pytest.raises(ValueError, match="unknown acquisition 'ei'"):
        s.ask(1, 2, 1, 0, acquisition="ei")
    with pytest.raises(ValueError, match="tell must finish the outstanding BF16 round"):
        s.ask(1, 2, 1, 0)
    s._pending = []
    with pytest.raises(ValueError, match="BF16 round shape exceeds pending capacity"):
        s.ask(3, 2, 1, 0)
    p = P.Proposals(s, [(0, 4)])
    assert p.arms == 1
    with pytest.raises(BufferError, match="does not export copies"):
        p.__dlpack__(copy=True)
    with pytest.raises(BufferError, match="cannot export to another device"):
        p.__dlpack__(dl_device=(1, 0))
    for bad in (0, -3):
        with pytest.raises(ValueError, match="invalid DLPack CUDA stream"):
            p.__dlpack__(stream=bad)
    with pytest.raises(ValueError, match="equal non-zero length"):
        s.tell(p, [1.0, 2.0])
    with pytest.raises(ValueError, match="values and variances must be finite"):
        s.tell(p, [float("nan")])
