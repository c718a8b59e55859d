"""Resident BF16 search on the GPU against the oracle and the reference's own
known answers (ops/bf16_parity.py:109-165, ops/bf16_bench.py:14-45)."""
import ctypes
import gc
import json
import math
import os

import numpy as np
import pytest

import oracle.search as S

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

from ennx_b200 import _abi, _dlpack  # noqa: E402
from ennx_b200.experimental import ParamBlock, turbo_enn  # noqa: E402

LEAVES = [(17, 0, 257, 1.0e-6), (19, 257, 516, 1.0e-3), (23, 773, 257, 0.25)]
ACQ = {"ucb": 0, "thompson": 1, "pareto": 2}


def _dev_bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits, np.uint16).view(np.int16)).cuda().view(torch.bfloat16)


def _bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


class _Borrowed:
    """DLPack view of a device row owned by a search handle."""

    def __init__(self, pointer, n):
        self.pointer, self.n = pointer, n

    def __dlpack_device__(self):
        return (_dlpack.KDL_CUDA, torch.cuda.current_device())

    def __dlpack__(self, stream=None, max_version=None, dl_device=None, copy=None):
        return _dlpack.export(self, self.pointer, (self.n,), _dlpack.KDL_BFLOAT, 16,
                              (_dlpack.KDL_CUDA, torch.cuda.current_device()), lambda: None)


def _row_bits(handle, slot, n):
    ptr = ctypes.c_void_p()
    assert _abi.lib().ennx_b200_bf16_search_row(handle, slot, ctypes.byref(ptr)) == 0
    torch.cuda.synchronize()
    return _bits(torch.from_dlpack(_Borrowed(ptr.value, n)).clone())


def _golden_base(golden_dir):
    data = json.load(open(os.path.join(golden_dir, "bf16_parity.json")))
    case = next(c for c in data["cases"] if len(c["base"]) == 1030)
    return np.array(case["base"], np.uint16)


def test_reference_scenario(golden_dir):
    """check_search of ops/bf16_parity.py:109-165 with torch in place of JAX."""
    base = _golden_base(golden_dir)
    blocks = [ParamBlock(*leaf, w) for leaf, w in zip(LEAVES, (1.0, 0.5, 2.0))]
    search = turbo_enn(_dev_bf16(base), -0.75, blocks, 8, max_pending=2, base_variance=0.04)
    search.profile(True)
    proposals = search.ask(2, 4, 1, 3, beta=1.3, draw_seed=23)
    assert proposals.arms == 2
    assert search.last_profile is not None and search.last_profile[3] > 0.0
    batch = torch.from_dlpack(proposals)
    assert batch.shape == (2, 1030) and batch.dtype == torch.bfloat16
    assert bool(torch.isfinite(batch.float()).all())
    with pytest.raises(ValueError, match="live JAX proposals"):
        search.tell(proposals, [1.0, 0.5], [0.01, 0.09])
    del batch
    gc.collect()
    search.tell(proposals, [1.0, 0.5], [0.01, 0.09])
    assert search.sync() == [True, False]
    assert search.best == 1.0
    assert math.isclose(search.best_variance, 0.01, rel_tol=1e-6)
    assert search.history_len == 3 and search.len == 1030
    proposals = search.ask(2, 4, 1, 5, beta=1.3, draw_seed=29)
    search.tell(proposals, torch.tensor([1.5, 0.25], device="cuda"), torch.tensor([0.02, 0.03], device="cuda"))
    assert search.sync() == [True, False]
    assert search.best == 1.5
    assert math.isclose(search.best_variance, 0.02, rel_tol=1e-6)
    assert search.history_len == 5
    proposals = search.ask(2, 4, 1, 7, beta=1.3, draw_seed=31)
    search.tell(proposals, torch.tensor([2.0, 0.75], device="cuda"))
    assert search.sync() == [True, False]
    assert search.best == 2.0
    assert math.isclose(search.length, 1.6, rel_tol=1e-12)
    assert search.history_len == 7


def _near_tie(gpu_scores, cpr):
    """Accept the GPU's pick where it ties the oracle's within the tolerance
    of fp32 distance sums taken in another order."""
    def pick(region, oracle_pick, scores):
        first = region * cpr
        g = first + int(np.argmax(np.asarray(gpu_scores[first:first + cpr])))  # first max = lower index
        if g != oracle_pick:
            a, b = float(scores[g]), float(scores[oracle_pick])
            assert math.isclose(a, b, rel_tol=2e-5, abs_tol=1e-6), (region, g, oracle_pick, a, b)
        return g
    return pick


@pytest.mark.parametrize("n", [1030, 20011])
def test_rounds_match_oracle(n):
    rng = np.random.default_rng(n)
    base = (rng.standard_normal(n).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    cut = [0, n // 3, n // 3 + 7, n]
    leaves = [(1000 + i, cut[i], cut[i + 1] - cut[i], (0.02, 0.5, 0.003)[i], (1.0, 0.25, 3.0)[i]) for i in range(3)]
    capacity, pending = 5, 3
    search = turbo_enn(_dev_bf16(base), 0.1, [ParamBlock(*l) for l in leaves], capacity, max_pending=pending,
                       base_variance=0.01)
    o = S.SearchOracle(base, leaves, 0.1, capacity, max_pending=pending, base_variance=0.01)
    plan = [(3, 4, 1, "ucb"), (2, 5, 2, "thompson"), (3, 3, 3, "pareto"), (1, 6, 4, "ucb"), (3, 4, 5, "thompson"),
            (2, 3, 2, "ucb"), (3, 2, 4, "pareto")]
    for r, (arms, cpr, k, acq) in enumerate(plan):
        kw = dict(epistemic_scale=0.6, aleatoric_scale=0.04, y_scale=1.5, beta=1.2)
        proposals = search.ask(arms, cpr, k, 100 + r, acquisition=acq, draw_seed=7 * r, **kw)
        g_scores, g_dist = search._last_scores(arms * cpr, history=1)
        o_props = o.ask_round(arms, cpr, k, 100 + r, acquisition_kind=ACQ[acq], draw_seed=7 * r,
                              near_tie=_near_tie(g_scores, cpr), **kw)
        H = len(o.last_distances[0])
        g_d = np.array(g_dist).reshape(arms * cpr, S.MAX_HISTORY)[:, :H]
        np.testing.assert_allclose(g_d, o.last_distances, rtol=2e-5, atol=1e-9)
        np.testing.assert_allclose(g_scores, o.last_scores, rtol=2e-5, atol=1e-6)
        batch = torch.from_dlpack(proposals)
        assert np.array_equal(_bits(batch), o.batch), r
        del batch
        gc.collect()
        values = rng.normal(size=arms).astype(np.float32) + 0.1 * r
        variances = rng.uniform(0, 0.05, size=arms).astype(np.float32)
        if r % 2:
            search.tell(proposals, torch.from_numpy(values).cuda(), torch.from_numpy(variances).cuda())
        else:
            search.tell(proposals, values.tolist(), variances.tolist())
        o.tell_round(o_props, values.tolist(), variances.tolist())
        assert search.sync() == o.sync(), r
        assert (search.best, search.history_len, search.restarts) == (o.h_best, o.h_history, o.h_restarts)
        assert search.length == o.h_length and search.best_variance == o.h_best_variance
        for slot in range(capacity + pending + 1):
            assert np.array_equal(_bits(search._row(slot)), o.rows[slot]), (r, slot)


def _handle(base_bits, leaves, slots):
    h = ctypes.c_void_p()
    t = _dev_bf16(base_bits)
    arr = (_abi.Bf16Leaf * len(leaves))(*[_abi.Bf16Leaf(*l) for l in leaves])
    st = _abi.lib().ennx_b200_bf16_search_create(ctypes.c_void_p(t.data_ptr()), t.numel(), arr, len(leaves), slots,
                                                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
                                                  ctypes.byref(h))
    assert st == 0, _abi.lib().ennx_b200_last_error()
    return h


def test_seeded_ask_through_the_c_abi():
    """Bf16SearchEngine::ask with host seeds, explicit history and step."""
    rng = np.random.default_rng(4)
    n = 5000
    base = (rng.standard_normal(n).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    leaves = [(77, 0, 3000, 0.05, 1.0), (78, 3000, 2000, 0.01, 0.5)]
    L = _abi.lib()
    h = _handle(base, leaves, 6)
    try:
        assert L.ennx_b200_bf16_search_copy_row(h, 0, 1) == 0
        assert L.ennx_b200_bf16_search_init(h, 0.5, 0.02, 3, 0.8, 0.01, 1.6) == 0
        seeds = [int(s) for s in rng.integers(0, 2**63, size=6)]
        cfg = _abi.AskConfig(1, 0, 0.7, 0.05, 1.0, 1.0)
        sel = (_abi.Selection * 2)()
        slots = (ctypes.c_uint32 * 2)(4, 5)
        st = L.ennx_b200_bf16_search_ask(h, 0, 1, slots, 2, (ctypes.c_uint64 * 6)(*seeds), 3, ctypes.c_float(0.5),
                                         0, ctypes.byref(cfg), sel)
        assert st == 0, L.ennx_b200_last_error()
        rows = np.stack([base, base])
        scores = []
        for c, seed in enumerate(seeds):
            d, bad = S.distances(rows, 0, [1], leaves, seed, 0.5)
            assert not bad
            scores.append(S.acquisition(d.astype(np.float32), [0.5], [0.02], 1, 0, 0.7, 0.05, 1.0, 1.0, 0.0))
        for r in range(2):
            best = max(range(3 * r, 3 * r + 3), key=lambda c: (scores[c], -c))
            assert sel[r].index == best or math.isclose(scores[sel[r].index], scores[best], rel_tol=2e-5)
            row, _ = S.candidate_row(base, leaves, seeds[sel[r].index], 0.5)
            assert np.array_equal(_row_bits(h, (4, 5)[r], n), row)
        # shape and slot errors use the reference's text
        st = L.ennx_b200_bf16_search_ask(h, 0, 1, (ctypes.c_uint32 * 2)(4, 4), 2, (ctypes.c_uint64 * 6)(*seeds), 3,
                                         ctypes.c_float(0.5), 0, ctypes.byref(cfg), sel)
        assert st == _abi.INVALID_ARGUMENT and b"distinct from live rows" in L.ennx_b200_last_error()
        cfg.neighbors = 2
        st = L.ennx_b200_bf16_search_ask(h, 0, 1, slots, 2, (ctypes.c_uint64 * 6)(*seeds), 3, ctypes.c_float(0.5), 0,
                                         ctypes.byref(cfg), sel)
        assert st == _abi.INVALID_ARGUMENT and b"neighbor count exceeds" in L.ennx_b200_last_error()
    finally:
        L.ennx_b200_bf16_search_destroy(h)


def test_overflowing_candidates_reset_the_trial_rows():
    base = np.full(64, 0x7F7F, np.uint16)  # largest finite BF16
    leaves = [(31, 0, 64, 3.4028234663852886e38, 1.0)]
    L = _abi.lib()
    h = _handle(base, leaves, 4)
    try:
        assert L.ennx_b200_bf16_search_copy_row(h, 0, 1) == 0
        assert L.ennx_b200_bf16_search_init(h, 0.0, 0.0, 2, 0.8, 0.01, 1.6) == 0
        cfg = _abi.AskConfig(1, 0, 0.7, 0.05, 1.0, 1.0)
        sel = (_abi.Selection * 1)()
        st = L.ennx_b200_bf16_search_ask(h, 0, 1, (ctypes.c_uint32 * 1)(3), 1, (ctypes.c_uint64 * 2)(5, 6), 2,
                                         ctypes.c_float(1.0), 0, ctypes.byref(cfg), sel)
        assert st == _abi.OVERFLOW and b"overflowed" in L.ennx_b200_last_error()
        assert np.array_equal(_row_bits(h, 3, 64), base)
    finally:
        L.ennx_b200_bf16_search_destroy(h)


def test_invalid_device_rewards_fail_at_sync():
    n = 256
    search = turbo_enn(torch.zeros(n, dtype=torch.bfloat16, device="cuda"), 0.0, [ParamBlock(3, 0, n, 0.1)], 4)
    p = search.ask(1, 2, 1, 9)
    search.tell(p, torch.tensor([float("nan")], device="cuda"))
    with pytest.raises(ValueError, match="proposal or rewards are invalid"):
        search.sync()
    with pytest.raises(ValueError, match="device rewards must match the proposal count"):
        q = turbo_enn(torch.zeros(n, dtype=torch.bfloat16, device="cuda"), 0.0, [ParamBlock(3, 0, n, 0.1)], 4)
        q.tell(q.ask(1, 2, 1, 9), torch.zeros(2, device="cuda"))
    with pytest.raises(ValueError, match="BF16 trial does not match an outstanding ask"):
        r = turbo_enn(torch.zeros(n, dtype=torch.bfloat16, device="cuda"), 0.0, [ParamBlock(3, 0, n, 0.1)], 4)
        pr = r.ask(1, 2, 1, 9)
        r.tell(pr, [1.0])
        r.tell(pr, [1.0])


def test_reference_bench_known_answer_at_one_million():
    """ops/bf16_bench.py:14-45: 1e6 weights, capacity 8, 18 Thompson rounds of
    one arm and 8 candidates; rewards 1..18 -> [True], best 18, history 8."""
    n = 1_000_000
    search = turbo_enn(torch.zeros(n, dtype=torch.bfloat16, device="cuda"), 0.0,
                       [ParamBlock(71, 0, n, 0.01, 1.0 / n)], 8)
    search.profile(True)
    for r in range(18):
        p = search.ask(1, 8, 8, r, acquisition="thompson", draw_seed=r)
        search.tell(p, [float(r + 1)])
    assert search.sync() == [True]
    assert search.best == 18.0 and search.history_len == 8
    assert search.last_profile[3] < 250.0
