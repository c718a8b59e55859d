"""CPU restatement of the reference's resident BF16 TuRBO search.

TEST INFRASTRUCTURE ONLY: the checker for ``ennx_b200.search``, never the
product.  Follows, in one object:

* the host state of ``SearchState`` (rust/crates/ennx/src/bf16_search.rs:62-628):
  pending trials, free slots, ``failure_tolerance``, the queued round;
* the device engine ``Bf16SearchEngine`` (cuda/src/bf16_search.rs:129-1067)
  and its kernels: ``seed_bf16`` (cuda/kernels/src/lib.rs:1466-1480),
  ``distance_bf16``/``tile_distances`` (lib.rs:1310-1380, bf16.rs:278-330),
  ``score_bf16``/``acquisition_score`` (lib.rs:1382-1447, bf16.rs:178-275),
  ``draw_bf16``/``draw_normal`` (lib.rs:1452-1461, 316-343), ``pick_trial``
  (lib.rs:1660-1744), ``write_bf16`` (lib.rs:2053-2130) and ``tell_bf16`` with
  ``tell_validate``/``tell_history``/``tell_adapt`` (lib.rs:409-535, 2135-2258).

Distances are accumulated in double precision (the reference sums in fp32 in
its own tile order, which no other implementation reproduces); everything
after them -- neighbour selection, acquisition, pick, materialisation, the
tell bookkeeping -- follows the reference's float32 operation order.
"""
from __future__ import annotations

import ctypes
import math

import numpy as np

from . import lib

MAX_HISTORY = 128
MAX_PENDING = 32
F32 = np.float32


class EoBf16Leaf(ctypes.Structure):
    _fields_ = [("key", ctypes.c_uint64), ("offset", ctypes.c_uint64), ("length", ctypes.c_uint64),
                ("scale", ctypes.c_float), ("weight", ctypes.c_float)]


def _leaf_array(leaves):
    return (EoBf16Leaf * len(leaves))(*[EoBf16Leaf(*leaf) for leaf in leaves])


def trial_hash(lo: int, hi: int, element: int) -> int:
    return lib().eo_trial_hash(lo & 0xFFFFFFFF, hi & 0xFFFFFFFF, element & 0xFFFFFFFF)


def round_seed(root: int, index: int) -> int:
    """seed_bf16: the candidate seed of a resident round (lib.rs:1466-1480)."""
    lo, hi = root & 0xFFFFFFFF, (root >> 32) & 0xFFFFFFFF
    return trial_hash(lo, hi, index) | (trial_hash(hi, lo, index ^ 0x9E3779B9) << 32)


def candidate_row(base: np.ndarray, leaves, seed: int, coef: float) -> tuple[np.ndarray, bool]:
    base = np.ascontiguousarray(base, np.uint16)
    out = np.empty_like(base)
    bad = lib().eo_search_candidate(base.ctypes.data, base.size, _leaf_array(leaves), len(leaves), seed,
                                    float(F32(coef)), out.ctypes.data)
    return out, bool(bad)


def distances(rows: np.ndarray, base_slot: int, history_slots, leaves, seed: int, coef: float) -> tuple[np.ndarray, bool]:
    rows = np.ascontiguousarray(rows, np.uint16)
    hs = np.ascontiguousarray(history_slots, np.uint32)
    out = np.empty(len(hs), np.float64)
    bad = lib().eo_search_distances(rows.ctypes.data, rows.shape[1], base_slot, hs.ctypes.data, len(hs),
                                    _leaf_array(leaves), len(leaves), rows.shape[1], seed, float(F32(coef)),
                                    out.ctypes.data)
    return out, bool(bad)


def acquisition(dist: np.ndarray, outcomes, variances, neighbors: int, acq: int, eps, alea, y_scale, beta,
                draw: float) -> np.float32:
    """acquisition_score (bf16.rs:224-275): insertion k-NN (strict '<', lower
    observation first on ties), inverse-variance weights, f32 rounding per op."""
    nd = [F32(np.inf)] * neighbors
    ni = [0] * neighbors
    for o, d in enumerate(dist):
        d = F32(d)
        at = neighbors
        for k in range(neighbors):
            if d < nd[k] or (d == nd[k] and o < ni[k]):
                at = k
                break
        if at >= neighbors:
            continue
        nd[at + 1:] = nd[at:-1]
        ni[at + 1:] = ni[at:-1]
        nd[at], ni[at] = d, o
    wsum, wval = F32(0), F32(0)
    for k in range(neighbors):
        idx = ni[k]
        var = F32(F32(F32(F32(1e-9) + F32(eps) * nd[k]) + F32(alea)) + F32(variances[idx]))
        w = F32(1) / max(var, F32(1e-12))
        wsum = F32(wsum + w)
        wval = F32(wval + F32(w * F32(outcomes[idx])))
    mean = F32(wval / max(wsum, F32(1e-12)))
    se = F32(np.sqrt(F32(F32(1) / max(wsum, F32(1e-12)))) * F32(y_scale))
    if acq == 1:
        return F32(mean + F32(se * F32(draw)))
    if acq == 2:
        return F32(mean + se)
    return F32(mean + F32(F32(beta) * se))


def draw_normal(seed: int, index: int, metric: int = 0) -> float:
    return lib().eo_draw_normal(seed & (2**64 - 1), index, metric)


def failure_tolerance(dimensions: int, arms: int) -> int:
    """bf16_search.rs:542-548."""
    return max(1, math.ceil(max(4.0 / arms, dimensions / arms)))


class SearchOracle:
    """One resident search, its rows as a numpy matrix [slots, len]."""

    def __init__(self, base_bits, blocks, base_value, capacity, max_pending=1, base_variance=0.0, length_init=0.8,
                 length_min=0.0078125, length_max=1.6):
        base = np.ascontiguousarray(base_bits, np.uint16)
        self.len = base.size
        self.dimensions = base.size  # SearchState::dimensions, the failure-tolerance scale
        self.leaves = [tuple(b) for b in blocks]  # (key, offset, length, scale, weight)
        self.capacity = capacity
        self.pending_capacity = max_pending
        self.slots = capacity + max_pending + 1
        self.rows = np.zeros((self.slots, self.len), np.uint16)
        self.rows[0] = base
        self.rows[1] = base  # SearchState::create, copy_row(0, 1)
        self.hist_slots = [1]
        self.outcomes = [F32(base_value)]
        self.variances = [F32(base_variance)]
        self.s = dict(length=float(length_init), length_init=float(length_init), length_min=float(length_min),
                      length_max=float(length_max), trust_best=float(F32(base_value)),
                      hist_min=float(F32(base_value)), hist_max=float(F32(base_value)), best=F32(base_value),
                      best_variance=F32(base_variance), prev_obs=1, successes=0, failures=0, restarts=0, status=0)
        self.region_status = [0] * MAX_PENDING
        self.pending: list[tuple[int, int]] = []  # (id, slot)
        self.next_id = 0
        self.queued: int | None = None
        self.summary = None
        self.accepted: list[bool] = []
        self.batch = None
        self.last_scores = None
        self.last_distances = None
        self.last_selection = None
        # host copies updated at sync
        self.h_length, self.h_best, self.h_best_variance = float(length_init), F32(base_value), F32(base_variance)
        self.h_restarts, self.h_history = 0, 1

    # -- ask ---------------------------------------------------------------
    def free_slots(self, count):
        used = {slot for _, slot in self.pending}
        slots = [s for s in range(self.capacity + 1, self.slots) if s not in used][:count]
        if len(slots) != count:
            raise ValueError("not enough free BF16 model slots")
        return slots

    def ask_round(self, arms, candidates, neighbors, seed_root, epistemic_scale=0.7, aleatoric_scale=0.05,
                  y_scale=1.0, beta=1.0, acquisition_kind=0, draw_seed=0, near_tie=None):
        """``near_tie`` (test aid): a callable (region, oracle_pick, scores) ->
        index that may substitute another candidate whose score ties the
        oracle's best within the fp32 summation-order tolerance of the
        distances; the substitute is then materialised."""
        if self.pending:
            raise ValueError("tell must finish the outstanding BF16 round")
        if arms == 0 or arms > self.pending_capacity or candidates == 0:
            raise ValueError("BF16 round shape exceeds pending capacity")
        slots = self.free_slots(arms)
        H = len(self.hist_slots)
        K = min(neighbors, H)
        coef = F32(self.s["length"])
        C = arms * candidates
        seeds = [round_seed(seed_root, c) for c in range(C)]
        scores = np.empty(C, np.float32)
        dists = np.empty((C, H), np.float64)
        for c in range(C):
            d, bad = distances(self.rows, 0, self.hist_slots, self.leaves, seeds[c], coef)
            dists[c] = d
            d32 = d.astype(np.float32)
            if bad or not np.isfinite(d32[0]):
                scores[c] = -np.inf
            else:
                draw = draw_normal(draw_seed, c) if acquisition_kind == 1 else 0.0
                scores[c] = acquisition(d32, self.outcomes, self.variances, K, acquisition_kind, epistemic_scale,
                                        aleatoric_scale, y_scale, beta, draw)
        selection = []
        for r in range(arms):
            best, bi = F32(-np.inf), 0xFFFFFFFF  # pick_trial: higher score, then lower index
            for c in range(r * candidates, (r + 1) * candidates):
                if scores[c] > best or (scores[c] == best and c < bi):
                    best, bi = scores[c], c
            if near_tie is not None:
                bi = near_tie(r, bi, scores)
                best = scores[bi]
            selection.append((bi, F32(best)))
        self.batch = np.zeros((arms, self.len), np.uint16)
        for r, (idx, _) in enumerate(selection):
            row, bad = candidate_row(self.rows[0], self.leaves, seeds[idx], coef)
            self.rows[slots[r]] = row
            self.batch[r] = row
            self.region_status[r] = int(bad or self.s["status"] != 0)
        self.last_scores, self.last_distances, self.last_selection = scores, dists, selection
        proposals = []
        for slot in slots:
            proposals.append((self.next_id, slot))
            self.pending.append((self.next_id, slot))
            self.next_id += 1
        return proposals

    # -- tell --------------------------------------------------------------
    def tell_round(self, proposals, values, variances=None):
        n = len(proposals)
        variances = [0.0] * n if variances is None else list(variances)
        if n == 0 or len(values) != n or len(variances) != n:
            raise ValueError("BF16 trials, values, and variances must have equal non-zero length")
        vals = [F32(v) for v in values]
        vars_ = [F32(v) for v in variances]
        if any(not np.isfinite(v) for v in vals) or any(not np.isfinite(v) or v < 0 for v in vars_):
            raise ValueError("BF16 values and variances must be finite")
        self._check(proposals)
        self._device_tell([slot for _, slot in proposals], vals, vars_, failure_tolerance(self.dimensions, n))
        self.pending.clear()
        self.queued = n

    def tell_device(self, proposals, values, variances=None):
        """finish_round: the rewards are validated on the device."""
        n = len(proposals)
        vals = [F32(v) for v in values]
        vars_ = [F32(0)] * n if variances is None else [F32(v) for v in variances]
        self._check(proposals)
        self._device_tell([slot for _, slot in proposals], vals, vars_, failure_tolerance(self.dimensions, n))
        self.pending.clear()
        self.queued = n

    def _check(self, proposals):
        for i, p in enumerate(proposals):
            if p in proposals[:i]:
                raise ValueError("BF16 tell batch contains a duplicate trial")
            if p not in self.pending:
                raise ValueError("BF16 trial does not match an outstanding ask")

    def _device_tell(self, slots, values, variances, tolerance):
        s = self.s
        status = 0
        accepted = [False] * len(slots)
        for i in range(len(slots)):
            if not np.isfinite(values[i]) or not np.isfinite(variances[i]) or variances[i] < 0:
                status = 1
            status |= self.region_status[i]
        self.region_status = [0] * MAX_PENDING
        if status:
            s["status"] = status
            self.summary = dict(length=s["length"], best=s["best"], best_variance=s["best_variance"],
                                history=len(self.hist_slots), restarts=s["restarts"], restarted=0, status=status)
            self.accepted = accepted
            return
        best_slot = None
        copies = []
        for i, slot in enumerate(slots):
            v, var = values[i], variances[i]
            if v > s["best"]:
                s["best"], s["best_variance"], best_slot = v, var, slot
                accepted[i] = True
            if len(self.hist_slots) == self.capacity:
                dest = self.hist_slots.pop(0)
                self.outcomes.pop(0)
                self.variances.pop(0)
            else:
                dest = len(self.hist_slots) + 1
            copies.append((slot, dest))
            self.hist_slots.append(dest)
            self.outcomes.append(v)
            self.variances.append(var)
        prev = s["trust_best"]
        if math.isfinite(prev):
            scale = max(s["hist_max"] - s["hist_min"], 1e-6) if s["prev_obs"] >= 2 else 0.0
            if float(s["best"]) > prev + 1e-3 * scale:
                s["successes"] += 1
                s["failures"] = 0
            else:
                s["failures"] += 1
                s["successes"] = 0
            if s["successes"] >= 3:
                s["length"] = min(s["length"] * 2.0, s["length_max"])
                s["successes"] = 0
            elif s["failures"] >= tolerance:
                s["length"] *= 0.5
                s["failures"] = 0
        s["trust_best"] = float(s["best"])
        for v in values:
            s["hist_min"] = min(s["hist_min"], float(v))
            s["hist_max"] = max(s["hist_max"], float(v))
        s["prev_obs"] += len(slots)
        restarted = 0
        if s["length"] < s["length_min"]:
            s.update(length=s["length_init"], successes=0, failures=0, trust_best=-math.inf, hist_min=math.inf,
                     hist_max=-math.inf)
            s["restarts"] += 1
            self.hist_slots = [1]
            self.outcomes = [s["best"]]
            self.variances = [s["best_variance"]]
            restarted = 1
        s["status"] = 0
        # row copies in the reference's order: best -> 0, trials -> history, 0 -> 1 on restart
        if best_slot is not None:
            self.rows[0] = self.rows[best_slot]
        for src, dst in copies:
            self.rows[dst] = self.rows[src]
        if restarted:
            self.rows[1] = self.rows[0]
        self.summary = dict(length=s["length"], best=s["best"], best_variance=s["best_variance"],
                            history=len(self.hist_slots), restarts=s["restarts"], restarted=restarted, status=0)
        self.accepted = accepted

    def sync(self):
        if self.queued is None:
            return []
        if self.summary["status"] != 0:
            raise ValueError("CUDA BF16 proposal or rewards are invalid")
        self.queued = None
        sm = self.summary
        self.h_history, self.h_length, self.h_best = sm["history"], sm["length"], sm["best"]
        self.h_best_variance, self.h_restarts = sm["best_variance"], sm["restarts"]
        return list(self.accepted)
