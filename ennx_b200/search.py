"""Resident BF16 TuRBO search on the GPU: ``SearchState``, ``Proposals`` and
``turbo_enn`` by the names of ``ennx.experimental``.

Mirrors the PyO3 classes of rust/crates/ennx-py/src/py_bf16.rs:57-313 and the
host state they wrap, ``SearchState`` in rust/crates/ennx/src/bf16_search.rs:
62-628 (pending trials, free row slots, failure tolerance, the queued round),
over the handle API ``ennx_b200_bf16_search_*`` of ``libennx_b200.so``.  Every
row of the search (incumbent, history, trials) and the trust-region state stay
in device memory: ``ask`` -> evaluate the exported proposals -> ``tell`` with
device rewards runs without a host round trip until ``sync``.

Error text follows the reference.  Not thread-safe (the reference classes are
``unsendable``).
"""
from __future__ import annotations

import ctypes
import math
from typing import Sequence

from . import _abi, _dlpack
from .experimental import ParamBlock, _bf16_input

__all__ = ["Proposals", "SearchState", "turbo_enn"]

MAX_HISTORY = 128
MAX_PENDING = 32
_ACQUISITION = {"ucb": 0, "thompson": 1, "pareto": 2}


def _acquisition(name: str) -> int:
    """AcquisitionKind::parse (rust/crates/ennx/src/weights.rs:27-37)."""
    value = name.strip().lower()
    if value not in _ACQUISITION:
        raise ValueError(f"unknown acquisition {value!r}; expected 'ucb', 'thompson', or 'pareto'")
    return _ACQUISITION[value]


def _failure_tolerance(dimensions: int, arms: int) -> int:
    """failure_tolerance (bf16_search.rs:542-548)."""
    return max(1, math.ceil(max(4.0 / arms, dimensions / arms)))


def _f32(x) -> float:
    return float(ctypes.c_float(x).value)


class Proposals:
    """The trials of one resident round.  ``__dlpack__`` exports them as one
    read-only BF16 device matrix ``[arms, len]``; while an export is alive the
    search refuses ``ask`` and ``tell`` (py_bf16.rs:224-302)."""

    def __init__(self, owner: "SearchState", trials: list[tuple[int, int]]):
        self._owner = owner
        self._trials = trials  # (trial id, row slot)

    @property
    def arms(self) -> int:
        return len(self._trials)

    def __dlpack_device__(self) -> tuple[int, int]:
        return (_dlpack.KDL_CUDA, self._owner._device_index)

    def __dlpack__(self, stream: int | None = None, max_version: tuple[int, int] | None = None,
                   dl_device: tuple[int, int] | None = None, copy: bool | None = None):
        if copy is True:
            raise BufferError("Proposals does not export copies")
        if dl_device is not None and tuple(dl_device) != self.__dlpack_device__():
            raise BufferError("Proposals cannot export to another device")
        if stream is not None and (stream == 0 or stream < -1):
            raise ValueError("invalid DLPack CUDA stream")
        search = self._owner
        search._ensure_idle()
        pointer = search._device_round(self._trials, stream)
        search._exports += 1

        def release():
            search._exports -= 1

        return _dlpack.export(self, pointer, (self.arms, search._len), _dlpack.KDL_BFLOAT, 16,
                              self.__dlpack_device__(), release, max_version)


class SearchState:
    """Stateful TuRBO search over full-precision BF16 weights, resident on
    one CUDA device (py_bf16.rs:57-222; bf16_search.rs:62-628).

    ``SearchState(base, base_value, blocks, capacity, max_pending=1,
    base_variance=0.0, length_init=0.8, length_min=0.0078125, length_max=1.6)``
    copies ``base`` (a DLPack BF16 CUDA array) into ``capacity + max_pending
    + 1`` resident rows.  Work is enqueued on the torch stream that is current
    when the search is created.
    """

    def __init__(self, base, base_value: float, blocks: Sequence[ParamBlock], capacity: int, max_pending: int = 1,
                 base_variance: float = 0.0, length_init: float = 0.8, length_min: float = 0.0078125,
                 length_max: float = 1.6):
        torch, src = _bf16_input(base)
        for block in blocks:
            if not isinstance(block, ParamBlock):
                raise TypeError("SearchState blocks must be ParamBlock instances")
        n = src.numel()
        base_value, base_variance = _f32(base_value), _f32(base_variance)
        self._check_search(n, base_value, base_variance, blocks, capacity, max_pending)
        self._torch = torch
        self._device = src.device
        self._device_index = src.device.index or 0
        self._len = n
        self._capacity = capacity
        self._pending_capacity = max_pending
        self._slots = capacity + max_pending + 1
        self._handle = ctypes.c_void_p()
        leaves = (_abi.Bf16Leaf * len(blocks))(*[_abi.Bf16Leaf(b.key, b.offset, b.length, b.scale, b.weight)
                                                for b in blocks])
        with torch.cuda.device(self._device):
            self._stream = torch.cuda.current_stream()
            flat = src.reshape(-1)
            _abi.call("ennx_b200_bf16_search_create", ctypes.c_void_p(flat.data_ptr()), n, leaves, len(blocks),
                      self._slots, ctypes.c_void_p(self._stream.cuda_stream), ctypes.byref(self._handle))
            try:
                self._call("ennx_b200_bf16_search_copy_row", 0, 1)
                self._call("ennx_b200_bf16_search_init", base_value, base_variance, capacity, float(length_init),
                           float(length_min), float(length_max))
            except BaseException:
                _abi.lib().ennx_b200_bf16_search_destroy(self._handle)
                self._handle = ctypes.c_void_p()
                raise
        self._pending: list[tuple[int, int]] = []
        self._next_id = 0
        self._queued: int | None = None
        self._exports = 0
        self._history = 1
        self._length = float(length_init)
        self._best = base_value
        self._best_variance = base_variance
        self._restarts = 0

    def __del__(self):
        h = getattr(self, "_handle", None)
        if h is not None and h.value:
            _abi.lib().ennx_b200_bf16_search_destroy(h)
            self._handle = ctypes.c_void_p()

    @staticmethod
    def _check_search(n, base_value, base_variance, blocks, capacity, pending):
        """check_search (bf16_search.rs:552-590)."""
        if not math.isfinite(base_value) or not math.isfinite(base_variance) or base_variance < 0.0:
            raise ValueError("BF16 base value and variance are invalid")
        if capacity == 0 or capacity > MAX_HISTORY:
            raise ValueError(f"BF16 history capacity must be in 1..={MAX_HISTORY}")
        if pending == 0 or pending > MAX_PENDING:
            raise ValueError(f"BF16 pending capacity must be in 1..={MAX_PENDING}")
        expected = 0
        for block in blocks:
            if block.offset != expected:
                raise ValueError("BF16 blocks must form a contiguous layout")
            expected += block.length
        if expected == 0 or expected != n:
            raise ValueError(f"BF16 blocks cover {expected} weights, expected {n}")

    def _call(self, name, *args):
        with self._torch.cuda.device(self._device):
            _abi.call(name, self._handle, *args)

    def _ensure_idle(self):
        if self._exports:
            raise ValueError("release live JAX proposals before mutating the search")

    def _free_slots(self, count):
        used = {slot for _, slot in self._pending}
        slots = [s for s in range(self._capacity + 1, self._slots) if s not in used][:count]
        if len(slots) != count:
            raise ValueError("not enough free BF16 model slots")
        return slots

    def _check_trials(self, trials):
        for i, trial in enumerate(trials):
            if trial in trials[:i]:
                raise ValueError("BF16 tell batch contains a duplicate trial")
            if trial not in self._pending:
                raise ValueError("BF16 trial does not match an outstanding ask")

    def _device_round(self, trials, stream):
        self._check_trials(trials)
        batch = ctypes.c_void_p()
        self._call("ennx_b200_bf16_search_round", len(trials), ctypes.byref(batch))
        self._handoff(stream)
        return batch.value

    def _handoff(self, stream):
        """sync_stream (cuda/src/lib.rs:1014-1033): None synchronises, -1
        skips, any other value is a CUDA stream that waits on an event."""
        if stream is None:
            self._call("ennx_b200_bf16_search_handoff", None, 0)
        elif stream == -1:
            self._call("ennx_b200_bf16_search_handoff", None, 1)
        else:
            self._call("ennx_b200_bf16_search_handoff", ctypes.c_void_p(stream), 2)

    # -- ask / tell ---------------------------------------------------------
    def ask(self, arms: int, candidates: int, neighbors: int, seed: int, epistemic_scale: float = 0.7,
            aleatoric_scale: float = 0.05, y_scale: float = 1.0, beta: float = 1.0, acquisition: str = "ucb",
            draw_seed: int = 0) -> Proposals:
        """One resident round (py_bf16.rs:100-139 -> ask_round,
        bf16_search.rs:236-285): per arm, ``candidates`` seeded candidates
        around the incumbent, scored by the ENN acquisition against the
        history; the best of each arm is written to a trial row."""
        self._ensure_idle()
        kind = _acquisition(acquisition)
        if self._pending:
            raise ValueError("tell must finish the outstanding BF16 round")
        if arms == 0 or arms > self._pending_capacity or candidates == 0:
            raise ValueError("BF16 round shape exceeds pending capacity")
        slots = self._free_slots(arms)
        config = _abi.AskConfig(neighbors, kind, epistemic_scale, aleatoric_scale, y_scale, beta)
        slot_arr = (ctypes.c_uint32 * arms)(*slots)
        self._call("ennx_b200_bf16_search_ask_seeded", 0, slot_arr, arms, candidates, seed & (2**64 - 1),
                   draw_seed & (2**64 - 1), ctypes.byref(config))
        trials = []
        for slot in slots:
            trial = (self._next_id, slot)
            self._next_id = (self._next_id + 1) & (2**64 - 1)
            self._pending.append(trial)
            trials.append(trial)
        return Proposals(self, trials)

    def tell(self, proposals: Proposals, values, variances=None) -> None:
        """Queue the rewards of a round (py_bf16.rs:141-180): host sequences
        go through ``queue_round``, DLPack FP32 device arrays through
        ``finish_round`` without a host copy."""
        self._ensure_idle()
        trials = proposals._trials
        if hasattr(values, "__dlpack__"):
            d_values = self._f32_input(values)
            if d_values.numel() != proposals.arms:
                raise ValueError("device rewards must match the proposal count")
            d_vars = None if variances is None else self._f32_input(variances)
            if d_vars is not None and d_vars.numel() != proposals.arms:
                raise ValueError("device variances must match the proposal count")
            self._check_trials(trials)
            self._queue(trials, ctypes.c_void_p(d_values.data_ptr()),
                        None if d_vars is None else ctypes.c_void_p(d_vars.data_ptr()), True)
            return
        host_values = [float(v) for v in values]
        host_vars = [0.0] * len(host_values) if variances is None else [float(v) for v in variances]
        n = len(trials)
        if n == 0 or len(host_values) != n or len(host_vars) != n:
            raise ValueError("BF16 trials, values, and variances must have equal non-zero length")
        vals = [_f32(v) for v in host_values]
        vars_ = [_f32(v) for v in host_vars]
        if any(not math.isfinite(v) for v in vals) or any(not math.isfinite(v) or v < 0.0 for v in vars_):
            raise ValueError("BF16 values and variances must be finite")
        self._check_trials(trials)
        self._queue(trials, (ctypes.c_float * n)(*vals), (ctypes.c_float * n)(*vars_), False)

    def _f32_input(self, x):
        torch = self._torch
        t = x if isinstance(x, torch.Tensor) else torch.from_dlpack(x)
        if t.dtype != torch.float32:
            raise ValueError("DLPack tensor must be FP32")
        if not t.is_cuda or t.device != self._device:
            raise ValueError("DLPack tensor must live on the search's CUDA device")
        if not t.is_contiguous():
            raise BufferError("FP32 input requires a contiguous DLPack tensor")
        if t.numel() == 0:
            raise ValueError("FP32 input requires a non-empty tensor")
        return t

    def _queue(self, trials, values, variances, on_device):
        n = len(trials)
        slots = (ctypes.c_uint32 * n)(*[slot for _, slot in trials])
        self._call("ennx_b200_bf16_search_tell", slots, n, values, variances, 1 if on_device else 0,
                   self._capacity, _failure_tolerance(self._len, n))
        self._pending.clear()
        self._queued = n

    def sync(self) -> list[bool]:
        """Read the outcome of the queued tell (bf16_search.rs:441-450):
        which trials became the incumbent."""
        if self._queued is None:
            return []
        n = self._queued
        accepted = (ctypes.c_uint8 * n)()
        summary = _abi.TellSummary()
        self._call("ennx_b200_bf16_search_collect", n, accepted, ctypes.byref(summary))
        self._queued = None
        self._history = summary.history
        self._length = summary.length
        self._best = summary.best
        self._best_variance = summary.best_variance
        self._restarts = summary.restarts
        return [bool(a) for a in accepted]

    # -- state --------------------------------------------------------------
    def profile(self, enabled: bool) -> None:
        self._call("ennx_b200_bf16_search_set_profiling", 1 if enabled else 0)

    @property
    def last_profile(self) -> tuple[float, float, float, float] | None:
        """(score_ms, pick_ms, materialize_ms, total_ms) of the last ask, or
        None when profiling is off.  Scoring and picking run in one pass here,
        so pick_ms is reported as 0 and its time is inside score_ms."""
        out = (ctypes.c_float * 4)()
        available = ctypes.c_int32(0)
        self._call("ennx_b200_bf16_search_last_profile", out, ctypes.byref(available))
        return tuple(out) if available.value else None

    @property
    def length(self) -> float:
        self.sync()
        return self._length

    @property
    def best(self) -> float:
        self.sync()
        return self._best

    @property
    def best_variance(self) -> float:
        self.sync()
        return self._best_variance

    @property
    def restarts(self) -> int:
        self.sync()
        return self._restarts

    @property
    def history_len(self) -> int:
        self.sync()
        return self._history

    @property
    def len(self) -> int:
        return self._len

    # -- test and tracing aids ---------------------------------------------
    def _last_scores(self, count: int, history: int = 0):
        """Scores and summed distances (stride 128) of the last ask."""
        scores = (ctypes.c_float * max(count, 1))()
        nd = count * MAX_HISTORY if history else 0
        dist = (ctypes.c_float * max(nd, 1))()
        self._call("ennx_b200_bf16_search_last_scores", scores, count, dist, nd)
        return list(scores)[:count], list(dist)[:nd]

    def _row(self, slot: int):
        """A copy of one resident row (BF16) as a new torch tensor."""
        ptr = ctypes.c_void_p()
        self._call("ennx_b200_bf16_search_row", slot, ctypes.byref(ptr))
        self._handoff(None)
        view = self._torch.from_dlpack(_RawRow(ptr.value, self._len, self._device_index, self))
        return view.clone()


class _RawRow:
    """DLPack producer for a borrowed device row (no lease)."""

    def __init__(self, pointer, n, device, owner):
        self._args = (pointer, n, device, owner)

    def __dlpack_device__(self):
        return (_dlpack.KDL_CUDA, self._args[2])

    def __dlpack__(self, stream=None, max_version=None, dl_device=None, copy=None):
        pointer, n, device, owner = self._args
        return _dlpack.export(owner, pointer, (n,), _dlpack.KDL_BFLOAT, 16, (_dlpack.KDL_CUDA, device),
                              lambda: None, None)


def turbo_enn(base, base_value: float, blocks: Sequence[ParamBlock], capacity: int, *, max_pending: int = 1,
              base_variance: float = 0.0, length_init: float = 0.8, length_min: float = 0.0078125,
              length_max: float = 1.6) -> SearchState:
    """``ennx.experimental.turbo_enn`` (src/ennx/experimental/__init__.py:45-70)."""
    return SearchState(base, base_value, blocks, capacity, max_pending=max_pending, base_variance=base_variance,
                       length_init=length_init, length_min=length_min, length_max=length_max)
