"""Python surface of the seeded dense perturbation path, by the names of
``ennx.experimental`` (src/ennx/experimental/__init__.py:7-46).

* ``ParamBlock``  - rust/crates/ennx-py/src/py_bf16.rs:15-55 (validation of
  rust/crates/ennx/src/bf16_search.rs:18-40);
* ``ParamBuffer`` - py_weights.rs:31-122 (the resident BF16 pytree:
  ``ParamBuffer::from_device`` + ``materialize``, rust/crates/ennx/src/dense/
  bf16.rs:107-150, cuda/src/lib.rs:1166-1252) with the DLPack lease;
* ``dense_apply`` / ``dense_dist2`` / ``dense_linear`` - py_weights.rs:188-252;
* ``DenseLinear`` - py_weights.rs:254-306 (rust/crates/ennx/src/dense/
  linear.rs:53-247).

Argument meaning, defaults and error text follow the reference: every
rejected input raises ``ValueError`` with the reference's message.  The work
runs on CUDA through ``libennx_b200.so``; there is no CPU path, so
``device`` accepts ``"auto"`` and ``"cuda"`` and names any other backend of
the reference as not available in this build.
"""
from __future__ import annotations

import ctypes
import math
from typing import Iterable, Sequence

import numpy as np

from . import _abi, _dlpack

__all__ = ["DenseLinear", "ParamBlock", "ParamBuffer", "dense_apply", "dense_dist2", "dense_linear",
           "tensor_key"]

_U64 = (1 << 64) - 1
_BACKENDS = {"cpu": "CPU", "metal": "Metal", "agx": "AGX", "opencl": "OpenCL", "ocl": "OpenCL"}


def tensor_key(name: str) -> int:
    """Stable 64-bit leaf key of a named tensor: an FNV-1a-style fold over the
    UTF-8 bytes with the reference's offset basis 1469598103934665603 (not
    the textbook FNV basis) and prime 1099511628211
    (rust/crates/ennx/src/dense.rs:57-64)."""
    key = 1_469_598_103_934_665_603
    for byte in name.encode():
        key = ((key ^ byte) * 1_099_511_628_211) & _U64
    return key


def _device(name: str, what: str) -> None:
    """ComputeDevice::parse (rust/crates/ennx/src/weights.rs:50-62), then the
    build's availability check."""
    value = name.strip().lower()
    if value in ("", "auto", "cuda"):
        return
    if value in _BACKENDS:
        raise ValueError(f"{_BACKENDS[value]} {what} not available in this build")
    raise ValueError(f"unknown compute device {value!r}; expected 'auto', 'cpu', 'metal', 'agx', 'opencl', "
                     "or 'cuda'")


def _f32(x) -> float:
    return float(np.float32(x))


def _leaves(raw: Iterable[Sequence]) -> list[tuple[int, int, int, float]]:
    """DenseLeaf::new per leaf (dense.rs:33-48)."""
    out = []
    for key, offset, length, scale in raw:
        scale = _f32(scale)
        if length == 0:
            raise ValueError("dense leaf length must be positive")
        if not math.isfinite(scale) or scale <= 0.0:
            raise ValueError("dense leaf scale must be finite and positive")
        out.append((int(key), int(offset), int(length), scale))
    return out


def _terms(raw: Iterable[Sequence]) -> list[tuple[int, float]]:
    """DenseTerm::new per term (dense.rs:66-73)."""
    out = []
    for seed, coefficient in raw:
        coefficient = _f32(coefficient)
        if not math.isfinite(coefficient):
            raise ValueError("dense coefficient must be finite")
        out.append((int(seed), coefficient))
    return out


def _view(raw: Sequence) -> _abi.DenseView:
    """DenseView::new (rust/crates/ennx/src/dense/linear.rs:22-28)."""
    key, start, scale = raw
    scale = _f32(scale)
    if not math.isfinite(scale) or scale <= 0.0:
        raise ValueError("dense view scale must be finite and positive")
    return _abi.DenseView(int(key), int(start), scale)


def _leaf_array(leaves):
    return (_abi.DenseLeaf * max(len(leaves), 1))(*[_abi.DenseLeaf(*leaf) for leaf in leaves])


def _term_array(terms):
    return (_abi.DenseTerm * max(len(terms), 1))(*[_abi.DenseTerm(*term) for term in terms])


def _has_direction(terms) -> bool:
    """Some seed's summed coefficient is non-zero (dense.rs:258-265)."""
    sums: dict[int, float] = {}
    for seed, coefficient in terms:
        sums[seed] = sums.get(seed, 0.0) + coefficient
    return any(v != 0.0 for v in sums.values())


def _vector(x, what: str) -> np.ndarray:
    a = np.ascontiguousarray(x, dtype=np.float32)
    if a.ndim != 1:
        raise ValueError(f"{what} must be one-dimensional")
    return a


def _matrix(x, what: str) -> np.ndarray:
    a = np.ascontiguousarray(x, dtype=np.float32)
    if a.ndim != 2:
        raise ValueError(f"{what} must be two-dimensional")
    return a


def _torch():
    import torch
    if not torch.cuda.is_available():
        raise _abi.EnnxB200Error(_abi.CUDA_ERROR, "ennx_b200 needs a CUDA device; none is visible")
    return torch


def _stream(torch):
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t) -> ctypes.c_void_p | None:
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def dense_dist2(leaves, left, right) -> float:
    """Squared L2 distance between the perturbations of two term lists:
    (sum of len * scale^2) * sum over seeds of (c_left - c_right)^2
    (py_weights.rs:207-221 -> dense.rs:191-196 -> ennx_dense_dist2).  Host
    arithmetic; no device is needed."""
    lv, lt, rt = _leaves(leaves), _terms(left), _terms(right)
    out = ctypes.c_double(0.0)
    _abi.call("ennx_b200_dense_dist2", _leaf_array(lv), len(lv), _term_array(lt), len(lt), _term_array(rt),
              len(rt), ctypes.byref(out))
    return out.value


def dense_apply(base, leaves, terms, device: str = "auto") -> tuple[np.ndarray, int]:
    """``values = base + scale * sum(c_i * sign_i)`` with the one-ulp rule, over
    an f32 flat pytree; returns ``(values, changed)`` (py_weights.rs:188-205,
    dense.rs:76-183).  Copies ``base`` to the device, runs
    ``ennx_b200_dense_apply_f32`` and copies the values back."""
    lv, tm = _leaves(leaves), _terms(terms)
    _device(device, "dense directions are")
    host = _vector(base, "dense base")
    if host.size == 0:
        raise ValueError("dense base cannot be empty")
    if not np.isfinite(host).all():
        raise ValueError("dense base values must be finite")
    torch = _torch()
    d_base = torch.from_numpy(host).cuda()
    d_out = torch.empty_like(d_base)
    changed = ctypes.c_size_t(0)
    _abi.call("ennx_b200_dense_apply_f32", _ptr(d_base), host.size, _leaf_array(lv), len(lv), _term_array(tm),
              len(tm), _ptr(d_out), ctypes.byref(changed), _stream(torch))
    return d_out.cpu().numpy(), changed.value


class ParamBlock:
    """One leaf of a BF16 pytree: ``(key, offset, length, scale, weight)``
    (py_bf16.rs:15-55; bf16_search.rs:18-40).  Immutable."""

    __slots__ = ("_key", "_offset", "_length", "_scale", "_weight")

    def __init__(self, key: int, offset: int, length: int, scale: float, weight: float = 1.0):
        scale, weight = _f32(scale), _f32(weight)
        if length == 0:
            raise ValueError("BF16 block length must be positive")
        if not math.isfinite(scale) or scale <= 0.0 or not math.isfinite(weight) or weight <= 0.0:
            raise ValueError("BF16 block scale and weight must be positive")
        if not 0 <= int(key) <= _U64 or int(offset) < 0 or int(length) < 0:
            raise OverflowError("ParamBlock fields are unsigned")
        object.__setattr__(self, "_key", int(key))
        object.__setattr__(self, "_offset", int(offset))
        object.__setattr__(self, "_length", int(length))
        object.__setattr__(self, "_scale", scale)
        object.__setattr__(self, "_weight", weight)

    def __setattr__(self, name, value):
        raise AttributeError("ParamBlock is immutable")

    key = property(lambda self: self._key)
    offset = property(lambda self: self._offset)
    length = property(lambda self: self._length)
    scale = property(lambda self: self._scale)
    weight = property(lambda self: self._weight)

    def __repr__(self):
        return (f"ParamBlock(key={self._key}, offset={self._offset}, length={self._length}, "
                f"scale={self._scale}, weight={self._weight})")


def _bf16_input(base):
    """DLPack import of a contiguous, non-empty BF16 CUDA tensor
    (rust/crates/ennx-py/src/dlpack.rs:86-160); returns a torch view."""
    torch = _torch()
    if isinstance(base, torch.Tensor):
        t = base
    elif hasattr(base, "__dlpack__"):
        t = torch.from_dlpack(base)
    else:
        raise TypeError("ParamBuffer base must support the DLPack protocol")
    if t.dtype != torch.bfloat16:
        raise ValueError("DLPack tensor must be BF16")
    if not t.is_cuda:
        raise ValueError("DLPack tensor must live on a CUDA device")
    if not t.is_contiguous():
        raise BufferError("BF16 input requires a contiguous DLPack tensor")
    if t.numel() == 0:
        raise ValueError("BF16 input requires a non-empty tensor")
    return torch, t


class ParamBuffer:
    """A resident BF16 pytree and one perturbed candidate of it.

    ``ParamBuffer(base, blocks)`` copies ``base`` (any DLPack BF16 CUDA
    tensor) into storage this object owns; ``materialize(terms)`` writes
    ``candidate = bf16(base + scale * sum(c_i * sign_i))`` with the one-ulp
    rule, rolling the candidate back to ``base`` on overflow; the candidate
    is exported zero-copy through ``__dlpack__``.  While an export is alive,
    ``materialize`` refuses, so the exported array never changes
    (py_weights.rs:31-122).  Not thread-safe (the reference class is
    ``unsendable``).
    """

    def __init__(self, base, blocks: Sequence[ParamBlock]):
        leaves = []
        for block in blocks:
            if not isinstance(block, ParamBlock):
                raise TypeError("ParamBuffer blocks must be ParamBlock instances")
            leaves.append((block.key, block.offset, block.length, block.scale))
        leaves = _leaves(leaves)
        torch, src = _bf16_input(base)
        n = src.numel()
        if not leaves:
            raise ValueError("at least one dense leaf is required")
        self._check_layout(n, leaves)
        self._device = src.device
        with torch.cuda.device(self._device):
            self._base = torch.empty(n, dtype=torch.bfloat16, device=self._device)
            self._base.copy_(src.reshape(-1))
            self._candidate = self._base.clone()
            torch.cuda.current_stream().synchronize()
            flag = ctypes.c_int32(0)
            _abi.call("ennx_b200_check_bf16", _ptr(self._base), n, ctypes.byref(flag), _stream(torch))
        if not flag.value:
            raise ValueError("CUDA BF16 base values must be finite")
        self._leaves = _leaf_array(leaves)
        self._num_leaves = len(leaves)
        self._exported = False

    @staticmethod
    def _check_layout(n, leaves):
        """validate_leaves (dense.rs:213-245) at construction, as
        ParamBuffer::from_device does; the C ABI repeats it per call."""
        end = 0
        for _, offset, length, _ in leaves:
            if offset != end:
                raise ValueError(f"dense leaf offset {offset} does not continue parameter offset {end}")
            end = offset + length
        if end != n:
            raise ValueError(f"dense leaves cover {end} parameters, expected {n}")

    def materialize(self, terms) -> None:
        if self._exported:
            raise ValueError("cannot materialize while a JAX candidate is alive")
        tm = _terms(terms)
        if not _has_direction(tm):
            raise ValueError("BF16 pytree terms cancel to zero")
        import torch
        with torch.cuda.device(self._device):
            _abi.call("ennx_b200_dense_apply_bf16", _ptr(self._base), self._base.numel(), self._leaves,
                      self._num_leaves, _term_array(tm), len(tm), _ptr(self._candidate), _stream(torch))

    def materialize_gaussian(self, seed: int, pair: int, sigma: float, sign: int = 1) -> None:
        """The Philox Gaussian direction of the population forward instead of
        Rademacher terms: for leaf j (in block order) and element i of it,
        ``candidate = bf16(base + s * bf16(sigma * scale_j * eps(seed, pair,
        j, i)))``, s = +1 or -1 (the antithetic sign) -- the same noise and
        rounding as ``ennx_b200_perturb_bf16``.  Rolls back to ``base`` and
        raises if any value overflows, like ``materialize``."""
        if self._exported:
            raise ValueError("cannot materialize while a JAX candidate is alive")
        if sign not in (1, -1):
            raise ValueError("the antithetic sign must be +1 or -1")
        sigma = _f32(sigma)
        if not math.isfinite(sigma) or sigma < 0.0:
            raise ValueError("sigma must be finite and non-negative")
        if not 0 <= int(seed) <= _U64 or not 0 <= int(pair) < 2 ** 32:
            raise ValueError("seed must be a u64 and pair a u32")
        import torch
        with torch.cuda.device(self._device):
            st = _stream(torch)
            for j in range(self._num_leaves):
                leaf = self._leaves[j]
                off, n = int(leaf.offset), int(leaf.len)
                aligned = off % 8 == 0  # the kernel takes 16-byte aligned rows; other leaves go through copies
                base = self._base[off:off + n] if aligned else self._base[off:off + n].clone()
                cand = self._candidate[off:off + n] if aligned else torch.empty_like(base)
                scaled = float(np.float32(sigma) * np.float32(leaf.scale))
                if sign > 0:
                    _abi.call("ennx_b200_perturb_bf16", _ptr(base), n, int(seed), int(pair), j, scaled, _ptr(cand),
                              None, st)
                else:  # the minus copy, into the candidate (the plus copy into a scratch)
                    scratch = torch.empty_like(cand)
                    _abi.call("ennx_b200_perturb_bf16", _ptr(base), n, int(seed), int(pair), j, scaled,
                              _ptr(scratch), _ptr(cand), st)
                if not aligned:
                    self._candidate[off:off + n].copy_(cand)
            flag = ctypes.c_int32(0)
            torch.cuda.current_stream().synchronize()
            _abi.call("ennx_b200_check_bf16", _ptr(self._candidate), self._candidate.numel(), ctypes.byref(flag), st)
        if not flag.value:
            self._candidate.copy_(self._base)
            torch.cuda.current_stream().synchronize()
            raise ValueError("BF16 Gaussian perturbation overflowed")

    def __dlpack_device__(self) -> tuple[int, int]:
        return (_dlpack.KDL_CUDA, self._device.index or 0)

    def __dlpack__(self, stream: int | None = None, max_version: tuple[int, int] | None = None,
                   dl_device: tuple[int, int] | None = None, copy: bool | None = None):
        if copy is True:
            raise BufferError("ParamBuffer does not export copies")
        if dl_device is not None and tuple(dl_device) != self.__dlpack_device__():
            raise BufferError("ParamBuffer cannot export to another device")
        if stream is not None and (stream == 0 or stream < -1):
            raise ValueError("invalid DLPack CUDA stream")
        if self._exported:
            raise ValueError("the current BF16 candidate is already exported")
        # materialize() synchronises before it returns, so the candidate is
        # complete on every stream and no event hand-off is needed.
        self._exported = True

        def release():
            self._exported = False

        return _dlpack.export(self, self._candidate.data_ptr(), (self._candidate.numel(),), _dlpack.KDL_BFLOAT,
                              16, self.__dlpack_device__(), release, max_version)

    @property
    def len(self) -> int:
        return self._base.numel()

    def __len__(self) -> int:
        return self._base.numel()


def _model(weight, bias, weight_view, bias_view):
    """validate_model (rust/crates/ennx/src/dense/linear.rs:392-431)."""
    w = _matrix(weight, "dense linear weight")
    rows, columns = w.shape
    if columns == 0 or w.size == 0:
        raise ValueError("dense linear weight must contain complete non-empty rows")
    b = None if bias is None else _vector(bias, "dense linear bias")
    if b is not None and b.size != rows:
        raise ValueError("dense linear bias length must equal the weight row count")
    if (b is None) != (bias_view is None):
        raise ValueError("dense linear bias and bias view must be supplied together")
    if not np.isfinite(w).all() or (b is not None and not np.isfinite(b).all()):
        raise ValueError("dense linear weights must be finite")
    if weight_view.start + w.size > _U64:
        raise ValueError("dense linear weight coordinates overflow u64")
    if bias_view is not None and bias_view.start + rows > _U64:
        raise ValueError("dense linear bias coordinates overflow u64")
    return w, b, rows, columns


def _eval_terms(x, columns, terms):
    """validate_eval (linear.rs:433-446)."""
    if x.size != columns or not np.isfinite(x).all():
        raise ValueError(f"dense linear input must contain {columns} finite values")
    if not terms:
        raise ValueError("dense linear requires finite perturbation terms")
    if not _has_direction(terms):
        raise ValueError("dense linear terms cancel to zero")


class DenseLinear:
    """A resident fused perturbed linear layer ``y = W~ x (+ b~)``.

    ``W`` (and ``b``) are copied to the device once; every ``eval(input,
    terms)`` copies the input up, runs ``ennx_b200_dense_linear_f32`` (one
    serial-``fma`` dot product per row, the order of linear_cpu,
    linear.rs:484-519) and reads the outputs back (py_weights.rs:254-306).
    """

    def __init__(self, weight, weight_view, bias=None, bias_view=None, device: str = "auto"):
        wv = _view(weight_view)
        bv = None if bias_view is None else _view(bias_view)
        _device(device, "dense linear is")
        w, b, self._rows, self._columns = _model(weight, bias, wv, bv)
        torch = _torch()
        self._weight = torch.from_numpy(w).cuda()
        self._bias = None if b is None else torch.from_numpy(b).cuda()
        self._out = torch.empty(self._rows, dtype=torch.float32, device=self._weight.device)
        self._wv = wv
        self._bv = bv if bv is not None else _abi.DenseView(0, 0, 1.0)

    def eval(self, input, terms) -> np.ndarray:
        x = _vector(input, "dense linear input")
        tm = _terms(terms)
        _eval_terms(x, self._columns, tm)
        import torch
        with torch.cuda.device(self._weight.device):
            d_x = torch.from_numpy(x).cuda()
            _abi.call("ennx_b200_dense_linear_f32", _ptr(d_x), self._columns, _ptr(self._weight), self._rows,
                      _ptr(self._bias), self._wv, self._bv, _term_array(tm), len(tm), _ptr(self._out),
                      _stream(torch))
            y = self._out.cpu().numpy()
        if not np.isfinite(y).all():
            raise ValueError("dense linear overflowed FP32")
        return y

    @property
    def input_size(self) -> int:
        return self._columns

    @property
    def output_size(self) -> int:
        return self._rows


def dense_linear(input, weight, weight_view, terms, bias=None, bias_view=None, device: str = "auto") -> np.ndarray:
    """One-shot fused perturbed linear layer (py_weights.rs:223-252 ->
    rust/crates/ennx/src/dense/linear.rs:249-389)."""
    wv = _view(weight_view)
    tm = _terms(terms)
    bv = None if bias_view is None else _view(bias_view)
    _device(device, "dense linear is")
    w, b, _, columns = _model(weight, bias, wv, bv)
    _eval_terms(_vector(input, "dense linear input"), columns, tm)
    return DenseLinear(w, weight_view, b, bias_view, device).eval(input, terms)


# The resident search classes live in ennx_b200.search (which imports this
# module's ParamBlock and DLPack import) and the packed model classes in
# ennx_b200.native; they resolve here on first use, as the reference's
# experimental namespace resolves its names lazily.
_SEARCH_NAMES = ("Proposals", "SearchState", "turbo_enn")
_NATIVE_NAMES = ("ModelPackage", "NativeKdaModel")
_QUANT_NAMES = ("quantize_int4", "quantize_fp4_e2m1")
__all__ += list(_SEARCH_NAMES) + list(_NATIVE_NAMES) + list(_QUANT_NAMES)


def __getattr__(name: str):
    if name in _SEARCH_NAMES:
        from . import search
        return getattr(search, name)
    if name in _NATIVE_NAMES:
        from . import native
        return getattr(native, name)
    if name in _QUANT_NAMES:
        from . import quantization
        return getattr(quantization, name)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
