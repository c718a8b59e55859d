"""Packed-weight model package and resident single-token decoder:
``ModelPackage`` and ``NativeKdaModel`` by the names of ``ennx.experimental``.

* ``ModelPackage(path)`` reads the reference's package format (a
  ``model.toml`` manifest naming a packed ``u8`` weight arena and little-endian
  ``f32`` scale and bias arenas, plus one ``[[linear]]`` table per packed
  linear) with the validation and error text of ``PackedModel::open``
  (rust/crates/ennx/src/forward_weights.rs:15-206) and the accessors of the
  PyO3 class (rust/crates/ennx-py/src/py_experimental.rs:20-80).
* ``NativeKdaModel(packed, scales, biases, linears, num_layers, hidden_size,
  heads, head_width, gate_rank, num_experts, top_k, expert_width,
  residual_scale, rms_epsilon, embedding_scale, device)`` is the greedy
  KDA-MoE decoder of py_experimental.rs:163-315 (Metal there) on the CUDA
  decoder of ``libennx_b200.so`` (``ennx_b200_kda_decoder_*``): the weights
  stay packed on the device, each token is one replayed CUDA graph.

The resident packed-trial search of the reference (``resident_session`` /
``ResidentBoSession``) is not part of this package.
"""
from __future__ import annotations

import ctypes
import os
import tomllib
from typing import Sequence

import numpy as np

from . import _abi

__all__ = ["ModelPackage", "NativeKdaModel"]

MANIFEST = "model.toml"
_FIELDS = ("byte_offset", "scale_offset", "bias_offset", "input_width", "output_width", "bits", "group_size",
           "element_offset", "perturb_whole", "perturb_threshold")


def _validate(d: dict) -> None:
    """KdaPackedLinear::validate (rust/crates/ennx/src/forward_program.rs:238-249)."""
    if d["input_width"] == 0 or d["output_width"] == 0 or d["group_size"] == 0:
        raise ValueError("packed KDA linear dimensions must be positive")
    if d["bits"] not in (4, 8):
        raise ValueError(f"packed KDA linear bits must be 4 or 8, got {d['bits']}")


def _packed_bytes(d: dict) -> int:
    per_byte = 2 if d["bits"] == 4 else 1
    return (d["input_width"] + per_byte - 1) // per_byte * d["output_width"]


def _groups_per_row(d: dict) -> int:
    return (d["input_width"] + d["group_size"] - 1) // d["group_size"]


def _read(directory: str, name: str) -> bytes:
    path = os.path.join(directory, name)
    try:
        with open(path, "rb") as f:
            return f.read()
    except OSError as error:
        raise ValueError(f"cannot read {path}: {error}") from None


def _read_f32(directory: str, name: str) -> np.ndarray:
    data = _read(directory, name)
    if len(data) % 4:
        raise ValueError(f"{os.path.join(directory, name)} is not a whole f32 arena")
    return np.frombuffer(data, dtype="<f4").astype(np.float32)


class ModelPackage:
    """An ENNX-native quantized model package (PackedModel::open)."""

    def __init__(self, path: str):
        manifest_path = os.path.join(path, MANIFEST)
        try:
            with open(manifest_path, "rb") as f:
                text = f.read().decode()
        except OSError as error:
            raise ValueError(f"cannot read {manifest_path}: {error}") from None
        try:
            manifest = tomllib.loads(text)
            files = {k: str(manifest[k]) for k in ("weights", "scales", "biases")}
            entries = manifest.get("linear", [])
        except (tomllib.TOMLDecodeError, KeyError, TypeError) as error:
            raise ValueError(f"invalid {manifest_path}: {error}") from None
        self._packed = np.frombuffer(_read(path, files["weights"]), dtype=np.uint8)
        self._scales = _read_f32(path, files["scales"])
        self._biases = _read_f32(path, files["biases"])
        self._linears: dict[str, dict] = {}
        for entry in entries:
            try:
                name = str(entry["name"])
                d = {k: int(entry[k]) for k in _FIELDS[:7]}
                d.update({k: int(entry.get(k, 0)) for k in _FIELDS[7:]})
            except (KeyError, TypeError, ValueError) as error:
                raise ValueError(f"invalid {manifest_path}: {error}") from None
            _validate(d)
            if d["byte_offset"] + _packed_bytes(d) > self._packed.size:
                raise ValueError(f"linear {name!r} exceeds weights arena")
            groups = _groups_per_row(d) * d["output_width"]
            if d["scale_offset"] + groups > self._scales.size or d["bias_offset"] + groups > self._biases.size:
                raise ValueError(f"linear {name!r} exceeds scale or bias arena")
            if name in self._linears:
                raise ValueError(f"duplicate linear name {name!r}")
            self._linears[name] = d

    def linear(self, name: str) -> tuple:
        """The packed descriptor: (byte_offset, scale_offset, bias_offset,
        input_width, output_width, bits, group_size, element_offset,
        perturb_whole, perturb_threshold)."""
        if name not in self._linears:
            raise ValueError(f"model package has no linear {name!r}")
        d = self._linears[name]
        return tuple(d[k] for k in _FIELDS)

    def vector(self, name: str) -> list[float]:
        """Decode a one-row INT8 linear used as a KDA control vector
        (forward_weights.rs:165-184): code * scale + bias per element."""
        d = self._linears.get(name)
        if d is None:
            raise ValueError(f"model package has no linear {name!r}")
        if d["output_width"] != 1 or d["bits"] != 8:
            raise ValueError(f"{name!r} must be a one-row INT8 linear")
        out = []
        for column in range(d["input_width"]):
            code = np.float32(self._packed[d["byte_offset"] + column])
            group = column // d["group_size"]
            out.append(float(np.float32(code * self._scales[d["scale_offset"] + group])
                             + self._biases[d["bias_offset"] + group]))
        return out

    def trial_leaves(self, scale: float = 1.0, weight: float = 1.0, radius: float = 1.0) -> list[tuple]:
        """Leaves of the packed parameter space in element order
        (forward_weights.rs:117-157): (offset, length, bits, scale, weight,
        radius) per linear, contiguous in elements and bytes."""
        element_offset = byte_offset = 0
        leaves = []
        for d in sorted(self._linears.values(), key=lambda d: d["element_offset"]):
            if d["element_offset"] != element_offset:
                raise ValueError(f"linear element offset {d['element_offset']} does not continue parameter "
                                 f"offset {element_offset}")
            if d["byte_offset"] != byte_offset:
                raise ValueError(f"linear byte offset {d['byte_offset']} does not continue packed byte offset "
                                 f"{byte_offset}")
            length = d["input_width"] * d["output_width"]
            leaves.append((d["element_offset"], length, d["bits"], scale, weight, radius))
            element_offset += length
            byte_offset += _packed_bytes(d)
        return leaves

    def linears(self) -> list[tuple]:
        """Every linear as (name, *descriptor), the argument NativeKdaModel takes."""
        return [(name,) + self.linear(name) for name in self._linears]

    @property
    def packed(self) -> np.ndarray:
        return self._packed

    @property
    def scales(self) -> np.ndarray:
        return self._scales

    @property
    def biases(self) -> np.ndarray:
        return self._biases

    @property
    def weight_bytes(self) -> int:
        return int(self._packed.size)

    @property
    def scale_count(self) -> int:
        return int(self._scales.size)

    @property
    def bias_count(self) -> int:
        return int(self._biases.size)


def _linear_struct(t: Sequence[int]) -> _abi.PackedLinear:
    byte, scale, bias, inp, out, bits, group, element, whole, threshold = t
    return _abi.PackedLinear(byte, scale, bias, inp, out, bits, group, element, whole, threshold)


class NativeKdaModel:
    """Resident KDA-MoE greedy decoder on packed weights (py_experimental.rs:
    163-315).  ``linears`` is a sequence of ``(name, byte_offset,
    scale_offset, bias_offset, input_width, output_width, bits, group_size,
    element_offset, perturb_whole, perturb_threshold)``."""

    def __init__(self, packed, scales, biases, linears, num_layers: int, hidden_size: int, heads: int,
                 head_width: int, gate_rank: int, num_experts: int, top_k: int, expert_width: int,
                 residual_scale: float, rms_epsilon: float, embedding_scale: float, device: str = "cuda"):
        value = device.strip().lower()
        if value not in ("", "auto", "cuda"):
            raise ValueError(f"{device!r} decoding is not available in this build; use device='cuda'")
        packed = np.asarray(packed)
        scales = np.asarray(scales)
        biases = np.asarray(biases)
        if packed.dtype != np.uint8 or packed.ndim != 1 or not packed.flags.c_contiguous:
            raise ValueError("packed model arena must be contiguous")
        if scales.dtype != np.float32 or scales.ndim != 1 or not scales.flags.c_contiguous:
            raise ValueError("scale arena must be contiguous")
        if biases.dtype != np.float32 or biases.ndim != 1 or not biases.flags.c_contiguous:
            raise ValueError("bias arena must be contiguous")
        named = {}
        for entry in linears:
            name, *desc = entry
            named[str(name)] = tuple(int(v) for v in desc)

        def get(name):
            if name not in named:
                raise ValueError(f"native model has no linear {name!r}")
            return _linear_struct(named[name])

        E = num_experts
        self._keep = []
        layers = (_abi.KdaDecoderLayer * num_layers)()
        for i in range(num_layers):
            att, moe = f"layers.{i}.attention", f"layers.{i}.moe"
            gate = (_abi.PackedLinear * E)(*[get(f"{moe}.experts.{e}.gate") for e in range(E)])
            up = (_abi.PackedLinear * E)(*[get(f"{moe}.experts.{e}.up") for e in range(E)])
            down = (_abi.PackedLinear * E)(*[get(f"{moe}.experts.{e}.down") for e in range(E)])
            self._keep += [gate, up, down]
            layers[i] = _abi.KdaDecoderLayer(
                get(f"{att}.qkv"), get(f"{att}.control"), get(f"{att}.output"), get(f"{att}.qkv_conv"),
                get(f"{att}.forget_b"), get(f"{att}.gate_b"), get(f"{att}.decay"), get(f"{att}.time_bias"),
                get(f"{att}.output_norm"), get(f"layers.{i}.attention_norm"), get(f"layers.{i}.moe_norm"),
                get(f"{moe}.router"), ctypes.cast(gate, ctypes.c_void_p), ctypes.cast(up, ctypes.c_void_p),
                ctypes.cast(down, ctypes.c_void_p))
        embedding, final_norm = get("embedding"), get("final_norm")
        cfg = _abi.KdaDecoderConfig(num_layers, hidden_size, heads, head_width, gate_rank, num_experts, top_k,
                                    expert_width, residual_scale, rms_epsilon, embedding_scale)
        self._vocab = embedding.output_width
        self._handle = ctypes.c_void_p()
        _abi.call("ennx_b200_kda_decoder_create", packed.ctypes.data_as(ctypes.c_void_p), packed.size,
                  scales.ctypes.data_as(ctypes.c_void_p), scales.size, biases.ctypes.data_as(ctypes.c_void_p),
                  biases.size, ctypes.byref(cfg), layers, ctypes.byref(embedding), ctypes.byref(final_norm), None,
                  ctypes.byref(self._handle))
        self._keep = None

    def __del__(self):
        h = getattr(self, "_handle", None)
        if h is not None and h.value:
            _abi.lib().ennx_b200_kda_decoder_destroy(h)
            self._handle = ctypes.c_void_p()

    def reset(self) -> None:
        """Clear the recurrent state and convolution history of every layer."""
        _abi.call("ennx_b200_kda_decoder_reset", self._handle)

    def prepare_candidate(self, seed: int) -> None:
        """Dequantise the norm, decay and time-bias vectors under ``seed``."""
        _abi.call("ennx_b200_kda_decoder_prepare", self._handle, seed & (2**64 - 1))

    def decode_token(self, token: int, seed: int = 0) -> int:
        out = ctypes.c_uint32(0)
        if not 0 <= token < 2**32:
            raise OverflowError("token must be a u32")
        _abi.call("ennx_b200_kda_decoder_decode_token", self._handle, token, seed & (2**64 - 1), ctypes.byref(out))
        return out.value

    def logits(self) -> np.ndarray:
        """fp32 logits of the last decoded token."""
        out = np.empty(self._vocab, np.float32)
        _abi.call("ennx_b200_kda_decoder_logits", self._handle, out.ctypes.data_as(ctypes.c_void_p), self._vocab)
        return out

    def logit_bits(self) -> list[int]:
        """The last logits as IEEE half bits (the reference's logits are half)."""
        return self.logits().astype(np.float16).view(np.uint16).tolist()

    def generate(self, prompt: Sequence[int], max_new_tokens: int, seed: int = 0) -> list[int]:
        p = np.ascontiguousarray(prompt, dtype=np.uint32)
        if p.size == 0:
            raise ValueError("generation prompt cannot be empty")
        out = np.empty(p.size + max_new_tokens, np.uint32)
        _abi.call("ennx_b200_kda_decoder_generate", self._handle, p.ctypes.data_as(ctypes.c_void_p), p.size,
                  max_new_tokens, seed & (2**64 - 1), out.ctypes.data_as(ctypes.c_void_p))
        return out.tolist()


class PackedKdaBlock:
    """The KDA attention block of one layer of a packed model over whole
    sequences -- the reference's 16k prefill ``KdaMoeMetalExecutor::kda``
    (forward_metal.rs:997-1129) for any length: ``block(normalized, hidden,
    batch, seq, state=None, seed=None)`` adds ``residual_scale * update`` to
    ``hidden`` (CUDA bf16 [batch*seq, hidden]) in place; ``seed`` enables the
    integer-code perturbation of every projection (None: the stored codes,
    the resident-row case), ``state`` (f32 [batch, heads, 128, 128]) carries
    the recurrence.  The arenas are copied to the device once."""

    NAMES = ("qkv", "control", "forget_b", "gate_b", "output", "decay", "time_bias", "output_norm")

    def __init__(self, packed, scales, biases, linears, layer: int, heads: int, gate_rank: int, rms_epsilon: float,
                 residual_scale: float):
        import torch
        named = {str(e[0]): tuple(int(v) for v in e[1:]) for e in linears}
        a = f"layers.{layer}.attention"
        missing = [n for n in self.NAMES if f"{a}.{n}" not in named]
        if missing:
            raise ValueError(f"packed model has no linear {a}.{missing[0]!r}")
        self._block = _abi.PackedKdaBlock(*[_linear_struct(named[f"{a}.{n}"]) for n in self.NAMES], heads, gate_rank,
                                          rms_epsilon, residual_scale)
        self._w = torch.from_numpy(np.ascontiguousarray(packed, np.uint8)).cuda()
        self._s = torch.from_numpy(np.ascontiguousarray(scales, np.float32)).cuda()
        self._b = torch.from_numpy(np.ascontiguousarray(biases, np.float32)).cuda()
        self.heads = heads
        self._ws = None

    def __call__(self, normalized, hidden, batch: int, seq: int, state=None, seed: int | None = None):
        import torch
        for t in (normalized, hidden):
            if t.dtype != torch.bfloat16 or not t.is_cuda or not t.is_contiguous():
                raise ValueError("normalized and hidden must be contiguous CUDA bf16 tensors")
        if normalized.shape != hidden.shape or normalized.shape[0] != batch * seq:
            raise ValueError("normalized and hidden must both be [batch * seq, hidden]")
        H = hidden.shape[1]
        n = _abi.lib().ennx_b200_packed_kda_prefill_workspace_size(ctypes.byref(self._block), batch, seq, H)
        if n == 0:
            _abi.call("ennx_b200_packed_kda_prefill", None, None, None, ctypes.byref(self._block),
                      _abi.PerturbSeed(0, 0, 0), None, None, None, batch, seq, H, None, 0, None)
        if self._ws is None or self._ws.numel() < n:
            self._ws = torch.empty(n, dtype=torch.uint8, device=hidden.device)
        ps = _abi.PerturbSeed(0, 0, 0) if seed is None else _abi.PerturbSeed(seed & 0xFFFFFFFF,
                                                                              (seed >> 32) & 0xFFFFFFFF, 1)
        _abi.call("ennx_b200_packed_kda_prefill", ctypes.c_void_p(self._w.data_ptr()),
                  ctypes.c_void_p(self._s.data_ptr()), ctypes.c_void_p(self._b.data_ptr()), ctypes.byref(self._block),
                  ps, ctypes.c_void_p(normalized.data_ptr()), ctypes.c_void_p(hidden.data_ptr()),
                  None if state is None else ctypes.c_void_p(state.data_ptr()), batch, seq, H,
                  ctypes.c_void_p(self._ws.data_ptr()), self._ws.numel(),
                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        return hidden
