"""CPU oracle for the ennx model-evaluation hot path.

TEST INFRASTRUCTURE ONLY.  This package is the checker the CUDA path is
compared against.  It may be imported by ``tests/``, ``__graft_entry__.smoke()``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` -- never by
the ``ennx_b200`` package itself.

Two layers:

* ``libennx_oracle.so`` (``ennx_oracle.c``): a C restatement of the
  reference's integer/rounding-defined math (perturbation hashes, BF16
  encode, fused linear, router reduction order, serial KDA recurrence) and
  scalar references for the forward ops.  Every C function cites the
  Kvutza/ennx file:line it restates.
* numpy definitions below for the dense contractions (GEMM, experts, the
  hybrid forward) in float64, used where a C triple loop would be too slow for
  the parity sizes.

The reference itself is Rust + Zig + Metal and cannot be compiled in this
image (no cargo/rustc/zig, no macOS), so there is no ``oracle/_ref``.
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "libennx_oracle.so"
_lib = None


def build() -> Path:
    """Compile the C oracle (idempotent)."""
    src = _HERE / "ennx_oracle.c"
    if not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.check_call(["make", "-s", "-C", str(_HERE)])
    return _LIB_PATH


class Leaf(ctypes.Structure):
    _fields_ = [("key", ctypes.c_uint64), ("offset", ctypes.c_size_t),
                ("len", ctypes.c_size_t), ("scale", ctypes.c_float)]


class Term(ctypes.Structure):
    _fields_ = [("seed", ctypes.c_uint64), ("coefficient", ctypes.c_float)]


class View(ctypes.Structure):
    _fields_ = [("key", ctypes.c_uint64), ("start", ctypes.c_uint64), ("scale", ctypes.c_float)]


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(_LIB_PATH))
        u64, u32, f32, sz, i32 = (ctypes.c_uint64, ctypes.c_uint32, ctypes.c_float,
                                  ctypes.c_size_t, ctypes.c_int32)
        P = ctypes.c_void_p
        sig = {
            "eo_mix64": (u64, [u64]),
            "eo_dense_sign": (f32, [u64, u64, u64]),
            "eo_tensor_key": (u64, [ctypes.c_char_p]),
            "eo_dense_next": (f32, [f32, ctypes.c_int]),
            "eo_bf16_encode": (ctypes.c_uint16, [f32]),
            "eo_bf16_next": (ctypes.c_uint16, [ctypes.c_uint16, ctypes.c_int]),
            "eo_dense_apply_f32": (i32, [P, sz, P, sz, P, sz, P, P]),
            "eo_dense_apply_bf16": (i32, [P, sz, P, sz, P, sz, P]),
            "eo_dense_dist2": (i32, [P, sz, P, sz, P, sz, P]),
            "eo_dense_linear_f32": (i32, [P, sz, P, sz, P, View, View, P, sz, P]),
            "eo_trial_hash": (u32, [u32, u32, u32]),
            "eo_perturb_code": (u32, [u32, u32, u32, u32, u32, u32, u32]),
            "eo_packed_hash": (u32, [u32, u32, u32]),
            "eo_packed_dequantize": (None, [P, P, P, P, u32, u32, u32, P]),
            "eo_philox4x32_10": (None, [P, P, P]),
            "eo_noise8": (None, [u64, u32, u32, u64, P]),
            "eo_perturb_bf16": (None, [P, sz, u64, u32, u32, f32, ctypes.c_int, P]),
            "eo_perturb_bf16_at": (None, [P, sz, sz, u64, u32, u32, f32, ctypes.c_int, P]),
            "eo_es_update": (None, [P, sz, u64, u32, P, u32, u32, P]),
            "eo_rmsnorm": (None, [P, P, sz, sz, f32, P]),
            "eo_router_logits": (None, [P, P, sz, sz, sz, P]),
            "eo_router_topk": (None, [P, sz, sz, sz, P, P]),
            "eo_kda_gate_beta": (None, [P, P, P, P, sz, sz, sz, P, P]),
            "eo_l2norm_heads": (None, [P, sz, sz]),
            "eo_kda_recurrence": (None, [P, P, P, P, P, sz, sz, sz, sz, sz, P, P]),
            "eo_kda_postprocess": (None, [P, P, P, sz, sz, sz, f32, P]),
            "eo_rope": (None, [P, sz, sz, sz, sz, ctypes.c_double]),
            "eo_gqa_attention": (None, [P, P, P, sz, sz, sz, sz, sz, P]),
            "eo_cross_entropy_rows": (None, [P, P, sz, sz, P]),
            "eo_bf16_seed": (ctypes.c_uint16, [ctypes.c_uint16, u64, u64, u64, f32, f32]),
            "eo_search_candidate": (i32, [P, sz, P, sz, u64, f32, P]),
            "eo_search_distances": (i32, [P, sz, sz, P, sz, P, sz, sz, u64, f32, P]),
            "eo_draw_normal": (ctypes.c_double, [u64, u32, u32]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# ---------------------------------------------------------------------------
# perturbation family
# ---------------------------------------------------------------------------

def mix64(x: int) -> int:
    return lib().eo_mix64(x)


def dense_sign(seed: int, key: int, element: int) -> float:
    return lib().eo_dense_sign(seed, key, element)


def tensor_key(name: str) -> int:
    return lib().eo_tensor_key(name.encode())


def bf16_encode(x: float) -> int:
    return lib().eo_bf16_encode(x)


def bf16_next(v: int, positive: bool) -> int:
    return lib().eo_bf16_next(v, int(positive))


def _leaves(leaves):
    arr = (Leaf * len(leaves))(*[Leaf(int(k), int(o), int(n), float(s)) for k, o, n, s in leaves])
    return arr


def _terms(terms):
    return (Term * max(len(terms), 1))(*[Term(int(s), float(c)) for s, c in terms])


def dense_apply_f32(base, leaves, terms):
    base = _c(base, np.float32)
    out = np.zeros_like(base)
    changed = ctypes.c_size_t(0)
    lv, tm = _leaves(leaves), _terms(terms)
    st = lib().eo_dense_apply_f32(_p(base), base.size, ctypes.cast(lv, ctypes.c_void_p), len(leaves),
                                  ctypes.cast(tm, ctypes.c_void_p), len(terms), _p(out),
                                  ctypes.cast(ctypes.pointer(changed), ctypes.c_void_p))
    return st, out, changed.value


def dense_apply_bf16(base_bits, leaves, terms):
    base = _c(base_bits, np.uint16)
    out = np.zeros_like(base)
    lv, tm = _leaves(leaves), _terms(terms)
    st = lib().eo_dense_apply_bf16(_p(base), base.size, ctypes.cast(lv, ctypes.c_void_p), len(leaves),
                                   ctypes.cast(tm, ctypes.c_void_p), len(terms), _p(out))
    return st, out


def dense_dist2(leaves, left, right):
    out = ctypes.c_double(0)
    lv, a, b = _leaves(leaves), _terms(left), _terms(right)
    st = lib().eo_dense_dist2(ctypes.cast(lv, ctypes.c_void_p), len(leaves), ctypes.cast(a, ctypes.c_void_p),
                              len(left), ctypes.cast(b, ctypes.c_void_p), len(right),
                              ctypes.cast(ctypes.pointer(out), ctypes.c_void_p))
    return st, out.value


def dense_linear_f32(x, weight, bias, weight_view, bias_view, terms):
    x = _c(x, np.float32)
    w = _c(weight, np.float32)
    rows = w.size // x.size
    out = np.zeros(rows, np.float32)
    b = None if bias is None else _c(bias, np.float32)
    tm = _terms(terms)
    st = lib().eo_dense_linear_f32(_p(x), x.size, _p(w), rows, None if b is None else _p(b),
                                   View(*weight_view), View(*(bias_view or (0, 0, 1.0))),
                                   ctypes.cast(tm, ctypes.c_void_p), len(terms), _p(out))
    return st, out


def trial_hash(lo: int, hi: int, element: int) -> int:
    return lib().eo_trial_hash(lo, hi, element)


class PackedLinear(ctypes.Structure):
    """eo_packed_linear: field order of KdaPackedLinear (forward_program.rs:224-235)."""
    _fields_ = [("byte_offset", ctypes.c_uint64), ("scale_offset", ctypes.c_uint64),
                ("bias_offset", ctypes.c_uint64), ("input_width", ctypes.c_uint64),
                ("output_width", ctypes.c_uint64), ("bits", ctypes.c_uint32), ("group_size", ctypes.c_uint32),
                ("element_offset", ctypes.c_uint64), ("perturb_whole", ctypes.c_uint32),
                ("perturb_threshold", ctypes.c_uint32)]


def packed_hash(lo: int, hi: int, element: int) -> int:
    return int(lib().eo_packed_hash(lo, hi, element))


def packed_dequantize(weights, scales, biases, linear: "PackedLinear", seed=(0, 0, 0)) -> np.ndarray:
    """float32 [output_width, input_width] of the (perturbed) packed weights."""
    w, sc, bi = _c(weights, np.uint8), _c(scales, np.float32), _c(biases, np.float32)
    out = np.zeros((linear.output_width, linear.input_width), np.float32)
    lib().eo_packed_dequantize(_p(w), _p(sc), _p(bi), ctypes.byref(linear), seed[0], seed[1], seed[2], _p(out))
    return out


def perturb_code(code, lo, hi, element, bits, whole, threshold) -> int:
    return lib().eo_perturb_code(code, lo, hi, element, bits, whole, threshold)


# ---------------------------------------------------------------------------
# population noise
# ---------------------------------------------------------------------------

def philox4x32_10(ctr, key):
    c = _c(ctr, np.uint32)
    k = _c(key, np.uint32)
    out = np.zeros(4, np.uint32)
    lib().eo_philox4x32_10(_p(c), _p(k), _p(out))
    return out


def noise(seed: int, pair: int, tensor: int, n: int, start: int = 0) -> np.ndarray:
    """N(0,1) draws for elements [start, start+n) of one tensor (start % 8 == 0)."""
    assert start % 8 == 0
    out = np.zeros(((n + 7) // 8) * 8, np.float32)
    buf = np.zeros(8, np.float32)
    for blk in range((n + 7) // 8):
        lib().eo_noise8(seed, pair, tensor, start // 8 + blk, _p(buf))
        out[8 * blk:8 * blk + 8] = buf
    return out[:n]


def es_coefficients(fitness, sigma, lr, total_pairs=None):
    """coef[p] = -lr (f[2p] - f[2p+1]) / (2 sigma total_pairs), float32 arithmetic."""
    f = np.asarray(fitness, np.float32)
    P = f.size // 2
    scale = np.float32(-lr) / (np.float32(2.0) * np.float32(sigma) * np.float32(total_pairs or P))
    return (scale * (f[0::2] - f[1::2])).astype(np.float32)


def es_update(w_bits, seed, tensor, coef, first_pair=0):
    """bf16 bits of W + sum_p coef[p] eps(seed, first_pair + p, tensor, .)."""
    w = _c(w_bits, np.uint16).reshape(-1)
    c = _c(coef, np.float32)
    out = np.zeros_like(w)
    lib().eo_es_update(_p(w), w.size, seed, tensor, _p(c), first_pair, c.size, _p(out))
    return out.reshape(np.shape(w_bits))


def noise_step_bf16(n, seed, pair, tensor, sigma):
    """bf16 bits of the noise step e = bf16(sigma * eps) for elements [0, n)."""
    out = np.zeros(n, np.uint16)
    lib().eo_perturb_bf16_at(None, n, 0, seed, pair, tensor, sigma, 1, _p(out))
    return out


def perturb_bf16(w_bits, seed, pair, tensor, sigma, sign):
    """bf16 bits of W + sign*sigma*eps.  Tensors above 4 M elements are split
    over host threads (the C function releases the GIL under ctypes)."""
    w = _c(w_bits, np.uint16).reshape(-1)
    out = np.zeros_like(w)
    n = w.size
    chunk = 1 << 22
    if n <= chunk:
        lib().eo_perturb_bf16(_p(w), n, seed, pair, tensor, sigma, int(sign), _p(out))
        return out.reshape(np.shape(w_bits))
    import concurrent.futures as cf

    def run(s0):
        m = min(chunk, n - s0)
        lib().eo_perturb_bf16_at(w[s0:].ctypes.data_as(ctypes.c_void_p), m, s0, seed, pair, tensor, sigma, int(sign),
                                 out[s0:].ctypes.data_as(ctypes.c_void_p))
    with cf.ThreadPoolExecutor(os.cpu_count() or 1) as ex:
        list(ex.map(run, range(0, n, chunk)))
    return out.reshape(np.shape(w_bits))


# ---------------------------------------------------------------------------
# bf16 helpers (round-to-nearest-even, same formula as the reference)
# ---------------------------------------------------------------------------

def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)


def from_bf16_bits(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    return from_bf16_bits(to_bf16_bits(x))


# ---------------------------------------------------------------------------
# forward ops
# ---------------------------------------------------------------------------

def gemm(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """C = A . B^T in float64 (A [M,K], B [N,K])."""
    return np.asarray(a, np.float64) @ np.asarray(b, np.float64).T


def rmsnorm(x, w, eps=1e-6):
    x = _c(x, np.float32)
    rows, width = x.reshape(-1, x.shape[-1]).shape
    out = np.zeros_like(x)
    lib().eo_rmsnorm(_p(x), _p(_c(w, np.float32)), rows, width, eps, _p(out))
    return out


def router_logits(x_bits, w_bits):
    x = _c(x_bits, np.uint16)
    w = _c(w_bits, np.uint16)
    T, H = x.shape
    E = w.shape[0]
    assert H % 256 == 0
    out = np.zeros((T, E), np.float32)
    lib().eo_router_logits(_p(x), _p(w), T, H, E, _p(out))
    return out


def router_topk(logits, k):
    lg = _c(logits, np.float32)
    T, E = lg.shape
    idx = np.zeros((T, k), np.int32)
    gate = np.zeros((T, k), np.float32)
    lib().eo_router_topk(_p(lg), T, E, k, _p(idx), _p(gate))
    return idx, gate


def silu(x):
    return x / (1.0 + np.exp(-x))


def moe_experts(x, idx, gate, w_gate, w_up, w_down):
    """y[t] = sum_r gate[t,r] * W_d[e] (silu(W_g[e] x) * (W_u[e] x)), float64.

    Restates kda_moe.metal:691-755.  w_gate/w_up: [E, I, H], w_down: [E, H, I]."""
    x = np.asarray(x, np.float64)
    T, H = x.shape
    y = np.zeros((T, H), np.float64)
    E = w_gate.shape[0]
    for e in range(E):
        rows, ranks = np.nonzero(idx == e)
        if rows.size == 0:
            continue
        xe = x[rows]
        a = silu(xe @ np.asarray(w_gate[e], np.float64).T) * (xe @ np.asarray(w_up[e], np.float64).T)
        out = a @ np.asarray(w_down[e], np.float64).T
        np.add.at(y, rows, out * gate[rows, ranks][:, None])
    return y


def kda_gate_beta(raw_gate, raw_beta, decay, time_bias, heads, head_width):
    rg = _c(raw_gate, np.float32)
    rb = _c(raw_beta, np.float32)
    tokens = rg.size // (heads * head_width)
    g = np.zeros_like(rg)
    b = np.zeros_like(rb)
    lib().eo_kda_gate_beta(_p(rg), _p(rb), _p(_c(decay, np.float32)), _p(_c(time_bias, np.float32)),
                           tokens, heads, head_width, _p(g), _p(b))
    return g, b


def l2norm_heads(x):
    y = _c(x, np.float32).copy()
    lib().eo_l2norm_heads(_p(y), y.size // y.shape[-1], y.shape[-1])
    return y


def kda_recurrence(q, k, v, g, beta, state=None):
    """Serial reference recurrence; q,k,g [B,T,H,dk], v [B,T,H,dv], beta [B,T,H]."""
    q, k, v, g, beta = (_c(a, np.float32) for a in (q, k, v, g, beta))
    B, T, H, dk = q.shape
    dv = v.shape[-1]
    st = np.zeros((B, H, dk, dv), np.float32) if state is None else _c(state, np.float32).copy()
    out = np.zeros((B, T, H, dv), np.float32)
    lib().eo_kda_recurrence(_p(q), _p(k), _p(v), _p(g), _p(beta), B, T, H, dk, dv, _p(st), _p(out))
    return out, st


def kda_postprocess(o, gate, norm, eps=1e-6):
    o = _c(o, np.float32)
    heads, width = o.shape[-2], o.shape[-1]
    tokens = o.size // (heads * width)
    out = np.zeros_like(o)
    lib().eo_kda_postprocess(_p(o), _p(_c(gate, np.float32)), _p(_c(norm, np.float32)), tokens,
                             heads, width, eps, _p(out))
    return out


def rope(x, theta=1e6):
    y = _c(x, np.float32).copy()
    B, S, H, D = y.shape
    lib().eo_rope(_p(y), B, S, H, D, theta)
    return y


def gqa_attention(q, k, v):
    q, k, v = (_c(a, np.float32) for a in (q, k, v))
    B, S, Hq, D = q.shape
    Hkv = k.shape[2]
    out = np.zeros_like(q)
    lib().eo_gqa_attention(_p(q), _p(k), _p(v), B, S, Hq, Hkv, D, _p(out))
    return out


def cross_entropy_rows(logits, targets):
    lg = _c(logits, np.float32)
    t = _c(targets, np.int32)
    out = np.zeros(lg.shape[0], np.float64)
    lib().eo_cross_entropy_rows(_p(lg), _p(t), lg.shape[0], lg.shape[1], _p(out))
    return out


def softplus(x):
    return np.maximum(x, 0) + np.log1p(np.exp(-np.abs(x)))


__all__ = [n for n in dir() if not n.startswith("_")]
_ = (math, os)
