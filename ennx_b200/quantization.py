"""Bit-packed weight quantisers of ``ennx.experimental``:
``quantize_int4`` and ``quantize_fp4_e2m1`` (src/ennx/quantization.py,
rust/crates/ennx/src/quantization.rs:7-45).

Both map ``value / scale`` (float32) to a 4-bit code and pack pairs of codes
into bytes, low nibble first, zero-padding an odd count.  INT4 rounds half to
even and clamps to 0..15 (NaN -> 0); FP4 E2M1 takes the nearest entry of the
E2M1 table, the first one on ties (NaN -> code 0).  These are host-side
format converters (they produce the packed arenas the packed decoder reads),
vectorised with numpy.
"""
from __future__ import annotations

import numpy as np

__all__ = ["FP4_E2M1_LUT", "quantize_fp4_e2m1", "quantize_int4"]

FP4_E2M1_LUT = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0],
                        dtype=np.float32)


def _pack(codes: np.ndarray) -> np.ndarray:
    codes = codes.astype(np.uint8)
    if codes.size % 2:
        codes = np.concatenate([codes, np.zeros(1, np.uint8)])
    return ((codes[0::2] & 0x0F) | ((codes[1::2] & 0x0F) << 4)).astype(np.uint8)


def quantize_int4(arr, scale: float = 1.0) -> np.ndarray:
    q = np.rint(np.asarray(arr, dtype=np.float32).ravel() / np.float32(scale))  # ties to even
    codes = np.where(np.isnan(q) | (q <= 0), 0, np.where(q >= 15, 15, np.nan_to_num(q)))
    return _pack(codes)


def quantize_fp4_e2m1(arr, scale: float = 1.0) -> np.ndarray:
    scaled = np.asarray(arr, dtype=np.float32).ravel() / np.float32(scale)
    dist = np.abs(scaled[:, None] - FP4_E2M1_LUT[None, :])
    dist = np.where(np.isnan(dist), np.inf, dist)
    codes = np.argmin(dist, axis=1)  # first minimum, as the strict '<' scan
    codes = np.where(np.isnan(scaled), 0, codes)
    return _pack(codes)
