"""Packed-weight quantisers against the reference's known answers
(rust/crates/ennx/src/quantization.rs:47-66) and a scalar restatement of its
loops on random inputs."""
import numpy as np

from ennx_b200.quantization import FP4_E2M1_LUT, quantize_fp4_e2m1, quantize_int4


def test_reference_known_answers():
    assert quantize_int4([0.0, 1.0, 2.0], 1.0).tolist() == [0x10, 0x02]          # pack_odd
    assert quantize_fp4_e2m1([0.0, 1.0, 2.0], 1.0).tolist() == [0x20, 0x04]
    assert quantize_int4([0.5, 1.5, 2.5, 3.5], 1.0).tolist() == [0x20, 0x42]     # round_even
    assert quantize_int4([-3.0, 20.0], 1.0).tolist() == [0xF0]                   # clamp


def _int4_scalar(v, scale):
    q = np.rint(np.float32(v) / np.float32(scale))
    return 0 if (np.isnan(q) or q <= 0) else 15 if q >= 15 else int(q)


def _fp4_scalar(v, scale):
    s = np.float32(v) / np.float32(scale)
    best, code = np.inf, 0
    for c, cand in enumerate(FP4_E2M1_LUT):
        d = abs(s - cand)
        if d < best:
            best, code = d, c
    return code


def _unpack(b, n):
    codes = np.empty(2 * len(b), np.int64)
    codes[0::2], codes[1::2] = b & 15, b >> 4
    return codes[:n].tolist()


def test_vectorised_matches_the_scalar_loops():
    rng = np.random.default_rng(0)
    v = np.concatenate([rng.normal(0, 6, 997).astype(np.float32), [np.nan, np.inf, -np.inf, 0.25, -0.25, 7.5]])
    for scale in (1.0, 0.5, 3.0):
        assert _unpack(quantize_int4(v, scale), len(v)) == [_int4_scalar(x, scale) for x in v]
        assert _unpack(quantize_fp4_e2m1(v, scale), len(v)) == [_fp4_scalar(x, scale) for x in v]


def test_exported_by_experimental():
    from ennx_b200 import experimental
    assert experimental.quantize_int4 is quantize_int4
    assert experimental.quantize_fp4_e2m1 is quantize_fp4_e2m1
