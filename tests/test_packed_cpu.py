"""Packed int4/int8 weights: oracle properties of the Metal restatement
(kda_moe.metal:63-96, 351-395).  The reference has no CPU implementation or
known-answer vectors for this path (Metal only), so these pin the rules the
source states: hash variant, code range, step size and reflection."""
import numpy as np

import oracle as O


def _linear(inp, out, bits, group, whole=0, threshold=0, element_offset=0):
    return O.PackedLinear(byte_offset=0, scale_offset=0, bias_offset=0, input_width=inp, output_width=out,
                          bits=bits, group_size=group, element_offset=element_offset, perturb_whole=whole,
                          perturb_threshold=threshold)


def _codes(rng, inp, out, bits):
    codes = rng.integers(0, 1 << bits, size=(out, inp), dtype=np.uint32)
    if bits == 8:
        return codes, codes.astype(np.uint8).reshape(-1)
    row_bytes = (inp + 1) // 2
    packed = np.zeros((out, row_bytes), np.uint8)
    for c in range(inp):
        packed[:, c // 2] |= (codes[:, c] << (4 * (c & 1))).astype(np.uint8)
    return codes, packed.reshape(-1)


def test_metal_hash_differs_from_cuda_trial_hash():
    # kda_moe.metal XORs seed.high after the last multiply; cuda lib.rs before it
    diff = sum(O.packed_hash(5, 9, e) != O.trial_hash(5, 9, e) for e in range(64))
    assert diff > 60


def test_unperturbed_is_code_times_scale_plus_bias():
    rng = np.random.default_rng(0)
    for bits in (4, 8):
        inp, out, group = 70, 5, 32  # ragged last group
        codes, packed = _codes(rng, inp, out, bits)
        groups = (inp + group - 1) // group
        sc = rng.standard_normal(out * groups).astype(np.float32)
        bi = rng.standard_normal(out * groups).astype(np.float32)
        w = O.packed_dequantize(packed, sc, bi, _linear(inp, out, bits, group))
        g = np.minimum(np.arange(inp) // group, groups - 1)
        ref = codes.astype(np.float64) * sc.reshape(out, groups)[:, g] + bi.reshape(out, groups)[:, g]
        np.testing.assert_allclose(w, ref, rtol=1e-6, atol=1e-6)


def test_perturbed_codes_stay_in_range_and_move_by_the_amount():
    rng = np.random.default_rng(1)
    for bits in (4, 8):
        inp, out = 64, 8
        codes, packed = _codes(rng, inp, out, bits)
        one, zero = np.ones(out, np.float32), np.zeros(out, np.float32)
        lin = _linear(inp, out, bits, inp, whole=1, threshold=0)  # amount exactly 1 everywhere
        w = O.packed_dequantize(packed, one, zero, lin, seed=(0x1234, 0x9876, 1)).astype(np.int64)
        assert w.min() >= 0 and w.max() <= (1 << bits) - 1
        assert np.all(np.abs(w - codes.astype(np.int64)) == 1)
        # disabled seed: unchanged
        w0 = O.packed_dequantize(packed, one, zero, lin, seed=(0x1234, 0x9876, 0))
        assert np.array_equal(w0.astype(np.int64), codes.astype(np.int64))


def test_threshold_gives_the_stated_probability():
    rng = np.random.default_rng(2)
    inp, out, bits = 256, 64, 8
    codes = np.full((out, inp), 100, np.uint32)
    packed = codes.astype(np.uint8).reshape(-1)
    one, zero = np.ones(out, np.float32), np.zeros(out, np.float32)
    lin = _linear(inp, out, bits, inp, whole=0, threshold=1 << 30)  # P(step) = 2^30 / 2^32
    w = O.packed_dequantize(packed, one, zero, lin, seed=(77, 88, 1))
    moved = np.mean(w != 100)
    assert abs(moved - 0.25) < 0.02
