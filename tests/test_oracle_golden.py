"""The CPU oracle against the reference's own golden vectors and known answers.

Sources (Kvutza/ennx paths):
* rust/crates/ennx/src/dense.rs:470-505  -- signs, tensor key, changed pytree, dist2
* rust/crates/ennx/src/dense/bf16.rs:321-390 -- sub-ulp change, limits, overflow rollback
* rust/crates/ennx/src/dense/linear.rs:566-610 -- fused linear == materialised
* ops/bf16_parity.py:18-106, 393-418 -- executed by tests/golden/make_golden.py
* buck2/tests/metal.rs:371-414 -- KDA decode known answer
* cuda/src/main.rs:316-345 -- packed-code perturbation over 36 cases
"""
import json
import math
import os

import numpy as np
import pytest

import oracle as O

SIGNS = [1.0, 1.0, 1.0, -1.0, 1.0, 1.0, 1.0, -1.0, -1.0, 1.0, -1.0, 1.0, 1.0, 1.0, 1.0, -1.0]


def test_signs_match_reference_golden():
    got = [O.dense_sign(0x123456789ABCDEF0, 11, e) for e in range(16)]
    assert got == SIGNS


def test_tensor_key_golden():
    assert O.tensor_key("blk.27.attn_q.weight") == 3843877851495245630


def test_dense_apply_changes_every_value():
    base = np.array([0.5, -1.0, 2.0, 0.25, 4.0, -2.0, 0.75, -0.125], np.float32)
    leaves = [(11, 0, 4, 0.5), (29, 4, 4, 1.25)]
    st, out, changed = O.dense_apply_f32(base, leaves, [(0x123456789ABCDEF0, 0.01)])
    assert st == 0 and changed == 8 and np.all(out != base)


def test_dist2_golden():
    st, d = O.dense_dist2([(11, 0, 4, 0.5), (29, 4, 4, 1.25)], [(7, 0.5)], [(7, -0.5)])
    assert st == 0 and d == 7.25


def test_golden_fixture_from_reference_python(golden_dir):
    data = json.load(open(os.path.join(golden_dir, "bf16_parity.json")))
    assert data["signs_seed_0x123456789abcdef0_key_11"][:16] == SIGNS
    for e, s in enumerate(data["signs_seed_0x123456789abcdef0_key_11"]):
        assert O.dense_sign(0x123456789ABCDEF0, 11, e) == s
    for x, y in zip(data["mix64"]["inputs"], data["mix64"]["outputs"]):
        assert O.mix64(x) == y
    for case in data["cases"]:
        st, out = O.dense_apply_bf16(np.array(case["base"], np.uint16), case["leaves"], case["terms"])
        assert st == 0, case["name"]
        assert out.tolist() == case["expected"], case["name"]


def test_bf16_sub_ulp_changes_every_weight():
    base = O.to_bf16_bits(np.array([1.0, -2.0, 4.0, -8.0], np.float32))
    st, out = O.dense_apply_bf16(base, [(11, 0, 4, 1e-6)], [(17, 1e-6)])
    assert st == 0 and np.all(out != base)


def test_bf16_next_stays_finite_at_limits():
    assert math.isfinite(float(O.from_bf16_bits(np.array([O.bf16_next(0x7F7F, True)]))[0]))
    assert math.isfinite(float(O.from_bf16_bits(np.array([O.bf16_next(0xFF7F, False)]))[0]))


def test_bf16_overflow_rolls_back():
    base = O.to_bf16_bits(np.array([1.0], np.float32))
    fmax = float(np.finfo(np.float32).max)
    st, out = O.dense_apply_bf16(base, [(7, 0, 1, fmax)], [(11, fmax)])
    assert st == 2 and out.tolist() == base.tolist()


def test_fused_linear_matches_materialised():
    x = np.array([0.25, -0.5, 1.5, 2.0], np.float32)
    w = np.array([0.5, -1.0, 0.75, 0.25, -0.5, 2.0, 1.25, -0.75], np.float32)
    b = np.array([0.125, -0.25], np.float32)
    terms = [(0x123456789ABCDEF0, 0.5), (91, -0.125)]
    st, y = O.dense_linear_f32(x, w, b, (11, 0, 0.02), (29, 0, 0.01), terms)
    assert st == 0
    # materialise through dense_apply with one leaf per tensor (element = index)
    _, mw, _ = O.dense_apply_f32(w, [(11, 0, 8, 0.02)], terms)
    _, mb, _ = O.dense_apply_f32(b, [(29, 0, 2, 0.01)], terms)
    for r in range(2):
        acc = np.float32(mb[r])
        for c in range(4):
            acc = np.float32(math.fma(float(x[c]), float(mw[r * 4 + c]), float(acc))) if hasattr(math, "fma") else np.float32(acc + x[c] * mw[r * 4 + c])
        assert abs(float(y[r]) - float(acc)) <= 2 * np.finfo(np.float32).eps * max(1.0, abs(float(acc)))


def test_kda_decode_known_answer():
    # q = k = e0, v = 2, beta = 0.5, g = 0, dk = dv = 4: state 1.0 then 1.5,
    # outputs 0.5 then 0.75 after the 1/sqrt(dk) scale.
    q = np.zeros((1, 2, 1, 4), np.float32); q[..., 0] = 1.0
    v = np.full((1, 2, 1, 4), 2.0, np.float32)
    g = np.zeros((1, 2, 1, 4), np.float32)
    beta = np.full((1, 2, 1), 0.5, np.float32)
    out, st = O.kda_recurrence(q, q, v, g, beta)
    assert out[0, 0, 0].tolist() == [0.5] * 4
    assert out[0, 1, 0].tolist() == [0.75] * 4
    assert st[0, 0, 0].tolist() == [1.5] * 4 and np.all(st[0, 0, 1:] == 0)


def _cpu_hash(seed, element):
    v = ((seed & 0xFFFFFFFF) ^ ((element * 0x9E3779B9) & 0xFFFFFFFF)) & 0xFFFFFFFF
    v ^= v >> 16
    v = (v * 0x7FEB352D) & 0xFFFFFFFF
    v ^= (seed >> 32) & 0xFFFFFFFF
    v = (v * 0x846CA68B) & 0xFFFFFFFF
    return v ^ (v >> 15)


@pytest.mark.parametrize("seed", [0, 1, 0x0123456789ABCDEF, 2**64 - 1])
def test_trial_hash_matches_host_restatement(seed):
    # cuda/src/main.rs:649-656 is the host copy of the device hash.
    for e in [0, 1, 255, 256, 257, 65535, 2**31, 2**32 - 1]:
        assert O.trial_hash(seed & 0xFFFFFFFF, seed >> 32, e) == _cpu_hash(seed, e)


def test_perturb_code_stays_in_range():
    for bits in (4, 8):
        mx = (1 << bits) - 1
        for code in range(0, mx + 1, 3):
            for whole in (0, 1, 2):
                for thr in (0, 2**31, 2**32 - 1):
                    c = O.perturb_code(code, 5, 9, code * 7 + whole, bits, whole, thr)
                    assert 0 <= c <= mx


def test_philox_known_answer():
    # Random123 known-answer vectors for philox4x32-10 (Salmon et al., SC'11 kat_vectors).
    assert O.philox4x32_10([0, 0, 0, 0], [0, 0]).tolist() == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    assert O.philox4x32_10([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2).tolist() == [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]
    assert O.philox4x32_10([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344], [0xA4093822, 0x299F31D0]).tolist() == [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]


def test_noise_is_standard_normal():
    z = O.noise(1234, 3, 7, 200000)
    assert abs(z.mean()) < 0.01 and abs(z.std() - 1.0) < 0.01
    assert np.all(np.isfinite(z))
