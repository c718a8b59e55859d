"""Seeded dense perturbation on the GPU against the oracle and the golden
vectors produced from the reference's own Python restatement.

Mirrors ops/bf16_parity.py:393-456 (bit-exact BF16, overflow, finiteness) and
rust/crates/ennx/examples/cuda_dense.rs:12-111 (fp32 apply, fused linear)."""
import ctypes
import json
import os

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

from ennx_b200 import _abi  # noqa: E402
from tests._gpu import dev_u16, host_u16, leaves_arr, ptr, stream, terms_arr  # noqa: E402


def apply_bf16(base_bits, leaves, terms):
    base = dev_u16(base_bits)
    out = torch.empty_like(base)
    lv, tm = leaves_arr(leaves), terms_arr(terms)
    st = _abi.lib().ennx_b200_dense_apply_bf16(ptr(base), base.numel(), lv, len(leaves), tm, len(terms), ptr(out), stream())
    return st, host_u16(out)


def test_bf16_golden_bit_exact(golden_dir):
    data = json.load(open(os.path.join(golden_dir, "bf16_parity.json")))
    for case in data["cases"]:
        st, out = apply_bf16(np.array(case["base"], np.uint16), case["leaves"], case["terms"])
        assert st == 0, (case["name"], _abi.lib().ennx_b200_last_error())
        assert out.tolist() == case["expected"], case["name"]


def test_bf16_large_matches_oracle():
    rng = np.random.default_rng(3)
    n = 70003 + 521
    base = O.to_bf16_bits(rng.standard_normal(n).astype(np.float32))
    leaves = [(O.tensor_key("w"), 0, 70003, 2e-3), (O.tensor_key("b"), 70003, 521, 0.5)]
    terms = [(11, 0.75), (29, -0.25), (2**64 - 1, 0.125)]
    st, out = apply_bf16(base, leaves, terms)
    ost, expect = O.dense_apply_bf16(base, leaves, terms)
    assert st == 0 and ost == 0
    assert np.array_equal(out, expect)


def test_bf16_overflow_rolls_back():
    st, out = apply_bf16(np.array([0x7F7F], np.uint16), [(31, 0, 1, 3.4028234663852886e38)],
                         [(101, 3.4028234663852886e38)])
    assert st == _abi.OVERFLOW
    assert b"overflowed" in _abi.lib().ennx_b200_last_error()
    assert out.tolist() == [0x7F7F]


def test_check_bf16_finiteness():
    flag = ctypes.c_int32(7)
    t = dev_u16(np.array([0x3F80, 0x7F80], np.uint16))
    assert _abi.lib().ennx_b200_check_bf16(ptr(t), 2, ctypes.byref(flag), stream()) == 0
    assert flag.value == 0
    t = dev_u16(np.array([0x3F80, 0x7F7F], np.uint16))
    assert _abi.lib().ennx_b200_check_bf16(ptr(t), 2, ctypes.byref(flag), stream()) == 0
    assert flag.value == 1


def test_dense_apply_f32_bit_exact():
    rng = np.random.default_rng(5)
    n = 70003 + 521
    base = rng.standard_normal(n).astype(np.float32)
    leaves = [(17, 0, 70003, 1e-3), (19, 70003, 521, 0.25)]
    terms = [(41, 0.25), (73, -0.125), (89, 0.03125)]
    b = torch.from_numpy(base).cuda()
    out = torch.empty_like(b)
    changed = ctypes.c_size_t(0)
    st = _abi.lib().ennx_b200_dense_apply_f32(ptr(b), n, leaves_arr(leaves), 2, terms_arr(terms), 3, ptr(out),
                                               ctypes.byref(changed), stream())
    assert st == 0 and changed.value == n
    ost, expect, _ = O.dense_apply_f32(base, leaves, terms)
    assert ost == 0
    assert np.array_equal(out.cpu().numpy().view(np.uint32), expect.view(np.uint32))


def test_cancelling_terms_rejected():
    b = torch.zeros(4, device="cuda")
    st = _abi.lib().ennx_b200_dense_apply_f32(ptr(b), 4, leaves_arr([(1, 0, 4, 1.0)]), 1,
                                               terms_arr([(5, 0.5), (5, -0.5)]), 2, ptr(b), None, stream())
    assert st == _abi.INVALID_ARGUMENT and b"cancel" in _abi.lib().ennx_b200_last_error()


@pytest.mark.parametrize("bias", [True, False])
def test_dense_linear_matches_oracle(bias):
    rng = np.random.default_rng(11)
    rows, cols = 7, 513
    x = rng.standard_normal(cols).astype(np.float32)
    w = rng.standard_normal(rows * cols).astype(np.float32)
    b = rng.standard_normal(rows).astype(np.float32)
    terms = [(0x123456789ABCDEF0, 0.5), (91, -0.125)]
    wv, bv = (11, 3, 0.02), (29, 0, 0.01)
    ost, expect = O.dense_linear_f32(x, w, b if bias else None, wv, bv, terms)
    assert ost == 0
    tx, tw, tb = (torch.from_numpy(a).cuda() for a in (x, w, b))
    out = torch.empty(rows, device="cuda")
    st = _abi.lib().ennx_b200_dense_linear_f32(ptr(tx), cols, ptr(tw), rows, ptr(tb) if bias else None,
                                                _abi.DenseView(*wv), _abi.DenseView(*bv), terms_arr(terms), 2,
                                                ptr(out), stream())
    assert st == 0
    np.testing.assert_allclose(out.cpu().numpy(), expect, rtol=2e-5, atol=2e-5)


def test_perturb_bf16_matches_oracle():
    rng = np.random.default_rng(2)
    n = 1 << 16
    w = O.to_bf16_bits(rng.standard_normal(n).astype(np.float32) * 0.02)
    tw = dev_u16(w)
    plus, minus = torch.empty_like(tw), torch.empty_like(tw)
    st = _abi.lib().ennx_b200_perturb_bf16(ptr(tw), n, 0xDEADBEEF12345678, 5, 17, 1e-3, ptr(plus), ptr(minus), stream())
    assert st == 0
    ep = O.perturb_bf16(w, 0xDEADBEEF12345678, 5, 17, 1e-3, +1)
    em = O.perturb_bf16(w, 0xDEADBEEF12345678, 5, 17, 1e-3, -1)
    gp, gm = host_u16(plus), host_u16(minus)
    # Box-Muller uses logf/sqrtf/sincospif on the device and fp64 libm in the
    # oracle: values agree to a few fp32 ulp, so bf16 outputs may differ by one
    # ulp where the sum sits on a rounding boundary.
    for g, e in ((gp, ep), (gm, em)):
        diff = np.abs(g.astype(np.int32) - e.astype(np.int32))
        assert diff.max() <= 1 and (diff > 0).mean() < 1e-3
    # odd length tail
    st = _abi.lib().ennx_b200_perturb_bf16(ptr(tw), 13, 7, 0, 3, 0.5, ptr(plus), None, stream())
    assert st == 0
    e = O.perturb_bf16(w[:13], 7, 0, 3, 0.5, +1)
    assert np.abs(host_u16(plus)[:13].astype(np.int32) - e.astype(np.int32)).max() <= 1


def test_perturb_noise_is_finite_over_many_draws():
    # 2^26 normals: the top Philox words (which once gave u1 = 1 and a NaN
    # radius) occur several times in this range; every output must be finite.
    n = 1 << 26
    w = torch.zeros(n, dtype=torch.int16, device="cuda")
    plus, minus = torch.empty_like(w), torch.empty_like(w)
    st = _abi.lib().ennx_b200_perturb_bf16(ptr(w), n, 12345, 7, 3, 1.0, ptr(plus), ptr(minus), stream())
    assert st == 0
    for t in (plus, minus):
        bits = t.view(torch.int16)
        assert not bool(((bits & 0x7F80) == 0x7F80).any().item())


def test_noise_step_matches_oracle():
    """The noise operand of the perturbed GEMM, e = bf16(sigma*eps), alone."""
    n = (1 << 16) + 5
    e = torch.empty(n, dtype=torch.int16, device="cuda")
    st = _abi.lib().ennx_b200_perturb_bf16(None, n, 0xDEADBEEF12345678, 5, 17, 1e-3, ptr(e), None, stream())
    assert st == 0
    # the Python form (ops.perturb_bf16 with w None) is the same call
    from ennx_b200 import ops
    e2 = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    ops.perturb_bf16(None, 0xDEADBEEF12345678, 5, 17, 1e-3, plus=e2)
    assert torch.equal(e2.view(torch.int16), e)
    ref = O.from_bf16_bits(O.noise_step_bf16(n, 0xDEADBEEF12345678, 5, 17, 1e-3)).astype(np.float64)
    got = O.from_bf16_bits(host_u16(e)).astype(np.float64)
    # Box-Muller on the SFU vs fp64 libm: sigma*eps agrees to ~1e-6 of sigma,
    # then one bf16 rounding: at most one bf16 ulp (<= 2^-7 relative) apart,
    # plus an absolute term for values near zero
    assert np.all(np.abs(got - ref) <= 2.0 ** -7 * np.abs(ref) + 1e-3 * 1e-5)
    # W +/- e from the same call sequence equals the perturbation with W given
    rng = np.random.default_rng(3)
    w = O.to_bf16_bits(rng.standard_normal(n).astype(np.float32) * 0.02)
    tw = dev_u16(w)
    plus, minus = torch.empty_like(tw), torch.empty_like(tw)
    assert _abi.lib().ennx_b200_perturb_bf16(ptr(tw), n, 0xDEADBEEF12345678, 5, 17, 1e-3, ptr(plus), ptr(minus),
                                             stream()) == 0
    wf = O.from_bf16_bits(w).astype(np.float64)
    ef = O.from_bf16_bits(host_u16(e)).astype(np.float64)
    assert np.array_equal(host_u16(plus), O.to_bf16_bits((wf + ef).astype(np.float32)))
    assert np.array_equal(host_u16(minus), O.to_bf16_bits((wf - ef).astype(np.float32)))
