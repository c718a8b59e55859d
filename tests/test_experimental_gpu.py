"""``ennx_b200.experimental`` on the GPU against the oracle and the golden
vectors: the calls a user of ``ennx.experimental`` makes (py_weights.rs:31-306,
py_bf16.rs:15-55), mirroring ops/bf16_parity.py:393-456 and
rust/crates/ennx/examples/cuda_dense.rs:12-111."""
import gc
import json
import os

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

from ennx_b200 import experimental as X  # noqa: E402


def _buffer(bits, leaves):
    base = torch.from_numpy(np.ascontiguousarray(bits, np.uint16).view(np.int16)).cuda().view(torch.bfloat16)
    return X.ParamBuffer(base, [X.ParamBlock(*leaf) for leaf in leaves])


def _bits(pb):
    t = torch.from_dlpack(pb)
    out = t.view(torch.int16).cpu().numpy().view(np.uint16).copy()
    del t
    gc.collect()
    return out


def test_param_buffer_golden_bit_exact(golden_dir):
    data = json.load(open(os.path.join(golden_dir, "bf16_parity.json")))
    for case in data["cases"]:
        pb = _buffer(np.array(case["base"], np.uint16), case["leaves"])
        assert len(pb) == pb.len == len(case["base"])
        pb.materialize(case["terms"])
        assert _bits(pb).tolist() == case["expected"], case["name"]


def test_param_buffer_lease_and_dlpack_rules():
    rng = np.random.default_rng(7)
    n = 4099
    base = O.to_bf16_bits(rng.standard_normal(n).astype(np.float32))
    leaves = [(3, 0, 4000, 1e-3), (4, 4000, 99, 0.5)]
    pb = _buffer(base, leaves)
    assert np.array_equal(_bits(pb), base)  # the candidate starts as the base
    pb.materialize([(17, 1.0)])
    _, expect = O.dense_apply_bf16(base, leaves, [(17, 1.0)])
    held = torch.from_dlpack(pb)
    assert held.dtype == torch.bfloat16 and held.is_cuda and held.numel() == n
    assert np.array_equal(held.view(torch.int16).cpu().numpy().view(np.uint16), expect)
    with pytest.raises(ValueError, match="cannot materialize while a JAX candidate is alive"):
        pb.materialize([(18, 1.0)])
    with pytest.raises(ValueError, match="already exported"):
        pb.__dlpack__(stream=1)
    del held
    gc.collect()
    with pytest.raises(BufferError, match="does not export copies"):
        pb.__dlpack__(copy=True)
    with pytest.raises(BufferError, match="cannot export to another device"):
        pb.__dlpack__(dl_device=(1, 0))
    for bad in (0, -2):
        with pytest.raises(ValueError, match="invalid DLPack CUDA stream"):
            pb.__dlpack__(stream=bad)
    pb.materialize([(18, -0.5), (19, 0.25)])
    _, expect = O.dense_apply_bf16(base, leaves, [(18, -0.5), (19, 0.25)])
    assert np.array_equal(_bits(pb), expect)
    with pytest.raises(ValueError, match="BF16 pytree terms cancel to zero"):
        pb.materialize([(5, 0.5), (5, -0.5)])


def test_param_buffer_owns_a_copy_and_rolls_back_on_overflow():
    src = torch.tensor([3.0e38, 1.0], dtype=torch.bfloat16, device="cuda")
    base_bits = src.view(torch.int16).cpu().numpy().view(np.uint16).copy()
    pb = X.ParamBuffer(src, [X.ParamBlock(31, 0, 2, 3.4028234663852886e38)])
    src.zero_()  # the buffer copied its base at construction
    with pytest.raises(ValueError, match="overflowed"):
        pb.materialize([(101, 3.4028234663852886e38)])
    assert np.array_equal(_bits(pb), base_bits)


def test_param_buffer_rejects_bad_inputs():
    with pytest.raises(ValueError, match="CUDA BF16 base values must be finite"):
        X.ParamBuffer(torch.tensor([1.0, float("inf")], dtype=torch.bfloat16, device="cuda"),
                      [X.ParamBlock(1, 0, 2, 1.0)])
    with pytest.raises(ValueError, match="dense leaves cover 3 parameters, expected 4"):
        X.ParamBuffer(torch.zeros(4, dtype=torch.bfloat16, device="cuda"), [X.ParamBlock(1, 0, 3, 1.0)])
    with pytest.raises(ValueError, match="must be BF16"):
        X.ParamBuffer(torch.zeros(4, device="cuda"), [X.ParamBlock(1, 0, 4, 1.0)])
    with pytest.raises(BufferError, match="contiguous"):
        X.ParamBuffer(torch.zeros(4, 2, dtype=torch.bfloat16, device="cuda").t(), [X.ParamBlock(1, 0, 8, 1.0)])


def test_dense_apply_matches_oracle_and_changes_everything():
    rng = np.random.default_rng(5)
    n = 70003 + 521
    base = rng.standard_normal(n).astype(np.float32)
    leaves = [(17, 0, 70003, 1e-3), (19, 70003, 521, 0.25)]
    terms = [(41, 0.25), (73, -0.125), (89, 0.03125)]
    values, changed = X.dense_apply(base, leaves, terms)
    _, expect, _ = O.dense_apply_f32(base, leaves, terms)
    assert changed == n and np.array_equal(values.view(np.uint32), expect.view(np.uint32))
    # dense.rs:488-496: every element of the pytree moves
    small = np.array([0.5, -1.0, 2.0, 0.25, 4.0, -2.0, 0.75, -0.125], np.float32)
    values, changed = X.dense_apply(small, [(11, 0, 4, 0.5), (29, 4, 4, 1.25)], [(0x123456789ABCDEF0, 0.01)],
                                    device="cuda")
    assert changed == 8 and (values != small).all()


@pytest.mark.parametrize("bias", [True, False])
def test_dense_linear_and_resident_layer_match_oracle(bias):
    rng = np.random.default_rng(11)
    rows, cols = 7, 513
    x = rng.standard_normal(cols).astype(np.float32)
    w = rng.standard_normal((rows, cols)).astype(np.float32)
    b = rng.standard_normal(rows).astype(np.float32)
    terms = [(0x123456789ABCDEF0, 0.5), (91, -0.125)]
    wv, bv = (11, 3, 0.02), (29, 0, 0.01)
    _, expect = O.dense_linear_f32(x, w.reshape(-1), b if bias else None, wv, bv, terms)
    kw = dict(bias=b, bias_view=bv) if bias else {}
    y = X.dense_linear(x, w, wv, terms, **kw)
    np.testing.assert_allclose(y, expect, rtol=2e-5, atol=2e-5)  # cuda_dense.rs:90-111
    layer = X.DenseLinear(w, wv, **kw)
    assert (layer.input_size, layer.output_size) == (cols, rows)
    for seed in (5, 6):
        t = [(seed, 1.0)]
        _, e = O.dense_linear_f32(x, w.reshape(-1), b if bias else None, wv, bv, t)
        np.testing.assert_allclose(layer.eval(x, t), e, rtol=2e-5, atol=2e-5)
    with pytest.raises(ValueError, match=f"dense linear input must contain {cols} finite values"):
        layer.eval(x[:-1], terms)


def test_dense_linear_known_case_matches_materialised_weights():
    # rust/crates/ennx/src/dense/linear.rs:570-610, within 2 * f32 epsilon
    x = np.array([0.25, -0.5, 1.5, 2.0], np.float32)
    w = np.array([[0.5, -1.0, 0.75, 0.25], [-0.5, 2.0, 1.25, -0.75]], np.float32)
    b = np.array([0.125, -0.25], np.float32)
    terms = [(0x123456789ABCDEF0, 0.5), (91, -0.125)]
    y = X.dense_linear(x, w, (11, 0, 0.02), terms, bias=b, bias_view=(29, 0, 0.01))
    _, expect = O.dense_linear_f32(x, w.reshape(-1), b, (11, 0, 0.02), (29, 0, 0.01), terms)
    assert np.abs(y - expect).max() <= 2 * np.finfo(np.float32).eps


def test_param_buffer_gaussian_direction_matches_oracle():
    """ParamBuffer with the population's Philox Gaussian direction: leaf j's
    elements are bf16(base +/- bf16(sigma * scale_j * eps(seed, pair, j, i)))."""
    import numpy as np
    import oracle as O
    from ennx_b200.experimental import ParamBlock, ParamBuffer
    rng = np.random.default_rng(4)
    n = 5000
    base = O.to_bf16_bits(rng.standard_normal(n).astype(np.float32) * 0.1)
    blocks = [ParamBlock(3, 0, 1203, 0.5), ParamBlock(9, 1203, 3797, 2.0)]  # second leaf not 16-byte aligned
    buf = ParamBuffer(torch.from_numpy(base.view(np.int16)).cuda().view(torch.bfloat16), blocks)
    for sign in (1, -1):
        buf.materialize_gaussian(0xFEED, 4, 1e-2, sign)
        got = torch.from_dlpack(buf).cpu().view(torch.int16).numpy().view(np.uint16)
        for j, b in enumerate(blocks):
            sl = slice(b.offset, b.offset + b.length)
            exp = O.perturb_bf16(base[sl], 0xFEED, 4, j, float(np.float32(1e-2) * np.float32(b.scale)), sign)
            d = np.abs(got[sl].astype(np.int32) - exp.astype(np.int32))
            assert d.max() <= 1 and (d > 0).mean() < 1e-2
        del got
    with pytest.raises(ValueError, match="antithetic sign"):
        buf.materialize_gaussian(1, 0, 1e-2, 0)
