"""Packed int4/int8 weights on the GPU against the oracle restatement of the
Metal path (kda_moe.metal:63-96, 351-420): dequantisation bit-exact (f32) /
RNE-exact (bf16), and the packed projection within the bf16 tolerance."""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

from ennx_b200 import _abi, ops  # noqa: E402


def _arena(rng, inp, out, bits, group, pad=(16, 32, 48)):
    """Packed codes and scale/bias arenas with nonzero offsets."""
    codes = rng.integers(0, 1 << bits, size=(out, inp), dtype=np.uint32)
    if bits == 8:
        packed = codes.astype(np.uint8)
    else:
        packed = np.zeros((out, (inp + 1) // 2), np.uint8)
        for c in range(inp):
            packed[:, c // 2] |= (codes[:, c] << (4 * (c & 1))).astype(np.uint8)
    groups = (inp + group - 1) // group
    w = np.concatenate([rng.integers(0, 255, pad[0], dtype=np.uint8), packed.reshape(-1)])
    sc = np.concatenate([rng.standard_normal(pad[1]), rng.uniform(0.001, 0.01, out * groups)]).astype(np.float32)
    bi = np.concatenate([rng.standard_normal(pad[2]), rng.uniform(-0.05, 0.05, out * groups)]).astype(np.float32)
    return w, sc, bi, pad


def _desc(cls, inp, out, bits, group, pad, whole, threshold, element_offset):
    return cls(byte_offset=pad[0], scale_offset=pad[1], bias_offset=pad[2], input_width=inp, output_width=out,
               bits=bits, group_size=group, element_offset=element_offset, perturb_whole=whole,
               perturb_threshold=threshold)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("inp,out,group,element_offset", [(256, 64, 64, 0), (200, 16, 48, 0), (37, 9, 8, 0),
                                                         (128, 8, 32, 2**32 - 300)])
@pytest.mark.parametrize("enabled", [0, 1])
def test_packed_dequantize_matches_oracle(bits, inp, out, group, element_offset, enabled):
    rng = np.random.default_rng(inp * 31 + bits)
    w, sc, bi, pad = _arena(rng, inp, out, bits, group)
    seed = (0x9E37 + inp, 0x51ED27 + bits, enabled)
    ref = O.packed_dequantize(w, sc, bi, _desc(O.PackedLinear, inp, out, bits, group, pad, 1, 1 << 31,
                                               element_offset), seed)
    dl = _desc(_abi.PackedLinear, inp, out, bits, group, pad, 1, 1 << 31, element_offset)
    tw, tsc, tbi = (torch.from_numpy(a).cuda() for a in (w, sc, bi))
    got32 = ops.packed_dequantize(tw, tsc, tbi, dl, seed, dtype=torch.float32).cpu().numpy()
    assert np.array_equal(got32.view(np.uint32), ref.view(np.uint32))
    got16 = ops.packed_dequantize(tw, tsc, tbi, dl, seed).view(torch.int16).cpu().numpy().view(np.uint16)
    assert np.array_equal(got16, O.to_bf16_bits(ref))


@pytest.mark.parametrize("bits", [4, 8])
def test_packed_linear_matches_oracle(bits):
    rng = np.random.default_rng(5 + bits)
    inp, out, tokens, group = 512, 384, 300, 64
    w, sc, bi, pad = _arena(rng, inp, out, bits, group)
    seed = (123, 456, 1)
    ref_w = O.packed_dequantize(w, sc, bi, _desc(O.PackedLinear, inp, out, bits, group, pad, 0, 1 << 30, 7), seed)
    x = O.round_bf16(rng.standard_normal((tokens, inp)).astype(np.float32))
    ref = O.gemm(x, O.round_bf16(ref_w))
    dl = _desc(_abi.PackedLinear, inp, out, bits, group, pad, 0, 1 << 30, 7)
    tw, tsc, tbi = (torch.from_numpy(a).cuda() for a in (w, sc, bi))
    y = ops.packed_linear(torch.from_numpy(x).cuda().to(torch.bfloat16), tw, tsc, tbi, dl, seed).float().cpu().numpy()
    err = np.abs(y - ref) - (1e-2 + 2e-2 * np.abs(ref))
    assert err.max() <= 0, err.max()


def test_packed_rejects_bad_descriptors():
    w = torch.zeros(64, dtype=torch.uint8, device="cuda")
    s = torch.ones(8, device="cuda")
    bad = _abi.PackedLinear(input_width=8, output_width=1, bits=3, group_size=8)
    with pytest.raises(_abi.EnnxB200Error, match="bits must be 4 or 8"):
        ops.packed_dequantize(w, s, s, bad)
    bad = _abi.PackedLinear(input_width=0, output_width=1, bits=4, group_size=8)
    with pytest.raises(_abi.EnnxB200Error, match="dimensions must be positive"):
        ops.packed_dequantize(w, s, s, bad)
