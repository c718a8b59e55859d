"""NativeKdaModel (packed-weight single-token decoder) on the GPU against the
decoder oracle (oracle/decode.py), on a synthetic package in the reference's
format.  The oracle computes in float64 and the device in fp32, so logits are
compared with a tolerance and greedy tokens exactly, except where the oracle's
two best logits are closer than that tolerance."""
import numpy as np
import pytest

import oracle.decode as D

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

from ennx_b200.native import ModelPackage, NativeKdaModel  # noqa: E402
from tests._native_model import CONFIG, write_package  # noqa: E402

TOL = 2e-3


def _pair(tmp_path):
    write_package(tmp_path)
    pkg = ModelPackage(str(tmp_path))
    model = NativeKdaModel(pkg.packed, pkg.scales, pkg.biases, pkg.linears(), **CONFIG)
    oracle = D.DecoderOracle(pkg.packed, pkg.scales, pkg.biases, pkg.linears(), **CONFIG)
    return model, oracle


def _close(got, ref):
    scale = float(np.abs(ref).max())
    np.testing.assert_allclose(got, ref, rtol=0, atol=TOL * scale)


def _margin(logits):
    top = np.sort(logits)[-2:]
    return float(top[1] - top[0]) / float(np.abs(logits).max())


@pytest.mark.parametrize("seed", [0, 12345, 2**63 + 17])
def test_decode_tokens_match_oracle(tmp_path, seed):
    model, oracle = _pair(tmp_path)
    model.prepare_candidate(seed)
    oracle.prepare(seed)
    for token in [3, 17, 99, 250, 7, 383]:  # the same inputs on both sides
        got = model.decode_token(token, seed)
        ref = oracle.decode_token(token, seed)
        _close(model.logits(), oracle.logits)
        if got != ref:
            assert _margin(oracle.logits) < 2 * TOL, (token, got, ref)
    bits = model.logit_bits()
    assert len(bits) == 384 and np.array_equal(np.array(bits, np.uint16).view(np.float16),
                                               model.logits().astype(np.float16))


def test_generate_matches_oracle_and_replays(tmp_path):
    model, oracle = _pair(tmp_path)
    prompt = [11, 42, 5]
    out = model.generate(prompt, 12, seed=7)
    ref = oracle.generate(prompt, 12, seed=7)
    assert out[:3] == prompt and len(out) == 15
    # sequences agree until a near-tie of the oracle (then they may diverge)
    o2 = D.DecoderOracle(oracle.packed, oracle.scales, oracle.biases,
                         [(n,) + d for n, d in oracle.named.items()], **CONFIG)
    for i in range(len(prompt) - 1):
        o2.decode_token(prompt[i], 7)
    nxt = o2.decode_token(prompt[-1], 7)
    for i in range(12):
        if out[3 + i] != ref[3 + i]:
            assert _margin(o2.logits) < 2 * TOL, (i, out, ref)
            break
        if i + 1 < 12:
            nxt = o2.decode_token(nxt, 7)
    # the captured step replays identically after a reset
    model.reset()
    assert model.generate(prompt, 12, seed=7) == out
    # and matches the eager token-by-token path
    model.reset()
    seq = [model.decode_token(t, 7) for t in prompt][-1:]
    for _ in range(11):
        seq.append(model.decode_token(seq[-1], 7))
    assert prompt + seq == out


def test_decoder_errors(tmp_path):
    model, _ = _pair(tmp_path)
    with pytest.raises(ValueError, match="token 384 exceeds the model vocabulary"):
        model.decode_token(384)
    with pytest.raises(ValueError, match="generation prompt cannot be empty"):
        model.generate([], 3)
