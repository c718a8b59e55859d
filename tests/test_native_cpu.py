"""ModelPackage (the reference's packed model format) and the decoder oracle,
on CPU: the reference's own package test (rust/crates/ennx/src/
forward_weights.rs:207-241), its validation errors, and the KDA decode-step
known answer (buck2/tests/metal.rs:371-414)."""
import os

import numpy as np
import pytest

import oracle.decode as D
from ennx_b200.native import ModelPackage, NativeKdaModel
from tests._native_model import CONFIG, write_package


def _write(directory, toml, weights=(1, 2, 3, 4), scales=(2.0, 3.0), biases=(0.0, 1.0)):
    os.makedirs(directory, exist_ok=True)
    with open(os.path.join(directory, "model.toml"), "w") as f:
        f.write(toml)
    np.array(weights, np.uint8).tofile(os.path.join(directory, "weights.bin"))
    np.array(scales, "<f4").tofile(os.path.join(directory, "scales.bin"))
    np.array(biases, "<f4").tofile(os.path.join(directory, "biases.bin"))


HEAD = "weights = 'weights.bin'\nscales = 'scales.bin'\nbiases = 'biases.bin'\n\n"
DECAY = ("[[linear]]\nname = 'layer.decay'\nbyte_offset = 0\nscale_offset = 0\nbias_offset = 0\ninput_width = 4\n"
         "output_width = 1\nbits = 8\ngroup_size = 2\n")


def test_reference_package_known_answer(tmp_path):
    """opens_native_quantized_package_without_python (forward_weights.rs:207-241)."""
    _write(tmp_path, HEAD + DECAY)
    model = ModelPackage(str(tmp_path))
    assert model.vector("layer.decay") == [2.0, 4.0, 10.0, 13.0]
    leaves = model.trial_leaves(1.0, 1.0, 1.0)
    assert len(leaves) == 1 and leaves[0][1] == 4
    assert model.linear("layer.decay") == (0, 0, 0, 4, 1, 8, 2, 0, 0, 0)
    assert (model.weight_bytes, model.scale_count, model.bias_count) == (4, 2, 2)


def test_package_validation_errors(tmp_path):
    with pytest.raises(ValueError, match="cannot read .*model.toml"):
        ModelPackage(str(tmp_path / "missing"))
    _write(tmp_path / "a", HEAD + DECAY.replace("bits = 8", "bits = 3"))
    with pytest.raises(ValueError, match="packed KDA linear bits must be 4 or 8, got 3"):
        ModelPackage(str(tmp_path / "a"))
    _write(tmp_path / "b", HEAD + DECAY.replace("input_width = 4", "input_width = 8"))
    with pytest.raises(ValueError, match="linear 'layer.decay' exceeds weights arena"):
        ModelPackage(str(tmp_path / "b"))
    _write(tmp_path / "c", HEAD + DECAY.replace("group_size = 2", "group_size = 1"))
    with pytest.raises(ValueError, match="linear 'layer.decay' exceeds scale or bias arena"):
        ModelPackage(str(tmp_path / "c"))
    _write(tmp_path / "d", HEAD + DECAY + DECAY)
    with pytest.raises(ValueError, match="duplicate linear name 'layer.decay'"):
        ModelPackage(str(tmp_path / "d"))
    _write(tmp_path / "e", HEAD + DECAY.replace("input_width = 4", "input_width = 0"))
    with pytest.raises(ValueError, match="packed KDA linear dimensions must be positive"):
        ModelPackage(str(tmp_path / "e"))
    _write(tmp_path / "f", HEAD + DECAY)
    with open(tmp_path / "f" / "scales.bin", "ab") as f:
        f.write(b"\x00")
    with pytest.raises(ValueError, match="is not a whole f32 arena"):
        ModelPackage(str(tmp_path / "f"))
    _write(tmp_path / "g", HEAD + DECAY)
    m = ModelPackage(str(tmp_path / "g"))
    with pytest.raises(ValueError, match="model package has no linear 'nope'"):
        m.linear("nope")
    _write(tmp_path / "h", HEAD + DECAY.replace("output_width = 1", "output_width = 1\nelement_offset = 3"))
    with pytest.raises(ValueError, match="linear element offset 3 does not continue parameter offset 0"):
        ModelPackage(str(tmp_path / "h")).trial_leaves()


def test_synthetic_package_parses_and_tiles_its_parameters(tmp_path):
    cfg = write_package(tmp_path)
    pkg = ModelPackage(str(tmp_path))
    leaves = pkg.trial_leaves()
    assert sum(l[1] for l in leaves) == sum(
        pkg.linear(n[0])[3] * pkg.linear(n[0])[4] for n in pkg.linears())
    assert pkg.linear("embedding")[4] == 384 and cfg["num_layers"] == 2


def test_oracle_decode_step_known_answer():
    """q = k = e0, v = 2, beta = 0.5, g = 0, d_k = d_v = 4: the state of key
    row 0 goes 0 -> 1.0 -> 1.5 and the outputs 0.5 -> 0.75 (1/sqrt(d_k))."""
    state = np.zeros((4, 4))
    e0 = np.array([1.0, 0, 0, 0])
    out = D.decode_step(state, e0, e0, np.full(4, 2.0), np.zeros(4), 0.5)
    assert state[0].tolist() == [1.0] * 4 and np.all(state[1:] == 0) and out.tolist() == [0.5] * 4
    out = D.decode_step(state, e0, e0, np.full(4, 2.0), np.zeros(4), 0.5)
    assert state[0].tolist() == [1.5] * 4 and out.tolist() == [0.75] * 4


def test_oracle_argmax_rule():
    logits = np.zeros(600)
    logits[[1, 256]] = 5.0  # lane 0 holds 256, lane 1 holds 1: lane 0 wins the tree
    assert D.argmax_lanes(logits) == 256
    logits[1] = 5.5
    assert D.argmax_lanes(logits) == 1


def test_oracle_decoder_runs_on_the_synthetic_package(tmp_path):
    write_package(tmp_path)
    pkg = ModelPackage(str(tmp_path))
    o = D.DecoderOracle(pkg.packed, pkg.scales, pkg.biases, pkg.linears(), **CONFIG)
    out = o.generate([3, 17], 3, seed=5)
    assert out[:2] == [3, 17] and len(out) == 5 and all(0 <= t < 384 for t in out)
    assert np.isfinite(o.logits).all() and o.logits.std() > 0


def test_native_model_argument_errors(tmp_path):
    write_package(tmp_path)
    pkg = ModelPackage(str(tmp_path))
    with pytest.raises(ValueError, match="'metal' decoding is not available in this build"):
        NativeKdaModel(pkg.packed, pkg.scales, pkg.biases, pkg.linears(), **CONFIG, device="metal")
    with pytest.raises(ValueError, match="native model has no linear 'layers.0.attention.qkv'"):
        NativeKdaModel(pkg.packed, pkg.scales, pkg.biases,
                       [l for l in pkg.linears() if l[0] != "layers.0.attention.qkv"], **CONFIG)
    with pytest.raises(ValueError, match="packed model arena must be contiguous"):
        NativeKdaModel(pkg.packed[::2], pkg.scales, pkg.biases, pkg.linears(), **CONFIG)
