"""Host-side behaviour of ``ennx_b200.experimental`` (the ``ennx.experimental``
dense subset): argument validation with the reference's error text, the
known answers of rust/crates/ennx/src/dense.rs:480-505, ``dense_dist2``
against the C oracle, and the DLPack lease.  No GPU is used."""
import gc

import numpy as np
import pytest

import oracle as O
from ennx_b200 import _abi, _dlpack
from ennx_b200 import experimental as X

torch = pytest.importorskip("torch")

LEAVES = [(11, 0, 4, 0.5), (29, 4, 4, 1.25)]  # dense.rs:463-468


def test_tensor_key_known_answer():
    assert X.tensor_key("blk.27.attn_q.weight") == 3843877851495245630  # dense.rs:480-486
    assert X.tensor_key("w") == O.tensor_key("w")


def test_dist2_known_answer():
    # dense.rs:498-505: energy 4*0.25 + 4*1.5625 = 7.25, coefficient distance 1
    assert X.dense_dist2(LEAVES, [(7, 0.5)], [(7, -0.5)]) == 7.25


@pytest.mark.parametrize("case", range(6))
def test_dist2_matches_oracle(case):
    rng = np.random.default_rng(case)
    nl = int(rng.integers(1, 5))
    lens = rng.integers(1, 1000, nl)
    offs = np.concatenate([[0], np.cumsum(lens)[:-1]])
    leaves = [(int(rng.integers(0, 2**63)), int(o), int(n), float(rng.uniform(1e-4, 2)))
              for o, n in zip(offs, lens)]
    seeds = [3, 5, 3, 9, 2**64 - 1]
    left = [(int(rng.choice(seeds)), float(rng.normal())) for _ in range(int(rng.integers(0, 5)))]
    right = [(int(rng.choice(seeds)), float(rng.normal())) for _ in range(int(rng.integers(0, 5)))]
    st, expect = O.dense_dist2(leaves, left, right)
    assert st == 0
    assert X.dense_dist2(leaves, left, right) == expect


def test_dist2_rejects_bad_layout_and_terms():
    with pytest.raises(ValueError, match="at least one dense leaf is required"):
        X.dense_dist2([], [(1, 1.0)], [])
    with pytest.raises(ValueError, match="does not continue parameter offset 4"):
        X.dense_dist2([(1, 0, 4, 1.0), (2, 5, 4, 1.0)], [(1, 1.0)], [])
    with pytest.raises(ValueError, match="dense coefficient must be finite"):
        X.dense_dist2(LEAVES, [(1, float("nan"))], [])
    with pytest.raises(ValueError, match="dense leaf length must be positive"):
        X.dense_dist2([(1, 0, 0, 1.0)], [], [])
    with pytest.raises(ValueError, match="dense leaf scale must be finite and positive"):
        X.dense_dist2([(1, 0, 3, -1.0)], [], [])


def test_param_block_validation_and_fields():
    b = X.ParamBlock(5, 10, 20, 0.25)
    assert (b.key, b.offset, b.length, b.scale, b.weight) == (5, 10, 20, 0.25, 1.0)
    with pytest.raises(AttributeError):
        b.scale = 2.0
    with pytest.raises(ValueError, match="BF16 block length must be positive"):
        X.ParamBlock(1, 0, 0, 1.0)
    for scale, weight in ((0.0, 1.0), (float("inf"), 1.0), (1.0, -1.0), (1.0, float("nan"))):
        with pytest.raises(ValueError, match="BF16 block scale and weight must be positive"):
            X.ParamBlock(1, 0, 4, scale, weight)


def test_device_names():
    base = np.ones(4, np.float32)
    for name, label in (("cpu", "CPU"), ("Metal", "Metal"), ("ocl", "OpenCL"), ("agx", "AGX")):
        with pytest.raises(ValueError, match=f"{label} dense directions are not available in this build"):
            X.dense_apply(base, [(1, 0, 4, 1.0)], [(3, 1.0)], device=name)
        with pytest.raises(ValueError, match=f"{label} dense linear is not available in this build"):
            X.DenseLinear(np.ones((2, 2), np.float32), (1, 0, 1.0), device=name)
    with pytest.raises(ValueError, match="unknown compute device 'tpu'"):
        X.dense_apply(base, [(1, 0, 4, 1.0)], [(3, 1.0)], device="tpu")


def test_dense_apply_validation():
    with pytest.raises(ValueError, match="dense base cannot be empty"):
        X.dense_apply(np.zeros(0, np.float32), [(1, 0, 1, 1.0)], [(3, 1.0)])
    with pytest.raises(ValueError, match="dense base values must be finite"):
        X.dense_apply(np.array([1.0, np.inf], np.float32), [(1, 0, 2, 1.0)], [(3, 1.0)])
    with pytest.raises(ValueError, match="dense coefficient must be finite"):
        X.dense_apply(np.ones(2, np.float32), [(1, 0, 2, 1.0)], [(3, float("inf"))])


def test_dense_linear_validation():
    w = np.ones((3, 4), np.float32)
    x = np.ones(4, np.float32)
    t = [(7, 1.0)]
    with pytest.raises(ValueError, match="dense view scale must be finite and positive"):
        X.dense_linear(x, w, (1, 0, 0.0), t)
    with pytest.raises(ValueError, match="dense linear weight must contain complete non-empty rows"):
        X.dense_linear(x, np.ones((3, 0), np.float32), (1, 0, 1.0), t)
    with pytest.raises(ValueError, match="bias length must equal the weight row count"):
        X.dense_linear(x, w, (1, 0, 1.0), t, bias=np.ones(2, np.float32), bias_view=(2, 0, 1.0))
    with pytest.raises(ValueError, match="bias and bias view must be supplied together"):
        X.dense_linear(x, w, (1, 0, 1.0), t, bias=np.ones(3, np.float32))
    with pytest.raises(ValueError, match="dense linear weights must be finite"):
        X.dense_linear(x, np.full((3, 4), np.nan, np.float32), (1, 0, 1.0), t)
    with pytest.raises(ValueError, match="dense linear weight coordinates overflow u64"):
        X.dense_linear(x, w, (1, 2**64 - 5, 1.0), t)
    with pytest.raises(ValueError, match="dense linear input must contain 4 finite values"):
        X.dense_linear(np.ones(3, np.float32), w, (1, 0, 1.0), t)
    with pytest.raises(ValueError, match="dense linear requires finite perturbation terms"):
        X.dense_linear(x, w, (1, 0, 1.0), [])
    with pytest.raises(ValueError, match="dense linear terms cancel to zero"):
        X.dense_linear(x, w, (1, 0, 1.0), [(7, 0.5), (7, -0.5)])


def test_no_cpu_path_without_a_device():
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is visible")
    with pytest.raises(_abi.EnnxB200Error, match="needs a CUDA device"):
        X.dense_apply(np.ones(4, np.float32), [(1, 0, 4, 1.0)], [(3, 1.0)])
    with pytest.raises(_abi.EnnxB200Error, match="needs a CUDA device"):
        X.ParamBuffer(torch.zeros(4, dtype=torch.bfloat16), [X.ParamBlock(1, 0, 4, 1.0)])


@pytest.mark.parametrize("max_version", [None, (1, 0), (1, 7), (2, 0)])
def test_dlpack_lease_is_released_by_the_consumer(max_version):
    """The export helper on a host buffer (device kDLCPU) so torch can consume
    it here: the lease holds until the consumer drops the tensor, and an
    unconsumed capsule releases it when collected."""
    buf = np.arange(12, dtype=np.float32)
    released = []

    class Producer:
        def __dlpack_device__(self):
            return (_dlpack.KDL_CPU, 0)

        def __dlpack__(self, stream=None, max_version=None, dl_device=None, copy=None):
            return _dlpack.export(buf, buf.ctypes.data, (3, 4), _dlpack.KDL_FLOAT, 32, (_dlpack.KDL_CPU, 0),
                                  lambda: released.append(1), max_version=mv)

    mv = max_version
    before = _dlpack.live_exports()
    t = torch.from_dlpack(Producer())
    assert t.shape == (3, 4) and t[2, 3].item() == 11.0 and t.data_ptr() == buf.ctypes.data
    assert _dlpack.live_exports() == before + 1 and released == []
    del t
    gc.collect()
    assert _dlpack.live_exports() == before and released == [1]
    cap = Producer().__dlpack__()
    assert _dlpack.live_exports() == before + 1
    del cap
    gc.collect()
    assert _dlpack.live_exports() == before and released == [1, 1]


def test_param_buffer_host_rules_without_a_device():
    """The lease and DLPack argument rules of py_weights.rs:61-103, which run
    before any device work."""
    pb = object.__new__(X.ParamBuffer)
    pb._exported = True
    with pytest.raises(ValueError, match="cannot materialize while a JAX candidate is alive"):
        pb.materialize([(1, 1.0)])
    pb._exported = False
    with pytest.raises(ValueError, match="BF16 pytree terms cancel to zero"):
        pb.materialize([(1, 1.0), (1, -1.0)])
    with pytest.raises(ValueError, match="dense coefficient must be finite"):
        pb.materialize([(1, float("inf"))])
    with pytest.raises(BufferError, match="does not export copies"):
        pb.__dlpack__(copy=True)
    pb._device = torch.device("cuda", 0)
    with pytest.raises(BufferError, match="cannot export to another device"):
        pb.__dlpack__(dl_device=(1, 0))
    with pytest.raises(ValueError, match="invalid DLPack CUDA stream"):
        pb.__dlpack__(stream=0)
    pb._exported = True
    with pytest.raises(ValueError, match="already exported"):
        pb.__dlpack__(stream=1)
