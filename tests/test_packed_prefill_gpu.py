"""The packed model's KDA attention block over whole sequences (the
reference's 16k prefill KdaMoeMetalExecutor::kda, forward_metal.rs:997-1129)
against the CPU restatement in oracle/decode.py: int4/int8 codes, integer-
code perturbation on and off, recurrent state carried between calls."""
import numpy as np
import pytest

import oracle as O
from oracle import decode as OD

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

from ennx_b200 import ops  # noqa: E402
from ennx_b200.native import ModelPackage, PackedKdaBlock  # noqa: E402

from _native_model import CONFIG, write_package  # noqa: E402

CFG = dict(CONFIG, gate_rank=64)  # the GEMM path takes ranks in multiples of 64
RTOL, ATOL = 2e-2, 1e-2


@pytest.fixture(scope="module")
def package(tmp_path_factory):
    d = tmp_path_factory.mktemp("prefill_pkg")
    write_package(str(d), seed=11, cfg=CFG)
    return ModelPackage(str(d))


def close(got, ref, what):
    err = np.abs(np.asarray(got, np.float64) - ref) - (ATOL + RTOL * np.abs(ref))
    assert err.max() <= 0, f"{what}: max excess {err.max():.3e}"


@pytest.mark.parametrize("layer,batch,seq,seed", [(0, 2, 100, None), (1, 1, 192, 0x1234_5678_9ABC), (0, 3, 64, 7)])
def test_packed_kda_block_matches_oracle(package, layer, batch, seq, seed):
    H, heads, r = CFG["hidden_size"], CFG["heads"], CFG["gate_rank"]
    blk = PackedKdaBlock(package.packed, package.scales, package.biases, package.linears(), layer, heads, r,
                         CFG["rms_epsilon"], CFG["residual_scale"])
    rng = np.random.default_rng(layer * 100 + seq)
    # Without the q/k L2 norm the delta rule is stable only while beta*|k|^2 < 2;
    # inputs at 0.15 of unit RMS keep this test package's keys there
    xn = O.round_bf16((0.15 * rng.standard_normal((batch * seq, H))).astype(np.float32))
    h0 = O.round_bf16(rng.standard_normal((batch * seq, H)).astype(np.float32))
    state0 = (rng.standard_normal((batch, heads, 128, 128)) * 0.05).astype(np.float32)
    hid = torch.from_numpy(h0).cuda().bfloat16()
    st = torch.from_numpy(state0).cuda()
    blk(torch.from_numpy(xn).cuda().bfloat16(), hid, batch, seq, state=st, seed=seed)
    ops.device_status()
    ref, ref_state = OD.kda_prefill_block(package.packed, package.scales, package.biases, package.linears(),
                                          layer, heads, r, CFG["rms_epsilon"], CFG["residual_scale"], xn, h0,
                                          batch, seq, seed=seed, state=state0)
    close(hid.float().cpu().numpy(), ref, "hidden")
    close(st.cpu().numpy(), ref_state, "state")


def test_packed_kda_block_state_carries_and_seed_matters(package):
    H, heads, r = CFG["hidden_size"], CFG["heads"], CFG["gate_rank"]
    blk = PackedKdaBlock(package.packed, package.scales, package.biases, package.linears(), 0, heads, r,
                         CFG["rms_epsilon"], CFG["residual_scale"])
    rng = np.random.default_rng(3)
    xn = torch.from_numpy(O.round_bf16((0.15 * rng.standard_normal((128, H))).astype(np.float32))).cuda().bfloat16()
    # one call over 128 tokens == two calls over 64 with the state carried
    full = torch.zeros(128, H, device="cuda", dtype=torch.bfloat16)
    blk(xn, full, 1, 128, state=torch.zeros(1, heads, 128, 128, device="cuda"), seed=5)
    st = torch.zeros(1, heads, 128, 128, device="cuda")
    halves = [torch.zeros(64, H, device="cuda", dtype=torch.bfloat16) for _ in range(2)]
    blk(xn[:64].contiguous(), halves[0], 1, 64, state=st, seed=5)
    blk(xn[64:].contiguous(), halves[1], 1, 64, state=st, seed=5)
    a, b = full.float().cpu().numpy(), torch.cat(halves).float().cpu().numpy()
    assert np.all(np.abs(a - b) <= ATOL + RTOL * np.abs(b))
    other = torch.zeros(128, H, device="cuda", dtype=torch.bfloat16)
    blk(xn, other, 1, 128, state=torch.zeros(1, heads, 128, 128, device="cuda"), seed=6)
    assert not torch.equal(other, full)  # the integer-code perturbation follows the seed
    with pytest.raises(Exception, match="multiples of 64"):
        PackedKdaBlock(package.packed, package.scales, package.biases, package.linears(), 0, heads, 16,
                       CFG["rms_epsilon"], 1.0)(xn, full, 1, 128)
