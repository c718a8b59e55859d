"""The zeroth-order update (the population's tell) and the closed
ask -> evaluate -> tell loops on the GPU, against the CPU oracle."""
import numpy as np
import pytest

import oracle as O
from oracle import forward as OF

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

from ennx_b200 import _abi, ops  # noqa: E402
from ennx_b200.model import (HybridConfig, PopulationEvaluator, ResidentForwardSearch, flat_layout,  # noqa: E402
                             flat_size, init_weights, weights_from_flat)
from ennx_b200.population import PopulationStep, ResidentEsState  # noqa: E402

from _gpu import dev_u16, host_u16, ptr, stream  # noqa: E402

SMALL = HybridConfig(layers=4, hidden=256, vocab=1152, attn_period=4, q_heads=2, kv_heads=1, kda_heads=2,
                     gate_rank=64, experts=8, top_k=2, expert_width=128)


@pytest.fixture(autouse=True)
def _clean():
    yield
    ops.device_status()


def _bits(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def update_close(got_bits, exp_bits, coef):
    """Device vs oracle update: the Philox normals agree to ~1e-6 (SFU vs
    libm), so each sum agrees to ~1e-6 * sum|c|; after one bf16 rounding the
    values are at most one ulp (2^-7 relative) plus that apart.  Values that
    the update moves near zero have no bit-level agreement, hence values."""
    g, e = O.from_bf16_bits(got_bits).astype(np.float64), O.from_bf16_bits(exp_bits).astype(np.float64)
    tol = 2.0 ** -7 * np.abs(e) + 1e-5 * float(np.abs(np.asarray(coef, np.float64)).sum())
    assert np.all(np.abs(g - e) <= tol), f"max excess {(np.abs(g - e) - tol).max():.3e}"
    assert (g != e).mean() < 1e-2


def test_es_update_matches_oracle():
    rng = np.random.default_rng(0)
    n = (1 << 18) + 3
    w = O.to_bf16_bits(rng.standard_normal(n).astype(np.float32) * 0.02)
    coef = (rng.standard_normal(16) * 1e-3).astype(np.float32)
    tw = dev_u16(w)
    tc = torch.from_numpy(coef).cuda()
    assert _abi.lib().ennx_b200_es_update_bf16(ptr(tw), n, 77, 21, ptr(tc), 3, 16, stream()) == 0
    ref = O.es_update(w, 77, 21, coef, 3)
    update_close(host_u16(tw), ref, coef)
    assert (host_u16(tw) != w).mean() > 0.5  # the update moved most weights


def test_es_coefficients_bit_exact():
    f = torch.rand(32, generator=torch.Generator().manual_seed(1)) + 7.0
    c = torch.empty(16, device="cuda")
    assert _abi.lib().ennx_b200_es_coefficients(ptr(f.cuda()), 16, 16, 1e-3, 0.05, ptr(c), stream()) == 0
    ref = O.es_coefficients(f.numpy(), 1e-3, 0.05)
    assert np.array_equal(c.cpu().numpy(), ref)
    assert _abi.lib().ennx_b200_es_coefficients(ptr(f.cuda()), 16, 16, 0.0, 0.05, ptr(c), stream()) == \
        _abi.INVALID_ARGUMENT


def test_population_update_matches_oracle():
    cfg = SMALL
    w = init_weights(cfg, seed=4, std=0.05)
    before = {"embedding": _bits(w["embedding"]), "final_norm": _bits(w["final_norm"]),
              "layers": [{k: _bits(v) for k, v in L.items()} for L in w["layers"]]}
    ev = PopulationEvaluator(cfg, w, 1, 32)
    coef = torch.tensor([2e-3, -1e-3, 5e-4], device="cuda")
    ev.update(99, coef)
    torch.cuda.synchronize()
    ref = OF.population_update(cfg, before, 99, coef.cpu().numpy())
    pairs = [(w["embedding"], ref["embedding"]), (w["final_norm"], ref["final_norm"])]
    for L, R in zip(w["layers"], ref["layers"]):
        pairs += [(L[k], R[k]) for k in R]
    for got, exp in pairs:
        update_close(_bits(got).reshape(-1), exp.reshape(-1), coef.cpu().numpy())


def test_resident_es_state_closed_loop():
    """ask -> evaluate -> tell on one GPU: the fitness of a round is the
    forward of the weights the previous tells produced, and the update is the
    oracle's update of that round's fitness."""
    cfg = SMALL
    w = init_weights(cfg, seed=5, std=0.05)
    B, S = 2, 64
    tok = torch.randint(0, cfg.vocab, (B, S + 1), generator=torch.Generator().manual_seed(6), dtype=torch.int32)
    ev = PopulationEvaluator(cfg, w, B, S)
    step = PopulationStep(ev, num_pairs=3, sigma=1e-2, lr=0.05, coefficients=ev.coefficients, update=ev.update)
    state = ResidentEsState(step, seed=40)
    snap = {"embedding": _bits(w["embedding"]), "final_norm": _bits(w["final_norm"]),
            "layers": [{k: _bits(v) for k, v in L.items()} for L in w["layers"]]}
    r0, f0 = state.ask_evaluate(tok.cuda())
    assert r0.seed == 40 and state.seed == 41 and state.rounds == 1
    ref_fit = OF.population_forward(cfg, snap, tok.numpy(), 40, 1e-2, 0, 3)
    np.testing.assert_allclose(f0.cpu().numpy(), ref_fit, rtol=2e-3, atol=2e-3)
    coef = O.es_coefficients(f0.cpu().numpy(), 1e-2, 0.05)
    ref_w = OF.population_update(cfg, snap, 40, coef)
    update_close(_bits(w["layers"][1]["w_gate_up"]).reshape(-1), ref_w["layers"][1]["w_gate_up"].reshape(-1), coef)
    r1 = state.ask()
    with pytest.raises(ValueError, match="tell must finish"):
        state.ask()
    with pytest.raises(ValueError, match="does not match"):
        state.tell(type(r1)(r1.seed + 1, r1.step), f0)
    f1 = ev(tok.cuda(), r1.seed, 1e-2, 0, 3)
    state.tell(r1, f1)
    with pytest.raises(ValueError, match="no resident forward round"):
        state.tell(r1, f1)
    assert state.seed == 42 and state.rounds == 2


def test_resident_forward_search_round():
    """The resident BF16 search proposes a whole-model row; the forward
    scores it; the search is told -CE on the device."""
    from ennx_b200.experimental import ParamBlock, turbo_enn
    cfg = SMALL
    n = flat_size(cfg)
    base = torch.zeros(n, dtype=torch.bfloat16, device="cuda")
    w0 = init_weights(cfg, seed=8, std=0.05)
    view = weights_from_flat(cfg, base)
    view["embedding"].copy_(w0["embedding"])
    view["final_norm"].copy_(w0["final_norm"])
    for L, L0 in zip(view["layers"], w0["layers"]):
        for k in L:
            L[k].copy_(L0[k])
    blocks = [ParamBlock(1000 + i, off, int(np.prod(shape)), 1e-3) for i, (_, _, off, shape) in
              enumerate(flat_layout(cfg))]
    # the layout pads tensors to 16 elements: cover the gaps with small blocks
    covered, cursor, full = [], 0, []
    for b in sorted(blocks, key=lambda b: b.offset):
        if b.offset > cursor:
            full.append(ParamBlock(7, cursor, b.offset - cursor, 1e-6))
        full.append(b)
        cursor = b.offset + b.length
    if cursor < n:
        full.append(ParamBlock(7, cursor, n - cursor, 1e-6))
    B, S = 1, 48
    tok = torch.randint(0, cfg.vocab, (B, S + 1), generator=torch.Generator().manual_seed(9), dtype=torch.int32).cuda()
    base_fit = PopulationEvaluator(cfg, view, B, S)(tok, 0, 0.0, 0, 1)[0].item()
    search = turbo_enn(base, -base_fit, full, 4)
    loop = ResidentForwardSearch(cfg, search, B, S)
    reward = loop.ask_evaluate(tok, seed=3)
    accepted = search.sync()
    # re-score the trial the search now holds as incumbent or history
    assert torch.isfinite(reward).all() and abs(reward.item() + base_fit) < 0.5
    assert len(accepted) == 1
    assert search.history_len == 2
