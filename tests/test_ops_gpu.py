"""Forward-path operators on the GPU against the CPU oracle.

Routing indices are compared bit-exactly; bf16 outputs
within |x - ref| <= 1e-2 + 2e-2 |ref| unless stated."""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

from ennx_b200 import ops  # noqa: E402
from ennx_b200.model import gate_up_interleave  # noqa: E402

RTOL, ATOL = 2e-2, 1e-2


def rnd(shape, seed, std=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * std).to(torch.bfloat16)


def bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def close(got, ref, rtol=RTOL, atol=ATOL):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    err = np.abs(got - ref) - (atol + rtol * np.abs(ref))
    assert err.max() <= 0, f"max excess {err.max():.3e} at {np.unravel_index(err.argmax(), err.shape)}"


def test_rmsnorm():
    x, w = rnd((777, 2048), 0), rnd((2048,), 1)
    y = ops.rmsnorm(x.cuda(), w.cuda())
    close(y.float().cpu().numpy(), O.rmsnorm(x.float().numpy(), w.float().numpy()))


@pytest.mark.parametrize("tokens,hidden,experts,k", [(16384, 2048, 64, 8), (1000, 256, 8, 2), (333, 1024, 40, 8)])
def test_router_indices_bit_exact(tokens, hidden, experts, k):
    x = rnd((tokens, hidden), 2)
    w = rnd((experts, hidden), 3, 0.02)
    idx, gate, logits = ops.moe_route(x.cuda(), w.cuda(), k, with_logits=True)
    ref_logits = O.router_logits(bits(x), bits(w))
    assert np.array_equal(logits.cpu().numpy().view(np.uint32), ref_logits.view(np.uint32))
    ridx, rgate = O.router_topk(ref_logits, k)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    np.testing.assert_allclose(gate.cpu().numpy(), rgate, rtol=1e-5, atol=1e-6)


def test_router_ties_keep_lower_index():
    # identical expert rows -> identical logits; the lower index must win
    x = rnd((64, 256), 4)
    w = rnd((1, 256), 5).repeat(16, 1)
    idx, gate = ops.moe_route(x.cuda(), w.cuda(), 8)
    assert idx.cpu().numpy().tolist() == [list(range(8))] * 64
    np.testing.assert_allclose(gate.cpu().numpy(), 0.125, rtol=1e-6)


@pytest.mark.parametrize("tokens,hidden,experts,k,inter", [(512, 256, 8, 2, 128), (2048, 1024, 16, 8, 256)])
def test_moe_layer(tokens, hidden, experts, k, inter):
    x = rnd((tokens, hidden), 6)
    wr = rnd((experts, hidden), 7, 0.02)
    wg, wu = rnd((experts, inter, hidden), 8, 0.02), rnd((experts, inter, hidden), 9, 0.02)
    wd = rnd((experts, hidden, inter), 10, 0.02)
    res = rnd((tokens, hidden), 11)
    y, idx, gate = ops.moe_layer(x.cuda(), wr.cuda(), gate_up_interleave(wg, wu).cuda(), wd.cuda(), k,
                                 residual=res.cuda(), return_routing=True)
    ridx, rgate = O.router_topk(O.router_logits(bits(x), bits(wr)), k)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    ref = O.moe_experts(x.float().numpy(), ridx, rgate, wg.float().numpy(), wu.float().numpy(), wd.float().numpy())
    close(y.float().cpu().numpy(), ref + res.float().numpy())


@pytest.mark.parametrize("B,S,Hq,Hkv", [(1, 256, 4, 1), (2, 200, 4, 2), (1, 1, 2, 1), (1, 129, 8, 2)])
def test_gqa_attention(B, S, Hq, Hkv):
    q, k, v = rnd((B, S, Hq, 128), 12), rnd((B, S, Hkv, 128), 13), rnd((B, S, Hkv, 128), 14)
    rq = O.round_bf16(O.rope(q.float().numpy(), 1e6))
    rk = O.round_bf16(O.rope(k.float().numpy(), 1e6))
    ref = O.gqa_attention(rq, rk, v.float().numpy())
    o = ops.gqa_attention(q.cuda(), k.cuda(), v.cuda(), 1e6)
    close(o.float().cpu().numpy(), ref)


def _kda_inputs(B, T, H, seed, gscale):
    rng = np.random.default_rng(seed)
    q = O.l2norm_heads(rng.standard_normal((B, T, H, 128)).astype(np.float32))
    k = O.l2norm_heads(rng.standard_normal((B, T, H, 128)).astype(np.float32))
    q, k = O.round_bf16(q), O.round_bf16(k)
    v = O.round_bf16(rng.standard_normal((B, T, H, 128)).astype(np.float32))
    g = (rng.uniform(-5.0, 0.0, (B, T, H, 128)) / gscale).astype(np.float32)
    beta = (1.0 / (1.0 + np.exp(-rng.standard_normal((B, T, H))))).astype(np.float32)
    return q, k, v, g, beta


@pytest.mark.parametrize("B,T,H,gscale", [(1, 64, 1, 64.0), (2, 200, 2, 64.0), (1, 300, 1, 1.0), (1, 130, 2, 16.0)])
def test_kda_chunked_matches_serial_recurrence(B, T, H, gscale):
    q, k, v, g, beta = _kda_inputs(B, T, H, 20 + T, gscale)
    ref, ref_state = O.kda_recurrence(q, k, v, g, beta)
    tq, tk, tv = (torch.from_numpy(a).cuda().to(torch.bfloat16) for a in (q, k, v))
    state = torch.zeros(B, H, 128, 128, device="cuda")
    o = ops.kda_chunked(tq, tk, tv, torch.from_numpy(g).cuda(), torch.from_numpy(beta).cuda(), state)
    close(o.float().cpu().numpy(), ref, rtol=2e-2, atol=1e-2)
    close(state.cpu().numpy(), ref_state, rtol=2e-2, atol=2e-2)


def test_kda_state_carries_across_calls():
    q, k, v, g, beta = _kda_inputs(1, 256, 1, 5, 64.0)
    ref, _ = O.kda_recurrence(q, k, v, g, beta)
    dev = [torch.from_numpy(a).cuda() for a in (q, k, v, g, beta)]
    for i in range(3):
        dev[i] = dev[i].to(torch.bfloat16)
    state = torch.zeros(1, 1, 128, 128, device="cuda")
    halves = []
    for sl in (slice(0, 128), slice(128, 256)):
        parts = [d[:, sl].contiguous() for d in dev]
        halves.append(ops.kda_chunked(*parts, state=state).float().cpu().numpy())
    close(np.concatenate(halves, 1), ref)


@pytest.fixture(autouse=True)
def _device_status_clean():
    yield
    ops.device_status()  # a kernel that gave up on a bounded wait fails the test


def test_l2norm_heads_per_element():
    """kda_normalize_qk (kda_moe.metal:510-534): every element within bf16 rounding."""
    x = rnd((1000, 16 * 128), 30, 3.0)
    x[7, 256:384] = 0  # an all-zero head: max(|x|, 1e-6) keeps it zero
    y = ops.l2norm_heads(x.clone().cuda()).float().cpu().numpy()
    ref = O.l2norm_heads(x.float().numpy().reshape(1000, 16, 128)).reshape(1000, -1)
    close(y, ref, rtol=4e-3, atol=1e-6)
    assert np.all(y[7, 256:384] == 0)


def test_kda_gate_beta_per_element():
    """kda_make_gate_beta_16k (kda_moe.metal:869-895): g including the -5 clamp, beta."""
    T, heads = 777, 16
    raw = rnd((T, heads * 128), 31, 4.0)
    rbeta = rnd((T, heads), 32, 2.0)
    decay = rnd((heads,), 33, 0.7)
    tb = rnd((heads * 128,), 34, 0.5)
    g, b = ops.kda_gate_beta(raw.cuda(), rbeta.cuda(), decay.cuda(), tb.cuda())
    rg, rb = O.kda_gate_beta(raw.float().numpy(), rbeta.float().numpy(), decay.float().numpy(), tb.float().numpy(),
                             heads, 128)
    g, b = g.cpu().numpy(), b.cpu().numpy()
    close(g, rg, rtol=1e-4, atol=1e-6)
    close(b, rb, rtol=1e-5, atol=1e-6)
    assert (rg == -5.0).any() and np.array_equal(g == -5.0, rg == -5.0)


def test_kda_postprocess_per_element():
    """kda_postprocess_16k (kda_moe.metal:898-921): per-head RMSNorm x norm x sigmoid(gate)."""
    T, heads = 500, 16
    o, gate, norm = rnd((T, heads * 128), 35), rnd((T, heads * 128), 36, 2.0), rnd((128,), 37)
    y = ops.kda_postprocess(o.cuda(), gate.cuda(), norm.cuda(), 1e-6).float().cpu().numpy()
    ref = O.kda_postprocess(o.float().numpy().reshape(T, heads, 128), gate.float().numpy(), norm.float().numpy(),
                            1e-6).reshape(T, -1)
    close(y, ref, rtol=5e-3, atol=1e-5)


@pytest.mark.parametrize("B,T,heads", [(2, 200, 2), (1, 1000, 4)])
def test_kda_gated_matches_oracle(B, T, heads):
    """The forward's fused KDA (q/k L2 norm and gate/beta formed inside the
    chunk preparation) against l2norm_heads + kda_gate_beta + the serial
    recurrence of the oracle."""
    hw = heads * 128
    rows = B * T
    qkv = rnd((rows, 3 * hw + 64), 40)
    raw = rnd((rows, hw), 41, 1.5)
    rbeta = rnd((rows, 8), 42)
    decay, tb = rnd((heads,), 43, 0.5), rnd((hw,), 44, 0.5)
    o = ops.kda_gated(qkv.cuda(), raw.cuda(), rbeta.cuda(), decay.cuda(), tb.cuda(), B, T).float().cpu().numpy()
    qf = qkv.float().numpy()
    q = O.round_bf16(O.l2norm_heads(qf[:, :hw].reshape(rows, heads, 128)))
    k = O.round_bf16(O.l2norm_heads(qf[:, hw:2 * hw].reshape(rows, heads, 128)))
    v = qf[:, 2 * hw:3 * hw]
    g, beta = O.kda_gate_beta(raw.float().numpy(), rbeta.float().numpy()[:, :heads].copy(), decay.float().numpy(),
                              tb.float().numpy(), heads, 128)
    ref, _ = O.kda_recurrence(q.reshape(B, T, heads, 128), k.reshape(B, T, heads, 128), v.reshape(B, T, heads, 128),
                              g.reshape(B, T, heads, 128), beta.reshape(B, T, heads))
    close(o, ref.reshape(rows, hw))
