"""Independent CPU checks of the oracle pieces that no reference test pins.

The reference has no CPU attention, RoPE, cross-entropy or chunk-free KDA
test of its own, so the C restatements in oracle/ are checked here against
torch's CPU operators (float64) and a plain torch loop written from the
gated delta rule's definition."""
import math

import numpy as np
import pytest

import oracle as O

torch = pytest.importorskip("torch")


def _rope_torch(x, theta):
    # rotate-half pairing (i, i + d/2), position = sequence index
    B, S, H, D = x.shape
    half = D // 2
    inv = theta ** (-2.0 * torch.arange(half, dtype=torch.float64) / D)
    ang = torch.arange(S, dtype=torch.float64)[:, None] * inv[None, :]
    c, s = torch.cos(ang)[None, :, None, :], torch.sin(ang)[None, :, None, :]
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


@pytest.mark.parametrize("B,S,Hq,Hkv,seed", [(1, 37, 4, 1, 0), (2, 64, 8, 2, 1), (1, 5, 2, 2, 2)])
def test_gqa_attention_and_rope_vs_torch_sdpa(B, S, Hq, Hkv, seed):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, S, Hq, 128)).astype(np.float32)
    k = rng.standard_normal((B, S, Hkv, 128)).astype(np.float32)
    v = rng.standard_normal((B, S, Hkv, 128)).astype(np.float32)
    rq, rk = O.rope(q, 1e6), O.rope(k, 1e6)
    tq, tk = _rope_torch(torch.from_numpy(q).double(), 1e6), _rope_torch(torch.from_numpy(k).double(), 1e6)
    np.testing.assert_allclose(rq, tq.numpy(), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(rk, tk.numpy(), rtol=1e-5, atol=1e-5)
    got = O.gqa_attention(rq, rk, v)
    ref = torch.nn.functional.scaled_dot_product_attention(
        tq.transpose(1, 2), tk.transpose(1, 2), torch.from_numpy(v).double().transpose(1, 2), is_causal=True,
        enable_gqa=True, scale=1.0 / math.sqrt(128)).transpose(1, 2)
    np.testing.assert_allclose(got, ref.numpy(), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("rows,vocab,seed", [(17, 1000, 0), (64, 151936, 1)])
def test_cross_entropy_rows_vs_torch(rows, vocab, seed):
    rng = np.random.default_rng(seed)
    logits = (rng.standard_normal((rows, vocab)) * 3).astype(np.float32)
    tgt = rng.integers(0, vocab, rows).astype(np.int32)
    got = O.cross_entropy_rows(logits, tgt)
    ref = torch.nn.functional.cross_entropy(torch.from_numpy(logits).double(), torch.from_numpy(tgt).long(),
                                            reduction="none")
    np.testing.assert_allclose(got, ref.numpy(), rtol=1e-9, atol=1e-9)


def _kda_torch(q, k, v, g, beta):
    """S_t = diag(exp g_t) S_{t-1}; u = beta (v - k^T S); S += k u^T; o = q^T S / sqrt(dk)."""
    B, T, H, dk = q.shape
    dv = v.shape[-1]
    S = torch.zeros(B, H, dk, dv, dtype=torch.float64)
    out = torch.zeros(B, T, H, dv, dtype=torch.float64)
    for t in range(T):
        S = S * torch.exp(g[:, t])[..., None]
        kt, vt, qt = k[:, t], v[:, t], q[:, t]
        u = beta[:, t][..., None] * (vt - torch.einsum("bhk,bhkv->bhv", kt, S))
        S = S + kt[..., None] * u[..., None, :]
        out[:, t] = torch.einsum("bhk,bhkv->bhv", qt, S) / math.sqrt(dk)
    return out, S


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_kda_recurrence_vs_torch_loop(seed):
    rng = np.random.default_rng(seed)
    B, T, H = 2, 40, 2
    q = O.l2norm_heads(rng.standard_normal((B, T, H, 128)).astype(np.float32))
    k = O.l2norm_heads(rng.standard_normal((B, T, H, 128)).astype(np.float32))
    v = rng.standard_normal((B, T, H, 128)).astype(np.float32)
    g = (rng.uniform(-5.0, 0.0, (B, T, H, 128)) / (1.0 + 15 * seed)).astype(np.float32)
    beta = (1.0 / (1.0 + np.exp(-rng.standard_normal((B, T, H))))).astype(np.float32)
    got, st = O.kda_recurrence(q, k, v, g, beta)
    ref, rst = _kda_torch(*(torch.from_numpy(a).double() for a in (q, k, v, g, beta)))
    np.testing.assert_allclose(got, ref.numpy(), rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(st, rst.numpy(), rtol=1e-4, atol=1e-5)


def test_l2norm_and_rmsnorm_vs_torch():
    rng = np.random.default_rng(5)
    x = rng.standard_normal((33, 4, 128)).astype(np.float32)
    x[3, 1] = 0
    ref = torch.nn.functional.normalize(torch.from_numpy(x).double(), dim=-1, eps=1e-6)
    np.testing.assert_allclose(O.l2norm_heads(x), ref.numpy(), rtol=1e-6, atol=1e-7)
    y, w = rng.standard_normal((9, 256)).astype(np.float32), rng.standard_normal(256).astype(np.float32)
    ref = torch.nn.functional.rms_norm(torch.from_numpy(y).double(), (256,), torch.from_numpy(w).double(), eps=1e-6)
    np.testing.assert_allclose(O.rmsnorm(y, w, 1e-6), ref.numpy(), rtol=1e-5, atol=1e-6)
