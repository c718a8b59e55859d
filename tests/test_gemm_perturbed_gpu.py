"""The perturbed GEMM (W +/- E formed in the operand path) on the GPU.

Two checks per case:
* bit-identical to the plain CTA-pair GEMM run on materialised copies of
  bf16(W + E) and bf16(W - E): both issue the same M256 N256 K16 MMAs in the
  same order, so the perturbed operand path must produce exactly the bytes
  a stored copy would;
* within the BASELINE bound (|x - ref| <= 1e-2 + 2e-2 |ref|) of the float64
  oracle applied to the oracle's own perturbed weights.
"""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

from ennx_b200 import _abi, ops  # noqa: E402

RTOL, ATOL = 2e-2, 1e-2


@pytest.fixture(autouse=True)
def _pair_plain_gemm(monkeypatch):
    monkeypatch.setenv("ENNX_B200_GEMM_PAIR", "1")  # the plain kernel in the same MMA shape
    yield
    ops.device_status()


def rnd(shape, seed, std=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * std).to(torch.bfloat16)


def plus_minus(w, e):
    return (w.float() + e.float()).bfloat16(), (w.float() - e.float()).bfloat16()


def oracle_pm(w, e):
    """bf16(W +/- E) by the oracle's rounding rule, as float32 values."""
    wf, ef = w.float().numpy().astype(np.float64), e.float().numpy().astype(np.float64)
    return O.round_bf16((wf + ef).astype(np.float32)), O.round_bf16((wf - ef).astype(np.float32))


def close(got, ref):
    err = np.abs(np.asarray(got, np.float64) - ref) - (ATOL + RTOL * np.abs(ref))
    assert err.max() <= 0, f"max excess {err.max()} at {np.unravel_index(err.argmax(), err.shape)}"


@pytest.mark.parametrize("tc,n,k,resid", [(1000, 6416, 2048, True), (4096, 2048, 2048, False),
                                          (100, 264, 128, False), (1, 8, 64, True)])
def test_perturbed_dense_two_signs(tc, n, k, resid):
    a = rnd((2 * tc, k), 1)
    w, e = rnd((n, k), 2, 0.02), rnd((n, k), 3, 1e-3)
    r = rnd((2 * tc, n + (8 - n % 8) % 8), 4)[:, :n] if resid else None
    alpha = 0.5 if resid else 1.0
    wp, wm = plus_minus(w, e)
    r_dev = None if r is None else r.cuda()
    got = ops.gemm_perturbed(a.cuda(), w.cuda(), e.cuda(), pairs=1, alpha=alpha,
                             residual=r_dev, out=None if r is None else torch.empty_like(r_dev))
    plain = ops.gemm(a.cuda(), torch.cat([wp, wm]).cuda(), groups=2, b_group_rows=n, n=n, alpha=alpha,
                     residual=r_dev, out=None if r is None else torch.empty_like(r_dev))
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), plain.view(torch.int16))
    op, om = oracle_pm(w, e)
    af = a.float().numpy()
    ref = np.concatenate([alpha * O.gemm(af[:tc], op), alpha * O.gemm(af[tc:], om)])
    if r is not None:
        ref = ref + r.float().numpy()
    close(got.float().cpu().numpy(), ref)


@pytest.mark.parametrize("epi", [_abi.EPI_SWIGLU, _abi.EPI_ROWSCALE])
def test_perturbed_grouped_ragged(epi):
    """Expert-style groups: 2P ragged row segments (some empty, one sign of an
    expert larger than the other by more than a 256-row tile)."""
    P, k = 6, 256
    n = 512
    counts_p = [300, 0, 17, 600, 1, 256]
    counts_m = [290, 5, 0, 40, 513, 256]
    counts = counts_p + counts_m
    offs = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    M = int(offs[-1])
    a = rnd((M, k), 10)
    w, e = rnd((P, n, k), 11, 0.05), rnd((P, n, k), 12, 2e-3)
    scale = torch.rand(M, generator=torch.Generator().manual_seed(13)).float()
    wp, wm = plus_minus(w, e)
    kw = dict(epilogue=epi, b_group_rows=n, n=n, group_offsets=torch.from_numpy(offs).cuda(),
              row_scale=scale.cuda() if epi == _abi.EPI_ROWSCALE else None)
    got = ops.gemm_perturbed(a.cuda(), w.reshape(P * n, k).cuda(), e.reshape(P * n, k).cuda(), pairs=P, **kw)
    plain = ops.gemm(a.cuda(), torch.cat([wp, wm]).reshape(2 * P * n, k).cuda(), groups=2 * P, **kw)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), plain.view(torch.int16))
    op, om = oracle_pm(w, e)
    af = a.float().numpy()
    ref = []
    for g in range(2 * P):
        wg = (op if g < P else om)[g % P]
        acc = O.gemm(af[offs[g]:offs[g + 1]], wg)
        if epi == _abi.EPI_SWIGLU:
            blocks = acc.reshape(acc.shape[0], n // 256, 2, 128)
            acc = (O.silu(blocks[:, :, 0]) * blocks[:, :, 1]).reshape(acc.shape[0], n // 2)
        else:
            acc = acc * scale.numpy()[offs[g]:offs[g + 1], None]
        ref.append(acc)
    close(got.float().cpu().numpy(), np.concatenate(ref))


def test_perturbed_lse_head():
    """The LM-head form: online log-sum-exp partials and target logits over a
    vocabulary that is not a multiple of the tile width."""
    tc, V, k = 300, 5000, 512
    a = rnd((2 * tc, k), 20)
    w, e = rnd((V, k), 21, 0.05), rnd((V, k), 22, 1e-3)
    tgt = torch.randint(0, V, (2 * tc,), generator=torch.Generator().manual_seed(23), dtype=torch.int32).cuda()
    parts = 2 * ((V + 255) // 256)

    def run(fn, *args, **kw):
        lse = torch.empty(2 * tc, parts, 2, device="cuda")
        tl = torch.empty(2 * tc, device="cuda")
        fn(*args, epilogue=_abi.EPI_LSE, targets=tgt, lse_partial=lse, target_logit=tl, n=V, **kw)
        return lse, tl

    lse, tl = run(ops.gemm_perturbed, a.cuda(), w.cuda(), e.cuda(), pairs=1)
    wp, wm = plus_minus(w, e)
    lse2, tl2 = run(ops.gemm, a.cuda(), torch.cat([wp, wm]).cuda(), groups=2, b_group_rows=V)
    torch.cuda.synchronize()
    assert torch.equal(lse, lse2) and torch.equal(tl, tl2)
    # combine the partials into per-row cross-entropy and compare with the oracle
    m = lse[..., 0].cpu().numpy().astype(np.float64)
    ssum = lse[..., 1].cpu().numpy().astype(np.float64)
    mx = m.max(1, keepdims=True)
    got_lse = mx[:, 0] + np.log((ssum * np.exp(m - mx)).sum(1))
    op, om = oracle_pm(w, e)
    af = a.float().numpy()
    logits = np.concatenate([O.gemm(af[:tc], op), O.gemm(af[tc:], om)])
    lmx = logits.max(1, keepdims=True)
    ref_lse = lmx[:, 0] + np.log(np.exp(logits - lmx).sum(1))
    np.testing.assert_allclose(got_lse, ref_lse, rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(tl.cpu().numpy(), logits[np.arange(2 * tc), tgt.cpu().numpy()], rtol=1e-3, atol=1e-3)


def test_perturbed_rejects_odd_groups():
    a, w = rnd((128, 64), 30).cuda(), rnd((64, 64), 31).cuda()
    p = _abi.GemmParams(m=128, n=64, k=64, lda=64, ldb=64, ldc=64, groups=3, epilogue=_abi.EPI_BF16, alpha=1.0)
    out = torch.empty(128, 64, dtype=torch.bfloat16, device="cuda")
    import ctypes
    st = _abi.lib().ennx_b200_gemm_bf16_perturbed(ctypes.byref(p), ctypes.c_void_p(a.data_ptr()),
                                                  ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(w.data_ptr()),
                                                  ctypes.c_void_p(out.data_ptr()), None)
    assert st == _abi.INVALID_ARGUMENT and b"2 * pairs" in _abi.lib().ennx_b200_last_error()
