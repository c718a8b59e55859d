"""tcgen05 GEMM against the float64 oracle: C = A . B^T, bf16 in, fp32 accumulate.

Tolerance: |C - ref| <= 1e-2 + 2e-2 * |ref| for bf16
outputs; fp32 outputs are held to 2e-3 relative of the row scale."""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

from ennx_b200 import _abi, ops  # noqa: E402

RTOL, ATOL = 2e-2, 1e-2


@pytest.fixture(params=["0", "1"], ids=["1cta", "cta_pair"], autouse=True)
def gemm_variant(request, monkeypatch):
    """Run every GEMM test with the single-CTA and the CTA-pair (cta_group::2) kernel."""
    monkeypatch.setenv("ENNX_B200_GEMM_PAIR", request.param)
    return request.param


def rand_bf16(shape, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16)


def ref_gemm(a, b):
    return O.gemm(a.float().numpy(), b.float().numpy())


def close(got, ref, rtol=RTOL, atol=ATOL):
    got = np.asarray(got, np.float64)
    err = np.abs(got - ref) - (atol + rtol * np.abs(ref))
    assert err.max() <= 0, f"max excess {err.max()} at {np.unravel_index(err.argmax(), err.shape)}"


@pytest.mark.parametrize("m,n,k", [(2048, 2048, 2048), (128, 256, 64), (300, 200, 128), (129, 1000, 192),
                                   (1, 8, 64), (4096, 272, 2048)])
def test_gemm_bf16_shapes(m, n, k):
    a, b = rand_bf16((m, k), 0), rand_bf16((n, k), 1)
    c = ops.gemm(a.cuda(), b.cuda())
    torch.cuda.synchronize()
    close(c.float().cpu().numpy(), ref_gemm(a, b))


def test_gemm_f32_and_alpha():
    a, b = rand_bf16((256, 512), 2), rand_bf16((384, 512), 3)
    c = ops.gemm(a.cuda(), b.cuda(), epilogue=_abi.EPI_F32, alpha=0.5)
    ref = 0.5 * ref_gemm(a, b)
    np.testing.assert_allclose(c.cpu().numpy(), ref, rtol=1e-4, atol=1e-3)


def test_gemm_residual_in_place():
    a, b = rand_bf16((256, 256), 4), rand_bf16((512, 256), 5)
    r = rand_bf16((256, 512), 6).cuda()
    ref = O.round_bf16(r.float().cpu().numpy()) + ref_gemm(a, b)
    ops.gemm(a.cuda(), b.cuda(), out=r, residual=r)
    close(r.float().cpu().numpy(), ref)


def test_gemm_grouped_uniform_two_candidates():
    # two row segments (antithetic candidates) against two B blocks
    a = rand_bf16((512, 256), 7)
    b = rand_bf16((2 * 384, 256), 8)
    c = ops.gemm(a.cuda(), b.cuda(), groups=2, b_group_rows=384, n=384)
    ref = np.concatenate([ref_gemm(a[:256], b[:384]), ref_gemm(a[256:], b[384:])])
    close(c.float().cpu().numpy(), ref)


def test_gemm_grouped_device_offsets_ragged():
    counts = [0, 5, 130, 1, 300, 0, 64]
    offs = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    M, N, K, G = int(offs[-1]), 256, 128, len(counts)
    a = rand_bf16((M, K), 9)
    b = rand_bf16((G * N, K), 10)
    c = ops.gemm(a.cuda(), b.cuda(), groups=G, b_group_rows=N, n=N,
                 group_offsets=torch.from_numpy(offs).cuda())
    ref = np.zeros((M, N))
    for g in range(G):
        if counts[g]:
            ref[offs[g]:offs[g + 1]] = ref_gemm(a[offs[g]:offs[g + 1]], b[g * N:(g + 1) * N])
    close(c.float().cpu().numpy(), ref)


@pytest.mark.parametrize("epi", ["bf16", "swiglu", "rowscale"])
def test_gemm_grouped_tail_tiles(epi):
    # group sizes around the 256-row pair tile (partial last tiles of at most
    # and of more than 128 rows, empty groups), every fused epilogue
    counts = [256, 128, 129, 384, 0, 512, 640, 1, 255, 385]
    offs = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    M, N, K, G = int(offs[-1]), 512, 192, len(counts)
    a = rand_bf16((M, K), 20)
    b = rand_bf16((G * N, K), 21, 0.1)
    kw = dict(groups=G, b_group_rows=N, n=N, group_offsets=torch.from_numpy(offs).cuda())
    ref = np.zeros((M, N))
    for g in range(G):
        if counts[g]:
            ref[offs[g]:offs[g + 1]] = ref_gemm(a[offs[g]:offs[g + 1]], b[g * N:(g + 1) * N])
    if epi == "swiglu":
        c = ops.gemm(a.cuda(), b.cuda(), epilogue=_abi.EPI_SWIGLU, **kw)
        # each 256-column tile holds 128 gate columns, then their 128 up columns
        gate = np.concatenate([ref[:, t:t + 128] for t in range(0, N, 256)], 1)
        up = np.concatenate([ref[:, t + 128:t + 256] for t in range(0, N, 256)], 1)
        ref = O.silu(gate) * up
    elif epi == "rowscale":
        rs = torch.rand(M, generator=torch.Generator().manual_seed(22))
        c = ops.gemm(a.cuda(), b.cuda(), epilogue=_abi.EPI_ROWSCALE, row_scale=rs.cuda(), **kw)
        ref = ref * rs.double().numpy()[:, None]
    else:
        c = ops.gemm(a.cuda(), b.cuda(), **kw)
    close(c.float().cpu().numpy(), ref)


def test_gemm_swiglu_epilogue():
    M, I, K = 200, 512, 256
    a = rand_bf16((M, K), 11)
    wg, wu = rand_bf16((I, K), 12, 0.1), rand_bf16((I, K), 13, 0.1)
    blocks = [torch.cat([wg[i:i + 128], wu[i:i + 128]]) for i in range(0, I, 128)]
    b = torch.cat(blocks)
    c = ops.gemm(a.cuda(), b.cuda(), epilogue=_abi.EPI_SWIGLU)
    g, u = ref_gemm(a, wg), ref_gemm(a, wu)
    close(c.float().cpu().numpy(), O.silu(g) * u)


def test_gemm_rowscale_epilogue():
    a, b = rand_bf16((130, 128), 14), rand_bf16((256, 128), 15)
    s = torch.rand(130)
    c = ops.gemm(a.cuda(), b.cuda(), epilogue=_abi.EPI_ROWSCALE, row_scale=s.cuda())
    close(c.float().cpu().numpy(), ref_gemm(a, b) * s.numpy()[:, None].astype(np.float64))


@pytest.mark.parametrize("V", [1000, 1100, 1152])
def test_gemm_lse_epilogue_cross_entropy(V):
    M, K = 257, 128
    a, b = rand_bf16((M, K), 16, 0.5), rand_bf16((V, K), 17, 0.5)
    tg = torch.randint(0, V, (M,), generator=torch.Generator().manual_seed(0), dtype=torch.int32)
    nt = 2 * ((V + 255) // 256)
    lse = torch.empty(M, nt, 2, device="cuda")
    tl = torch.empty(M, device="cuda")
    ops.gemm(a.cuda(), b.cuda(), epilogue=_abi.EPI_LSE, targets=tg.cuda(), lse_partial=lse, target_logit=tl)
    part = lse.cpu().numpy().astype(np.float64)
    mx = part[..., 0].max(1)
    lse_tot = mx + np.log((part[..., 1] * np.exp(part[..., 0] - mx[:, None])).sum(1))
    loss = lse_tot - tl.cpu().numpy()
    logits = ref_gemm(a, b)
    ref = O.cross_entropy_rows(logits.astype(np.float32), tg.numpy())
    np.testing.assert_allclose(loss, ref, rtol=1e-4, atol=1e-4)


def test_gemm_rejects_bad_k():
    a, b = rand_bf16((128, 96), 0).cuda(), rand_bf16((128, 96), 1).cuda()
    with pytest.raises(ValueError if False else _abi.EnnxB200Error):
        ops.gemm(a, b)
