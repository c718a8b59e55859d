"""The allocation-free KDA entry point against the regular one.

ennx_b200_kda_chunked_noalloc serves callers that cannot allocate device
memory (inside a CUDA graph capture, under a host that owns all device memory,
in latency-critical loops): it takes its scratch from a static 32 MiB device
array instead of a caller workspace.  This file is collected last so that a
run stopping at the first failure has already run every other test; it also
passes on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

from ennx_b200 import _abi  # noqa: E402

RTOL, ATOL = 2e-2, 1e-2  # the chunked-KDA tolerance used by the other KDA tests


def _inputs(B, T, H, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.nn.functional.normalize(torch.randn(B, T, H, 128, generator=g, device="cuda"), dim=-1).bfloat16()
    k = torch.nn.functional.normalize(torch.randn(B, T, H, 128, generator=g, device="cuda"), dim=-1).bfloat16()
    v = torch.randn(B, T, H, 128, generator=g, device="cuda").bfloat16()
    gl = -5.0 * torch.rand(B, T, H, 128, generator=g, device="cuda") / 64.0
    beta = torch.sigmoid(torch.randn(B, T, H, generator=g, device="cuda"))
    return q, k, v, gl, beta


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _regular(q, k, v, gl, beta, state):
    B, T, H, _ = q.shape
    o = torch.empty_like(v)
    n = _abi.lib().ennx_b200_kda_workspace_size(B, T, H)
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    _abi.check(_abi.lib().ennx_b200_kda_chunked(_p(q), _p(k), _p(v), _p(gl), _p(beta), _p(state), _p(o), B, T, H,
                                                 _p(ws), n, _stream()), "kda_chunked")
    return o


def _noalloc(q, k, v, gl, beta, state):
    B, T, H, _ = q.shape
    o = torch.empty_like(v)
    _abi.check(_abi.lib().ennx_b200_kda_chunked_noalloc(_p(q), _p(k), _p(v), _p(gl), _p(beta), _p(state), _p(o),
                                                         B, T, H, _stream()), "kda_chunked_noalloc")
    return o


def test_noalloc_matches_regular_on_two_calls_in_a_row():
    torch.cuda.set_device(0)
    for call, (B, T, H, seed) in enumerate([(2, 300, 4, 1), (1, 1000, 8, 2)]):
        q, k, v, gl, beta = _inputs(B, T, H, seed)
        s_ref = torch.randn(B, H, 128, 128, device="cuda") * 0.1
        s_new = s_ref.clone()
        ref = _regular(q, k, v, gl, beta, s_ref)
        got = _noalloc(q, k, v, gl, beta, s_new)
        torch.cuda.synchronize()
        a, b = got.float().cpu().numpy(), ref.float().cpu().numpy()
        assert np.all(np.abs(a - b) <= ATOL + RTOL * np.abs(b)), f"call {call}: outputs differ"
        sa, sb = s_new.cpu().numpy(), s_ref.cpu().numpy()
        assert np.all(np.abs(sa - sb) <= ATOL + RTOL * np.abs(sb)), f"call {call}: final states differ"


def test_noalloc_rejects_problems_beyond_the_static_scratch():
    q, k, v, gl, beta = _inputs(1, 64, 1, 3)
    o = torch.empty_like(v)
    # 4 sequences x 16 heads x 16 chunks = 1024 chunk records > 508
    st = _abi.lib().ennx_b200_kda_chunked_noalloc(_p(q), _p(k), _p(v), _p(gl), _p(beta), None, _p(o), 4, 1024, 16,
                                                  _stream())
    assert st == _abi.INVALID_ARGUMENT
    assert b"static scratch" in _abi.lib().ennx_b200_last_error()
