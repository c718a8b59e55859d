"""torch-facing wrappers over the C ABI (device memory and streams from torch).

Every function here launches a kernel of ``libennx_b200.so``; none has a CPU
path.  Tensors must live on the current CUDA device.
"""
from __future__ import annotations

import ctypes

import torch

from . import _abi


def _ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _check_dev(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("ennx_b200 operates on CUDA tensors only")


def gemm(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None, *, epilogue: int = _abi.EPI_BF16,
         alpha: float = 1.0, groups: int = 1, b_group_rows: int = 0, group_offsets: torch.Tensor | None = None,
         residual: torch.Tensor | None = None, row_scale: torch.Tensor | None = None,
         targets: torch.Tensor | None = None, lse_partial: torch.Tensor | None = None,
         target_logit: torch.Tensor | None = None, n: int | None = None) -> torch.Tensor | None:
    """C = A . B^T on tcgen05 (see ``ennx_b200_gemm_bf16``).

    a: [M, K] bf16; b: [rows, K] bf16 where rows >= (groups-1)*b_group_rows + N.
    ``n`` defaults to b.shape[0] when there is one B block."""
    _check_dev(a, b, out, residual, row_scale, targets, group_offsets)
    if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
        raise ValueError("gemm operands must be bfloat16")
    M, K = a.shape
    N = n if n is not None else b.shape[0]
    if out is None and epilogue != _abi.EPI_LSE:
        cols = N // 2 if epilogue == _abi.EPI_SWIGLU else N
        out = torch.empty(M, cols, device=a.device,
                          dtype=torch.float32 if epilogue == _abi.EPI_F32 else torch.bfloat16)
    p = _abi.GemmParams(
        m=M, n=N, k=K, lda=a.stride(0), ldb=b.stride(0), ldc=0 if out is None else out.stride(0),
        groups=groups, b_group_rows=b_group_rows,
        group_offsets=None if group_offsets is None else group_offsets.data_ptr(),
        epilogue=epilogue, alpha=alpha,
        residual=None if residual is None else residual.data_ptr(),
        ldr=0 if residual is None else residual.stride(0),
        row_scale=None if row_scale is None else row_scale.data_ptr(),
        targets=None if targets is None else targets.data_ptr(),
        lse_partial=None if lse_partial is None else lse_partial.data_ptr(),
        target_logit=None if target_logit is None else target_logit.data_ptr())
    _abi.call("ennx_b200_gemm_bf16", ctypes.byref(p), _ptr(a), _ptr(b), _ptr(out), _stream())
    return out


def gemm_perturbed(a: torch.Tensor, w: torch.Tensor, e: torch.Tensor, out: torch.Tensor | None = None, *,
                   pairs: int = 1, epilogue: int = _abi.EPI_BF16, alpha: float = 1.0, b_group_rows: int = 0,
                   group_offsets: torch.Tensor | None = None, residual: torch.Tensor | None = None,
                   row_scale: torch.Tensor | None = None, targets: torch.Tensor | None = None,
                   lse_partial: torch.Tensor | None = None, target_logit: torch.Tensor | None = None,
                   n: int | None = None) -> torch.Tensor | None:
    """C = A . (W +/- E)^T with the perturbed operands formed inside the GEMM
    (see ``ennx_b200_gemm_bf16_perturbed``): 2*pairs row groups, the first
    `pairs` against W + E, the rest against W - E."""
    _check_dev(a, w, e, out, residual, row_scale, targets, group_offsets)
    if a.dtype != torch.bfloat16 or w.dtype != torch.bfloat16 or e.dtype != torch.bfloat16:
        raise ValueError("gemm operands must be bfloat16")
    if w.shape != e.shape or w.stride() != e.stride():
        raise ValueError("W and E must have the same shape and strides")
    M, K = a.shape
    N = n if n is not None else w.shape[0]
    if out is None and epilogue != _abi.EPI_LSE:
        cols = N // 2 if epilogue == _abi.EPI_SWIGLU else N
        out = torch.empty(M, cols, device=a.device,
                          dtype=torch.float32 if epilogue == _abi.EPI_F32 else torch.bfloat16)
    p = _abi.GemmParams(
        m=M, n=N, k=K, lda=a.stride(0), ldb=w.stride(0), ldc=0 if out is None else out.stride(0),
        groups=2 * pairs, b_group_rows=b_group_rows,
        group_offsets=None if group_offsets is None else group_offsets.data_ptr(),
        epilogue=epilogue, alpha=alpha,
        residual=None if residual is None else residual.data_ptr(),
        ldr=0 if residual is None else residual.stride(0),
        row_scale=None if row_scale is None else row_scale.data_ptr(),
        targets=None if targets is None else targets.data_ptr(),
        lse_partial=None if lse_partial is None else lse_partial.data_ptr(),
        target_logit=None if target_logit is None else target_logit.data_ptr())
    _abi.call("ennx_b200_gemm_bf16_perturbed", ctypes.byref(p), _ptr(a), _ptr(w), _ptr(e), _ptr(out), _stream())
    return out


def perturb_bf16(w: torch.Tensor, seed: int, pair: int, tensor: int, sigma: float,
                 plus: torch.Tensor | None = None, minus: torch.Tensor | None = None):
    """(W + sigma*eps, W - sigma*eps) with Philox noise keyed by (seed, pair, tensor, element).
    w None: `plus` receives the noise step bf16(sigma*eps) itself (minus must be None)."""
    if w is None:
        if plus is None or minus is not None:
            raise ValueError("the noise step alone needs `plus` and no `minus`")
        _check_dev(plus)
        n = plus.numel()
    else:
        _check_dev(w)
        plus = torch.empty_like(w) if plus is None else plus
        n = w.numel()
    _abi.call("ennx_b200_perturb_bf16", _ptr(w), n, seed, pair, tensor, sigma, _ptr(plus), _ptr(minus),
              _stream())
    return plus, minus


def device_status() -> None:
    """Synchronise and raise if any kernel recorded a bounded-wait timeout."""
    _abi.call("ennx_b200_device_status", _stream())


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6, out: torch.Tensor | None = None) -> torch.Tensor:
    _check_dev(x, w)
    out = torch.empty_like(x) if out is None else out
    _abi.call("ennx_b200_rmsnorm_bf16", _ptr(x), _ptr(w), x.shape[0], x.shape[1], eps, _ptr(out), _stream())
    return out


def packed_dequantize(weights: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, linear: _abi.PackedLinear,
                      seed: tuple[int, int, int] = (0, 0, 0), dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """Dequantised (and, when seed[2] != 0, code-perturbed) packed weights
    [output_width, input_width] (see ``ennx_b200_packed_dequantize_*``).
    weights: uint8 arena, scales/biases: float32 arenas, all on the device."""
    _check_dev(weights, scales, biases)
    out = torch.empty(linear.output_width, linear.input_width, device=weights.device, dtype=dtype)
    fn = "ennx_b200_packed_dequantize_bf16" if dtype == torch.bfloat16 else "ennx_b200_packed_dequantize_f32"
    if dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("packed_dequantize dtype must be bfloat16 or float32")
    _abi.call(fn, _ptr(weights), _ptr(scales), _ptr(biases), ctypes.byref(linear), _abi.PerturbSeed(*seed), _ptr(out),
              _stream())
    return out


def packed_linear(x: torch.Tensor, weights: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                  linear: _abi.PackedLinear, seed: tuple[int, int, int] = (0, 0, 0)) -> torch.Tensor:
    """out[t, r] = sum_c x[t, c] * W'[r, c] with the packed (perturbed) weights, bf16 in/out."""
    _check_dev(x, weights, scales, biases)
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.shape[1] != linear.input_width:
        raise ValueError("packed_linear input must be bfloat16 [tokens, input_width]")
    x = x.contiguous()
    out = torch.empty(x.shape[0], linear.output_width, device=x.device, dtype=torch.bfloat16)
    n = _abi.lib().ennx_b200_packed_linear_workspace_size(ctypes.byref(linear))
    ws = torch.empty(max(n, 16), device=x.device, dtype=torch.uint8)
    _abi.call("ennx_b200_packed_linear_bf16", _ptr(x), x.shape[0], _ptr(weights), _ptr(scales), _ptr(biases),
              ctypes.byref(linear), _abi.PerturbSeed(*seed), _ptr(out), _ptr(ws), ws.numel(), _stream())
    return out


def moe_route(x: torch.Tensor, w_router: torch.Tensor, top_k: int, with_logits: bool = False):
    """Routing indices (bit-exact with the CPU oracle) and renormalised gates."""
    _check_dev(x, w_router)
    T, H = x.shape
    E = w_router.shape[0]
    idx = torch.empty(T, top_k, dtype=torch.int32, device=x.device)
    gate = torch.empty(T, top_k, dtype=torch.float32, device=x.device)
    logits = torch.empty(T, E, dtype=torch.float32, device=x.device) if with_logits else None
    _abi.call("ennx_b200_moe_route", _ptr(x), _ptr(w_router), T, H, E, top_k, _ptr(logits), _ptr(idx), _ptr(gate),
              _stream())
    return (idx, gate, logits) if with_logits else (idx, gate)


def moe_layer(x: torch.Tensor, w_router: torch.Tensor, w_gate_up: torch.Tensor, w_down: torch.Tensor, top_k: int,
              residual: torch.Tensor | None = None, return_routing: bool = False):
    """y = (residual +) sum_r gate_r * W_d[e_r](silu(W_g[e_r] x) * W_u[e_r] x)."""
    _check_dev(x, w_router, w_gate_up, w_down, residual)
    T, H = x.shape
    E, I2, _ = w_gate_up.shape
    I = I2 // 2
    y = torch.empty_like(x)
    idx = torch.empty(T, top_k, dtype=torch.int32, device=x.device)
    gate = torch.empty(T, top_k, dtype=torch.float32, device=x.device)
    nbytes = _abi.lib().ennx_b200_moe_workspace_size(T, H, E, top_k, I)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
    _abi.call("ennx_b200_moe_layer", _ptr(x), _ptr(w_router), _ptr(w_gate_up), _ptr(w_down), T, H, E, top_k, I,
              _ptr(residual), _ptr(y), _ptr(idx), _ptr(gate), _ptr(ws), nbytes, _stream())
    return (y, idx, gate) if return_routing else y


def gqa_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, rope_theta: float = 1e6) -> torch.Tensor:
    """Causal GQA attention; q [B,S,Hq,128], k/v [B,S,Hkv,128] bf16.  q and k are
    rotated in place when rope_theta > 0."""
    _check_dev(q, k, v)
    B, S, Hq, D = q.shape
    o = torch.empty_like(q)
    _abi.call("ennx_b200_gqa_attention", _ptr(q), _ptr(k), _ptr(v), _ptr(o), B, S, Hq, k.shape[2], rope_theta,
              _stream())
    return o


def kda_chunked(q, k, v, g, beta, state: torch.Tensor | None = None) -> torch.Tensor:
    """Chunked KDA; q,k,v bf16 [B,T,H,128], g f32 [B,T,H,128], beta f32 [B,T,H]."""
    _check_dev(q, k, v, g, beta, state)
    B, T, H, D = q.shape
    o = torch.empty_like(v)
    nbytes = _abi.lib().ennx_b200_kda_workspace_size(B, T, H)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
    _abi.call("ennx_b200_kda_chunked", _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(state), _ptr(o), B, T, H,
              _ptr(ws), nbytes, _stream())
    return o


def l2norm_heads(x: torch.Tensor) -> torch.Tensor:
    """In-place per-head L2 normalisation of bf16 [rows, heads*128] (returns x)."""
    _check_dev(x)
    rows, width = x.shape
    _abi.call("ennx_b200_l2norm_heads_bf16", _ptr(x), rows, width // 128, x.stride(0), _stream())
    return x


def kda_gate_beta(raw_gate: torch.Tensor, raw_beta: torch.Tensor, decay: torch.Tensor, time_bias: torch.Tensor):
    """(g f32 [T, heads*128], beta f32 [T, heads]) from bf16 raw projections."""
    _check_dev(raw_gate, raw_beta, decay, time_bias)
    T, width = raw_gate.shape
    heads = width // 128
    g = torch.empty(T, width, dtype=torch.float32, device=raw_gate.device)
    b = torch.empty(T, heads, dtype=torch.float32, device=raw_gate.device)
    _abi.call("ennx_b200_kda_gate_beta", _ptr(raw_gate), raw_gate.stride(0), _ptr(raw_beta), raw_beta.stride(0),
              _ptr(decay), _ptr(time_bias), T, heads, _ptr(g), _ptr(b), _stream())
    return g, b


def kda_postprocess(o: torch.Tensor, gate: torch.Tensor, norm: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """Per-head RMSNorm x norm x sigmoid(gate); o, gate bf16 [T, heads*128], norm bf16 [128]."""
    _check_dev(o, gate, norm)
    T, width = o.shape
    out = torch.empty_like(o)
    _abi.call("ennx_b200_kda_postprocess", _ptr(o), _ptr(gate), gate.stride(0), _ptr(norm), T, width // 128, eps,
              _ptr(out), _stream())
    return out


def kda_gated(qkv: torch.Tensor, raw_gate: torch.Tensor, raw_beta: torch.Tensor, decay: torch.Tensor,
              time_bias: torch.Tensor, batch: int, seq: int, state: torch.Tensor | None = None) -> torch.Tensor:
    """The forward's fused KDA: qkv bf16 [batch*seq, >= 3*heads*128] (q, k not
    normalised), raw_gate bf16 [batch*seq, heads*128], raw_beta bf16
    [batch*seq, >= heads]; returns o bf16 [batch*seq, heads*128]."""
    _check_dev(qkv, raw_gate, raw_beta, decay, time_bias, state)
    heads = raw_gate.shape[1] // 128
    o = torch.empty(batch * seq, heads * 128, dtype=torch.bfloat16, device=qkv.device)
    nbytes = _abi.lib().ennx_b200_kda_workspace_size(batch, seq, heads)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=qkv.device)
    _abi.call("ennx_b200_kda_gated", _ptr(qkv), qkv.stride(0), _ptr(raw_gate), raw_gate.stride(0), _ptr(raw_beta),
              raw_beta.stride(0), _ptr(decay), _ptr(time_bias), _ptr(state), _ptr(o), batch, seq, heads, _ptr(ws),
              nbytes, _stream())
    return o
