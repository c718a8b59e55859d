"""CPU oracle of the hybrid KDA/GQA-MoE population forward (TEST INFRASTRUCTURE ONLY).

Composes the C-oracle pieces (ennx_oracle.c) and float64 numpy GEMMs in the
layer order of the reference's KdaMoeMetalExecutor::encode_decode_layer
(rust/crates/ennx/src/forward_metal.rs:614-810), with GQA layers every
``attn_period`` layers and a mean next-token cross-entropy at the end.  The
reference has no CPU forward at all, so this oracle is builder-written: its
per-op formulas cite kda_moe.metal through the C functions it calls.
Activations are rounded to bf16 at the same storage points as the device
path so that the comparison measures arithmetic, not storage precision.
"""
from __future__ import annotations

import numpy as np

from . import (from_bf16_bits, gemm, gqa_attention, kda_recurrence, l2norm_heads, perturb_bf16, rmsnorm,
               round_bf16, rope, router_logits, router_topk, silu, to_bf16_bits)

HEAD_DIM = 128
FIELDS = ("attn_norm", "w_qkv", "w_ctl", "w_forget", "w_ogate", "decay", "time_bias", "out_norm", "w_o",
          "moe_norm", "w_router", "w_gate_up", "w_down")


def _sig(x):
    return 1.0 / (1.0 + np.exp(-x))


def _softplus(x):
    return np.maximum(x, 0) + np.log1p(np.exp(-np.abs(x)))


def perturbed(bits: np.ndarray, seed: int, pair: int, tensor: int, sigma, sign: int) -> np.ndarray:
    """bf16 bits -> float32 values of W + sign*sigma*eps (sigma None: W itself)."""
    if sigma is None:
        return from_bf16_bits(bits)
    return from_bf16_bits(perturb_bf16(bits.reshape(-1), seed, pair, tensor, sigma, sign)).reshape(bits.shape)


def candidate_loss(cfg, W: dict, tokens: np.ndarray, seed: int, sigma: float, pair: int, sign: int,
                   return_rows: bool = False, hidden_at: dict | None = None, router_gaps: list | None = None,
                   routing: list | None = None, start_hidden=None, first_layer: int = 0):
    """Mean CE of one candidate.  W: {'embedding': bits, 'final_norm': bits,
    'layers': [ {field: bits} ]} (bf16 bit patterns as uint16 arrays).
    hidden_at: {n: None} -> filled with the residual stream [T, H] after the
    first n layers (float32 values of the bf16 activations).
    router_gaps: list -> appended per layer with each token's gap between its
    k-th and (k+1)-th router logit (how close its expert choice is to a tie).
    routing: list -> appended per layer with the expert indices [T, k].
    start_hidden [T, H] / first_layer: run W["layers"] as layers
    first_layer, first_layer + 1, ... from the given residual stream instead
    of the embedding (per-layer isolation)."""
    B, S1 = tokens.shape
    S = S1 - 1
    T = B * S
    H = cfg.hidden
    rs = float(np.float32(getattr(cfg, "residual_scale", 1.0)))  # decoder_residual scale (kda_moe.metal:556-565)
    inp = tokens[:, :S].reshape(-1)
    tgt = tokens[:, 1:].reshape(-1)
    emb = perturbed(W["embedding"], seed, pair, 0, sigma, sign)
    h = emb[inp].astype(np.float32) if start_hidden is None else np.asarray(start_hidden, np.float32)
    for l, L in enumerate(W["layers"], start=first_layer):
        P = {f: perturbed(L[f], seed, pair, 16 + 16 * l + i, sigma, sign) for i, f in enumerate(FIELDS) if f in L}
        x = round_bf16(rmsnorm(h, P["attn_norm"], cfg.rms_eps))
        qkv = round_bf16(gemm(x, P["w_qkv"]).astype(np.float32))
        if cfg.is_gqa(l):
            hq, hkv = cfg.q_heads, cfg.kv_heads
            q = qkv[:, :hq * HEAD_DIM].reshape(B, S, hq, HEAD_DIM)
            k = qkv[:, hq * HEAD_DIM:(hq + hkv) * HEAD_DIM].reshape(B, S, hkv, HEAD_DIM)
            v = qkv[:, (hq + hkv) * HEAD_DIM:].reshape(B, S, hkv, HEAD_DIM)
            q = round_bf16(rope(q, cfg.rope_theta))
            k = round_bf16(rope(k, cfg.rope_theta))
            o = round_bf16(gqa_attention(q, k, v)).reshape(T, hq * HEAD_DIM)
            h = round_bf16((h + rs * gemm(o, P["w_o"])).astype(np.float32))
        else:
            nh, r = cfg.kda_heads, cfg.gate_rank
            hw = nh * HEAD_DIM
            ctl = round_bf16(gemm(x, P["w_ctl"]).astype(np.float32))
            f = round_bf16(gemm(ctl[:, :r], P["w_forget"]).astype(np.float32))
            og = round_bf16(gemm(ctl[:, r:2 * r], P["w_ogate"]).astype(np.float32))
            raw = f.astype(np.float64) + P["time_bias"].astype(np.float64)[None, :]
            dec = np.repeat(np.exp(P["decay"].astype(np.float64)), HEAD_DIM)[None, :]
            g = np.maximum(-dec * _softplus(raw), -5.0).astype(np.float32)
            beta = _sig(ctl[:, 2 * r:2 * r + nh].astype(np.float64)).astype(np.float32)
            q = round_bf16(l2norm_heads(qkv[:, :hw].reshape(T, nh, HEAD_DIM)))
            k = round_bf16(l2norm_heads(qkv[:, hw:2 * hw].reshape(T, nh, HEAD_DIM)))
            v = qkv[:, 2 * hw:].reshape(T, nh, HEAD_DIM)
            o, _ = kda_recurrence(q.reshape(B, S, nh, HEAD_DIM), k.reshape(B, S, nh, HEAD_DIM),
                                  v.reshape(B, S, nh, HEAD_DIM), g.reshape(B, S, nh, HEAD_DIM),
                                  beta.reshape(B, S, nh))
            o = round_bf16(o).reshape(T, nh, HEAD_DIM).astype(np.float64)
            inv = 1.0 / np.sqrt((o * o).mean(-1, keepdims=True) + cfg.rms_eps)
            post = o * inv * P["out_norm"].astype(np.float64) * _sig(og.reshape(T, nh, HEAD_DIM).astype(np.float64))
            post = round_bf16(post.reshape(T, hw).astype(np.float32))
            h = round_bf16((h + rs * gemm(post, P["w_o"])).astype(np.float32))
        # MoE
        x = round_bf16(rmsnorm(h, P["moe_norm"], cfg.rms_eps))
        logits = router_logits(to_bf16_bits(x), to_bf16_bits(P["w_router"]))
        idx, gate = router_topk(logits, cfg.top_k)
        if routing is not None:
            routing.append(idx.copy())
        if router_gaps is not None:
            srt = -np.sort(-logits.astype(np.float64), axis=1)
            k = cfg.top_k
            router_gaps.append(srt[:, k - 1] - srt[:, k] if k < srt.shape[1] else np.full(T, np.inf))
        wg_, wu_ = _split_gate_up(P["w_gate_up"])
        y = h.astype(np.float64)
        for e in range(cfg.experts):
            rows, ranks = np.nonzero(idx == e)
            if rows.size == 0:
                continue
            xe = x[rows]
            act = round_bf16((silu(gemm(xe, wg_[e])) * gemm(xe, wu_[e])).astype(np.float32))
            out = round_bf16((gemm(act, P["w_down"][e]) * (rs * gate[rows, ranks])[:, None]).astype(np.float32))
            np.add.at(y, rows, out.astype(np.float64))
        h = round_bf16(y.astype(np.float32))
        if hidden_at is not None and (l + 1 - first_layer) in hidden_at:
            hidden_at[l + 1 - first_layer] = h.copy()
    fnorm = perturbed(W["final_norm"], seed, pair, 1, sigma, sign)
    x = round_bf16(rmsnorm(h, fnorm, cfg.rms_eps))
    logits = gemm(x, emb)
    mx = logits.max(1)
    lse = mx + np.log(np.exp(logits - mx[:, None]).sum(1))
    rows = lse - logits[np.arange(T), tgt]
    return (rows.mean(), rows) if return_rows else rows.mean()


def _split_gate_up(w):
    E, I2, H = w.shape
    x = w.reshape(E, I2 // 256, 2, 128, H)
    return x[:, :, 0].reshape(E, I2 // 2, H), x[:, :, 1].reshape(E, I2 // 2, H)


def population_forward(cfg, W: dict, tokens: np.ndarray, seed: int, sigma: float, first_pair: int, num_pairs: int):
    out = []
    for i in range(num_pairs):
        for sign in (+1, -1):
            out.append(candidate_loss(cfg, W, tokens, seed, sigma, first_pair + i, sign))
    return np.array(out)


def population_update(cfg, W: dict, seed: int, coef, first_pair: int = 0) -> dict:
    """The zeroth-order update of every tensor (the forward's tensor ids)."""
    from . import es_update
    out = {"embedding": es_update(W["embedding"], seed, 0, coef, first_pair),
           "final_norm": es_update(W["final_norm"], seed, 1, coef, first_pair), "layers": []}
    for l, L in enumerate(W["layers"]):
        out["layers"].append({f: es_update(L[f], seed, 16 + 16 * l + i, coef, first_pair)
                              for i, f in enumerate(FIELDS) if f in L})
    return out
