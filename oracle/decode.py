"""CPU restatement of the reference's resident single-token KDA-MoE decoder on
packed weights.

TEST INFRASTRUCTURE ONLY: the checker for ``ennx_b200.native.NativeKdaModel``,
never the product.  Follows KdaMoeMetalModel::decode_token / generate /
prepare_candidate (rust/crates/ennx/src/forward_metal.rs:1256-1394) and the
layer order of KdaMoeMetalExecutor::encode_decode_layer (:614-810), with the
math of the Metal kernels (kda_moe.metal): decoder_rms_norm (:536-554),
packed projection (:399-449), kda_short_conv_decode (:481-508),
kda_normalize_qk (:510-534), kda_split_control_16k (:847-867),
kda_make_gate_beta_16k (:869-896), kda_decode_step (:283-338),
kda_postprocess_16k (:898-921), decoder_residual (:556-565),
moe_router_topk_simd (:625-689), moe_gate_up_simd / moe_down_simd (:759-834),
packed_embedding_lookup (:929-946) and decoder_argmax (:948-975).

Weights come from ``oracle.packed_dequantize`` (the C restatement of
packed_weight_device, integer-code perturbation included); everything else
is float64 numpy.  The Metal kernels keep activations in half precision, so
the reference's own numbers are not reproducible bit for bit anywhere: parity
is against this restatement, with tolerances in the tests.
"""
from __future__ import annotations

import numpy as np

from . import PackedLinear, packed_dequantize


def rms_norm(x, w, eps):
    return x / np.sqrt(np.mean(x * x) + eps) * w


def silu(x):
    return x / (1.0 + np.exp(-x))


def softplus(x):
    return np.maximum(x, 0.0) + np.log1p(np.exp(-np.abs(x)))


def decode_step(state, q, k, v, gate, beta):
    """kda_decode_step for one head: state [kw, vw] (updated in place)."""
    kw = state.shape[0]
    state *= np.exp(gate)[:, None]
    read = k @ state
    state += np.outer(k, beta * (v - read))
    return (q @ state) / np.sqrt(kw)


def argmax_lanes(logits, lanes=256):
    """decoder_argmax: per-lane strided scan (strict '>'), then a tree that
    keeps the left entry unless the right one is strictly larger."""
    val = np.full(lanes, -np.inf)
    ind = np.zeros(lanes, np.int64)
    for lane in range(lanes):
        for i in range(lane, len(logits), lanes):
            if logits[i] > val[lane]:
                val[lane], ind[lane] = logits[i], i
    stride = lanes // 2
    while stride:
        for lane in range(stride):
            if val[lane + stride] > val[lane]:
                val[lane], ind[lane] = val[lane + stride], ind[lane + stride]
        stride //= 2
    return int(ind[0])


class DecoderOracle:
    def __init__(self, packed, scales, biases, linears, num_layers, hidden_size, heads, head_width, gate_rank,
                 num_experts, top_k, expert_width, residual_scale, rms_epsilon, embedding_scale):
        self.packed, self.scales, self.biases = packed, scales, biases
        self.named = {str(e[0]): tuple(int(v) for v in e[1:]) for e in linears}
        self.L, self.H, self.heads, self.hw = num_layers, hidden_size, heads, head_width
        self.rank, self.E, self.k, self.I = gate_rank, num_experts, top_k, expert_width
        self.rs, self.eps, self.emb_scale = residual_scale, rms_epsilon, embedding_scale
        self._cache = {}
        self.logits = None
        self.reset()
        self.prepare(0)

    def W(self, name, seed):
        key = (name, seed)
        if key not in self._cache:
            lin = PackedLinear(*self.named[name])
            s = (seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF, 1)  # MetalSeed::from
            self._cache[key] = packed_dequantize(self.packed, self.scales, self.biases, lin, s).astype(np.float64)
        return self._cache[key]

    def reset(self):
        W = self.heads * self.hw
        self.state = np.zeros((self.L, self.heads, self.hw, self.hw))
        self.hist = np.zeros((self.L, 3, 3 * W))

    def prepare(self, seed):
        self.vec = []
        for i in range(self.L):
            a = f"layers.{i}.attention"
            self.vec.append({n: self.W(name, seed)[0] for n, name in (
                ("attn_norm", f"layers.{i}.attention_norm"), ("moe_norm", f"layers.{i}.moe_norm"),
                ("decay", f"{a}.decay"), ("time_bias", f"{a}.time_bias"), ("out_norm", f"{a}.output_norm"))})
        self.final_norm = self.W("final_norm", seed)[0]

    def decode_token(self, token, seed=0):
        heads, hw, r = self.heads, self.hw, self.rank
        W = heads * hw
        x = self.W("embedding", seed)[token] * self.emb_scale
        for i in range(self.L):
            a, m, v = f"layers.{i}.attention", f"layers.{i}.moe", self.vec[i]
            n = rms_norm(x, v["attn_norm"], self.eps)
            qkv = self.W(f"{a}.qkv", seed) @ n
            taps = self.W(f"{a}.qkv_conv", seed)             # [3W, 4]
            h = self.hist[i]
            conv = h[0] * taps[:, 0] + h[1] * taps[:, 1] + h[2] * taps[:, 2] + qkv * taps[:, 3]
            self.hist[i] = np.stack([h[1], h[2], qkv])
            qkv = silu(conv)
            q, k, val = qkv[:W].reshape(heads, hw), qkv[W:2 * W].reshape(heads, hw), qkv[2 * W:].reshape(heads, hw)
            q = q / np.maximum(np.linalg.norm(q, axis=1, keepdims=True), 1e-6)
            k = k / np.maximum(np.linalg.norm(k, axis=1, keepdims=True), 1e-6)
            ctl = self.W(f"{a}.control", seed) @ n
            raw_gate = self.W(f"{a}.forget_b", seed) @ ctl[:r]
            og = self.W(f"{a}.gate_b", seed) @ ctl[r:2 * r]
            gate = np.maximum(-np.exp(np.repeat(v["decay"], hw)) * softplus(raw_gate + v["time_bias"]), -5.0)
            beta = 1.0 / (1.0 + np.exp(-ctl[2 * r:2 * r + heads]))
            o = np.stack([decode_step(self.state[i, hh], q[hh], k[hh], val[hh], gate[hh * hw:(hh + 1) * hw],
                                      beta[hh]) for hh in range(heads)])
            post = np.stack([rms_norm(o[hh], v["out_norm"], self.eps) for hh in range(heads)]).reshape(-1)
            post = post / (1.0 + np.exp(-og))
            x = x + self.rs * (self.W(f"{a}.output", seed) @ post)
            n = rms_norm(x, v["moe_norm"], self.eps)
            scores = self.W(f"{m}.router", seed) @ n
            vals, inds = [-np.inf] * self.k, [0] * self.k
            for e, sc in enumerate(scores):
                for rk in range(self.k):
                    if sc > vals[rk]:
                        vals[rk + 1:], inds[rk + 1:] = vals[rk:-1], inds[rk:-1]
                        vals[rk], inds[rk] = sc, e
                        break
            w = np.exp(np.array(vals) - vals[0])
            w = w / w.sum()
            y = np.zeros(self.H)
            for rk in range(self.k):
                e = inds[rk]
                act = silu(self.W(f"{m}.experts.{e}.gate", seed) @ n) * (self.W(f"{m}.experts.{e}.up", seed) @ n)
                y += w[rk] * (self.W(f"{m}.experts.{e}.down", seed) @ act)
            x = x + self.rs * y
        n = rms_norm(x, self.final_norm, self.eps)
        self.logits = self.W("embedding", seed) @ n
        return argmax_lanes(self.logits)

    def generate(self, prompt, max_new_tokens, seed=0):
        *prefix, last = prompt
        for t in prefix:
            self.decode_token(t, seed)
        nxt = self.decode_token(last, seed)
        out = list(prompt)
        for i in range(max_new_tokens):
            out.append(nxt)
            if i + 1 < max_new_tokens:
                nxt = self.decode_token(nxt, seed)
        return out


def kda_prefill_block(packed, scales, biases, linears, layer, heads, gate_rank, eps, residual_scale, normalized,
                      hidden, batch, seq, seed=None, state=None):
    """The 16k prefill KDA block (KdaMoeMetalExecutor::kda, forward_metal.rs:
    997-1129) in float64 between the points where the device stores bf16:
    packed projections, gate/beta, the serial recurrence (fp32 state), per-
    head norm x sigmoid(gate), output projection, residual.  No short
    convolution and no q/k L2 norm, as that path has none."""
    from . import kda_postprocess, kda_recurrence, round_bf16
    named = {str(e[0]): tuple(int(v) for v in e[1:]) for e in linears}
    a = f"layers.{layer}.attention"
    s = (0, 0, 0) if seed is None else (seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF, 1)

    def W(n):
        return packed_dequantize(packed, scales, biases, PackedLinear(*named[f"{a}.{n}"]), s).astype(np.float64)

    hw, r = heads * 128, gate_rank
    T = batch * seq
    x = np.asarray(normalized, np.float64)
    qkv = round_bf16((x @ W("qkv").T).astype(np.float32))
    ctl = round_bf16((x @ W("control").T).astype(np.float32))
    f = round_bf16((ctl[:, :r].astype(np.float64) @ W("forget_b").T).astype(np.float32))
    og = round_bf16((ctl[:, r:2 * r].astype(np.float64) @ W("gate_b").T).astype(np.float32))
    decay = round_bf16(W("decay")[0].astype(np.float32)).astype(np.float64)
    tb = round_bf16(W("time_bias")[0].astype(np.float32)).astype(np.float64)
    onorm = round_bf16(W("output_norm")[0].astype(np.float32))
    g = np.maximum(-np.repeat(np.exp(decay), 128)[None, :] * softplus(f.astype(np.float64) + tb[None, :]), -5.0)
    beta = 1.0 / (1.0 + np.exp(-ctl[:, 2 * r:2 * r + heads].astype(np.float64)))
    shp = (batch, seq, heads, 128)
    o, st = kda_recurrence(qkv[:, :hw].reshape(shp), qkv[:, hw:2 * hw].reshape(shp), qkv[:, 2 * hw:].reshape(shp),
                           g.astype(np.float32).reshape(shp), beta.astype(np.float32).reshape(batch, seq, heads),
                           state)
    o = round_bf16(o).reshape(T, heads, 128)
    post = round_bf16(kda_postprocess(o, og, onorm, eps).reshape(T, hw))
    upd = post.astype(np.float64) @ W("output").T
    out = round_bf16((np.asarray(hidden, np.float64) + residual_scale * upd).astype(np.float32))
    return out, st
