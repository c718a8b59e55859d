"""Hybrid KDA/GQA-MoE decoder: configuration, weight layout and the
population evaluator (host side of ``ennx_b200_population_forward``).

The evaluator is the B200 counterpart of the reference's evaluation seam,
``ForwardEvaluator::evaluate`` (rust/crates/ennx/src/forward_program.rs:
210-212): it scores a population of antithetic zeroth-order perturbations and
returns one scalar fitness (mean next-token cross-entropy) per candidate.
"""
from __future__ import annotations

import ctypes
from dataclasses import asdict, dataclass

import torch

from . import _abi

HEAD_DIM = 128


@dataclass(frozen=True)
class HybridConfig:
    layers: int = 24
    hidden: int = 2048
    vocab: int = 151936
    attn_period: int = 4          # [KDA, KDA, KDA, GQA] x 6
    q_heads: int = 16
    kv_heads: int = 4
    kda_heads: int = 16
    gate_rank: int = 128          # as buck2/tests/metal.rs:506
    experts: int = 64
    top_k: int = 8
    expert_width: int = 768
    rms_eps: float = 1e-6
    rope_theta: float = 1e6
    residual_scale: float = 1.0   # decoder_residual scale s (forward_program.rs:356; 0.22 in its tests)

    def is_gqa(self, layer: int) -> bool:
        return self.attn_period > 0 and layer % self.attn_period == self.attn_period - 1

    def layer_shapes(self, layer: int) -> dict:
        H, I, E = self.hidden, self.expert_width, self.experts
        if self.is_gqa(layer):
            s = {"attn_norm": (H,), "w_qkv": ((self.q_heads + 2 * self.kv_heads) * HEAD_DIM, H),
                 "w_o": (H, self.q_heads * HEAD_DIM)}
        else:
            hw = self.kda_heads * HEAD_DIM
            s = {"attn_norm": (H,), "w_qkv": (3 * hw, H), "w_ctl": (2 * self.gate_rank + self.kda_heads, H),
                 "w_forget": (hw, self.gate_rank), "w_ogate": (hw, self.gate_rank), "decay": (self.kda_heads,),
                 "time_bias": (hw,), "out_norm": (HEAD_DIM,), "w_o": (H, hw)}
        s.update({"moe_norm": (H,), "w_router": (E, H), "w_gate_up": (E, 2 * I, H), "w_down": (E, H, I)})
        return s

    def param_count(self) -> int:
        n = self.vocab * self.hidden + self.hidden
        for l in range(self.layers):
            for shp in self.layer_shapes(l).values():
                p = 1
                for d in shp:
                    p *= d
                n += p
        return n

    def flops_per_token(self, seq: int) -> float:
        """Algorithmic forward FLOPs per token (dense GEMMs + attention + KDA)."""
        H, I = self.hidden, self.expert_width
        f = 2.0 * self.vocab * H  # LM head
        avg_ctx = (seq + 1) / 2.0
        for l in range(self.layers):
            sh = self.layer_shapes(l)
            for name in ("w_qkv", "w_ctl", "w_forget", "w_ogate", "w_o", "w_router"):
                if name in sh:
                    f += 2.0 * sh[name][0] * sh[name][1]
            f += 2.0 * self.top_k * 3 * H * I
            if self.is_gqa(l):
                f += 4.0 * self.q_heads * HEAD_DIM * avg_ctx
            else:
                # chunked KDA, chunk 64: per token ~ 6*dk*dv (state read/update/output)
                # + 4*64*dk (intra-chunk products) + 2*64*dv (T.W)
                f += self.kda_heads * (6.0 * HEAD_DIM * HEAD_DIM + 4.0 * 64 * HEAD_DIM + 2.0 * 64 * HEAD_DIM)
        return f

    def to_c(self) -> _abi.ModelConfig:
        return _abi.ModelConfig(**asdict(self))


def gate_up_interleave(w_gate: torch.Tensor, w_up: torch.Tensor) -> torch.Tensor:
    """[E, I, H] gate and up -> [E, 2I, H] in blocks of 256 rows = [128 gate | 128 up]
    (the row layout the SwiGLU GEMM epilogue expects)."""
    E, I, H = w_gate.shape
    g = w_gate.reshape(E, I // 128, 128, H)
    u = w_up.reshape(E, I // 128, 128, H)
    return torch.cat([g, u], dim=2).reshape(E, 2 * I, H).contiguous()


def gate_up_split(w_gate_up: torch.Tensor):
    E, I2, H = w_gate_up.shape
    x = w_gate_up.reshape(E, I2 // 256, 2, 128, H)
    return x[:, :, 0].reshape(E, I2 // 2, H), x[:, :, 1].reshape(E, I2 // 2, H)


def init_weights(cfg: HybridConfig, seed: int = 0, device: str | torch.device = "cuda", std: float = 0.02) -> dict:
    """Random base weights, bf16: matrices ~ N(0, std), norm weights 1,
    KDA decay 0 (exp(decay) = 1), time bias 0."""
    g = torch.Generator(device=device).manual_seed(seed)

    def randn(*shape):
        return (torch.randn(*shape, generator=g, device=device, dtype=torch.float32) * std).to(torch.bfloat16)

    w = {"embedding": randn(cfg.vocab, cfg.hidden),
         "final_norm": torch.ones(cfg.hidden, device=device, dtype=torch.bfloat16), "layers": []}
    for l in range(cfg.layers):
        layer = {}
        for name, shp in cfg.layer_shapes(l).items():
            if name in ("attn_norm", "moe_norm", "out_norm"):
                layer[name] = torch.ones(*shp, device=device, dtype=torch.bfloat16)
            elif name in ("decay", "time_bias"):
                layer[name] = torch.zeros(*shp, device=device, dtype=torch.bfloat16)
            else:
                layer[name] = randn(*shp)
        w["layers"].append(layer)
    return w


def set_perturbation_mode(fused: bool) -> None:
    """Materialised W +/- e copies (False, the default) or the fused operand
    path of the perturbed GEMM (True) for every later population forward of
    this process; both give bit-identical perturbed weights."""
    _abi.call("ennx_b200_set_perturbation_mode", 1 if fused else 0)


class PopulationEvaluator:
    """Scores antithetic pairs of W +/- sigma*eps on one device.

    ``fitness = evaluator(tokens, seed, sigma, first_pair, num_pairs)`` returns a
    float32 CUDA tensor [2*num_pairs] (candidate 2i is W + sigma*eps_p, 2i+1 is
    W - sigma*eps_p, p = first_pair + i); tokens is int32 [batch, seq + 1]."""

    def __init__(self, cfg: HybridConfig, weights: dict, batch: int, seq: int):
        self.cfg, self.weights, self.batch, self.seq = cfg, weights, batch, seq
        self._ccfg = cfg.to_c()
        self._layers = (_abi.LayerWeights * cfg.layers)()
        for l, lw in enumerate(weights["layers"]):
            for f in _abi.LAYER_FIELDS:
                t = lw.get(f)
                setattr(self._layers[l], f, None if t is None else t.data_ptr())
        self._cw = _abi.ModelWeights(weights["embedding"].data_ptr(), weights["final_norm"].data_ptr(),
                                     self._layers)
        nbytes = _abi.lib().ennx_b200_population_workspace_size(ctypes.byref(self._ccfg), batch, seq)
        if nbytes == 0:
            _abi.check(_abi.INVALID_ARGUMENT, "population_workspace_size")
        self.workspace = torch.empty(nbytes, dtype=torch.uint8, device=weights["embedding"].device)

    def __call__(self, tokens: torch.Tensor, seed: int, sigma: float, first_pair: int, num_pairs: int,
                 out: torch.Tensor | None = None) -> torch.Tensor:
        if tokens.dtype != torch.int32 or tuple(tokens.shape) != (self.batch, self.seq + 1) or not tokens.is_cuda:
            raise ValueError(f"tokens must be a CUDA int32 tensor of shape {(self.batch, self.seq + 1)}")
        fit = torch.empty(2 * num_pairs, device=tokens.device, dtype=torch.float32) if out is None else out
        _abi.call("ennx_b200_population_forward", ctypes.byref(self._ccfg), ctypes.byref(self._cw), seed, sigma,
                  first_pair, num_pairs, ctypes.c_void_p(tokens.data_ptr()), self.batch, self.seq,
                  ctypes.c_void_p(fit.data_ptr()), ctypes.c_void_p(self.workspace.data_ptr()),
                  self.workspace.numel(), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        return fit

    def hidden(self, tokens: torch.Tensor, seed: int, sigma: float, pair: int, layers: int,
               with_routing: bool = False):
        """Residual stream after the first `layers` layers of antithetic pair
        `pair`: bf16 [2, batch*seq, hidden] (sign + first) -- a per-layer
        parity probe of the same device path as ``__call__``.  with_routing
        also returns the expert indices of layer `layers` - 1, int32
        [2, batch*seq, top_k]."""
        if tokens.dtype != torch.int32 or tuple(tokens.shape) != (self.batch, self.seq + 1) or not tokens.is_cuda:
            raise ValueError(f"tokens must be a CUDA int32 tensor of shape {(self.batch, self.seq + 1)}")
        out = torch.empty(2, self.batch * self.seq, self.cfg.hidden, device=tokens.device, dtype=torch.bfloat16)
        idx = torch.empty(2, self.batch * self.seq, self.cfg.top_k, device=tokens.device, dtype=torch.int32) \
            if with_routing else None
        _abi.call("ennx_b200_population_hidden", ctypes.byref(self._ccfg), ctypes.byref(self._cw), seed, sigma, pair,
                  layers, ctypes.c_void_p(tokens.data_ptr()), self.batch, self.seq, ctypes.c_void_p(out.data_ptr()),
                  None if idx is None else ctypes.c_void_p(idx.data_ptr()),
                  ctypes.c_void_p(self.workspace.data_ptr()), self.workspace.numel(),
                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        return (out, idx) if with_routing else out
