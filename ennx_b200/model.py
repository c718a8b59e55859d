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

    def coefficients(self, fitness: torch.Tensor, sigma: float, lr: float, total_pairs: int | None = None
                     ) -> torch.Tensor:
        """Update coefficients of the antithetic estimator from a device
        fitness vector [2P]: c_p = -lr (f+ - f-) / (2 sigma total_pairs)."""
        P = fitness.numel() // 2
        coef = torch.empty(P, device=fitness.device, dtype=torch.float32)
        _abi.call("ennx_b200_es_coefficients", ctypes.c_void_p(fitness.data_ptr()), P, total_pairs or P, sigma, lr,
                  ctypes.c_void_p(coef.data_ptr()), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        return coef

    def update(self, seed: int, coef: torch.Tensor, first_pair: int = 0) -> None:
        """W <- bf16(W + sum_p coef[p] eps_{first_pair + p}) for every tensor,
        in place in the weights this evaluator was built on (the noise of the
        forward's pairs, regenerated from `seed`)."""
        if coef.dtype != torch.float32 or not coef.is_cuda:
            raise ValueError("coefficients must be a CUDA float32 tensor")
        coef = coef.contiguous()
        _abi.call("ennx_b200_population_update", ctypes.byref(self._ccfg), ctypes.byref(self._cw), seed,
                  ctypes.c_void_p(coef.data_ptr()), first_pair, coef.numel(),
                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))

    def rebind(self, weights: dict) -> None:
        """Point the evaluator at other base weights of the same shapes (for
        example views into a search's resident row); the workspace is kept."""
        for l, lw in enumerate(weights["layers"]):
            for f in _abi.LAYER_FIELDS:
                t = lw.get(f)
                setattr(self._layers[l], f, None if t is None else t.data_ptr())
        self._cw = _abi.ModelWeights(weights["embedding"].data_ptr(), weights["final_norm"].data_ptr(),
                                     self._layers)
        self.weights = weights


def flat_layout(cfg: HybridConfig) -> list[tuple[str, int, int, tuple]]:
    """The model as one flat BF16 parameter vector: (name, layer, offset,
    shape) per tensor, every tensor starting on a 16-element boundary (the
    16-byte alignment the kernels need).  Names are the weight dict's keys."""
    out, off = [], 0

    def add(name, layer, shape):
        nonlocal off
        n = 1
        for d in shape:
            n *= d
        out.append((name, layer, off, tuple(shape)))
        off += (n + 15) // 16 * 16

    add("embedding", -1, (cfg.vocab, cfg.hidden))
    add("final_norm", -1, (cfg.hidden,))
    for l in range(cfg.layers):
        for name, shp in cfg.layer_shapes(l).items():
            add(name, l, shp)
    return out


def flat_size(cfg: HybridConfig) -> int:
    name, layer, off, shape = flat_layout(cfg)[-1]
    n = 1
    for d in shape:
        n *= d
    return off + (n + 15) // 16 * 16


def weights_from_flat(cfg: HybridConfig, flat: torch.Tensor) -> dict:
    """Weight dict of views into a flat BF16 vector laid out by ``flat_layout``."""
    w = {"layers": [dict() for _ in range(cfg.layers)]}
    for name, layer, off, shape in flat_layout(cfg):
        n = 1
        for d in shape:
            n *= d
        view = flat[off:off + n].view(*shape)
        if layer < 0:
            w[name] = view
        else:
            w["layers"][layer][name] = view
    return w


class ResidentForwardSearch:
    """The reference's resident BO round over the forward
    (``ResidentBoState::ask_evaluate``, forward_program.rs:706-720): the
    resident BF16 search proposes a trial row of the whole model's
    parameters, the population forward scores that row as the model (no
    population noise: sigma 0), and the mean cross-entropy goes back to the
    search as a device reward (-CE) without a host copy.

    ``search``: a ``SearchState`` whose rows are laid out by ``flat_layout``;
    ``tokens``: CUDA int32 [batch, seq + 1]."""

    def __init__(self, cfg: HybridConfig, search, batch: int, seq: int):
        from .search import SearchState
        if not isinstance(search, SearchState):
            raise TypeError("ResidentForwardSearch needs a SearchState")
        if search.len != flat_size(cfg):
            raise ValueError(f"search rows hold {search.len} values; the model needs {flat_size(cfg)}")
        self.cfg, self.search, self.batch, self.seq = cfg, search, batch, seq
        self._ev = None

    def ask_evaluate(self, tokens: torch.Tensor, seed: int, candidates: int = 8, neighbors: int = 8, **ask):
        """One round: ask (1 arm), evaluate the trial row, tell -CE.  Returns
        the device reward tensor [1]."""
        props = self.search.ask(1, candidates, neighbors, seed, **ask)
        batch = torch.from_dlpack(props)  # [1, len] trial row; the export lease lives with `batch`
        w = weights_from_flat(self.cfg, batch[0])
        if self._ev is None:
            self._ev = PopulationEvaluator(self.cfg, w, self.batch, self.seq)
        else:
            self._ev.rebind(w)
        fit = self._ev(tokens, 0, 0.0, 0, 1)  # both candidates of the pair are the row itself
        reward = (-fit[:1]).contiguous()
        self._ev.weights = None  # the evaluator keeps raw pointers only, not the lease
        del batch, w
        self.search.tell(props, reward)
        return reward
