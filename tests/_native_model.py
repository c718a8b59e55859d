"""Writes a small synthetic KDA-MoE model package in the reference's format
(model.toml + packed u8 codes + f32 scale and bias arenas, as read by
PackedModel::open, rust/crates/ennx/src/forward_weights.rs:15-106), for the
ModelPackage and NativeKdaModel tests.  Seeded; int4 and int8 linears, and
some linears with integer-code perturbation enabled."""
import os

import numpy as np

CONFIG = dict(num_layers=2, hidden_size=256, heads=2, head_width=128, gate_rank=16, num_experts=8, top_k=2,
              expert_width=64, residual_scale=0.5, rms_epsilon=1e-6, embedding_scale=1.0)
VOCAB = 384


def _plan(cfg):
    """(name, output_width, input_width, bits, group_size, kind, perturb_whole, perturb_threshold)"""
    H, heads, hw, r, E, I = (cfg[k] for k in ("hidden_size", "heads", "head_width", "gate_rank", "num_experts",
                                              "expert_width"))
    W = heads * hw
    plan = [("embedding", VOCAB, H, 8, 64, "matrix", 0, 0x30000000), ("final_norm", 1, H, 8, 64, "norm", 0, 0)]
    for i in range(cfg["num_layers"]):
        a, m = f"layers.{i}.attention", f"layers.{i}.moe"
        plan += [
            (f"layers.{i}.attention_norm", 1, H, 8, 64, "norm", 0, 0),
            (f"layers.{i}.moe_norm", 1, H, 8, 64, "norm", 0, 0),
            (f"{a}.qkv", 3 * W, H, 4, 32, "matrix", 0, 0x20000000),
            (f"{a}.qkv_conv", 3 * W, 4, 8, 4, "conv", 0, 0),
            (f"{a}.control", 2 * r + heads, H, 8, 64, "matrix", 1, 0),
            (f"{a}.forget_b", W, r, 4, 16, "matrix", 0, 0),
            (f"{a}.gate_b", W, r, 4, 16, "matrix", 0, 0x40000000),
            (f"{a}.output", H, W, 4, 64, "matrix", 0, 0),
            (f"{a}.decay", 1, heads, 8, heads, "decay", 0, 0),
            (f"{a}.time_bias", 1, W, 8, 64, "bias", 0, 0),
            (f"{a}.output_norm", 1, hw, 8, 64, "norm", 0, 0),
            (f"{m}.router", E, H, 8, 64, "matrix", 0, 0x10000000),
        ]
        for e in range(E):
            plan += [(f"{m}.experts.{e}.gate", I, H, 4, 32, "matrix", 0, 0),
                     (f"{m}.experts.{e}.up", I, H, 4, 32, "matrix", 0, 0x20000000),
                     (f"{m}.experts.{e}.down", H, I, 4, 32, "matrix", 0, 0)]
    return plan


def write_package(directory, seed=0, cfg=CONFIG):
    rng = np.random.default_rng(seed)
    codes, scales, biases, lines = [], [], [], ["weights = 'weights.bin'", "scales = 'scales.bin'",
                                               "biases = 'biases.bin'", ""]
    byte = scale_off = element = 0
    for name, out, inp, bits, group, kind, whole, threshold in _plan(cfg):
        maxc = (1 << bits) - 1
        c = rng.integers(0, maxc + 1, size=(out, inp))
        if bits == 4:
            padded = np.zeros((out, inp + (inp & 1)), np.int64)
            padded[:, :inp] = c
            packed = (padded[:, 0::2] | (padded[:, 1::2] << 4)).astype(np.uint8)
        else:
            packed = c.astype(np.uint8)
        groups = (inp + group - 1) // group
        mid = maxc / 2.0
        if kind == "matrix":
            s = np.full((out, groups), 3.0 / (maxc * np.sqrt(inp)), np.float32)
            b = (-s * mid).astype(np.float32)
        elif kind == "norm":
            s = np.full((out, groups), 0.2 / maxc, np.float32)
            b = np.full((out, groups), 1.0 - 0.1, np.float32)
        elif kind == "decay":
            s = np.full((out, groups), 1.0 / maxc, np.float32)
            b = np.full((out, groups), -1.5, np.float32)
        elif kind == "bias":
            s = np.full((out, groups), 0.4 / maxc, np.float32)
            b = np.full((out, groups), -0.2, np.float32)
        else:  # conv taps in [-0.5, 0.5]
            s = np.full((out, groups), 1.0 / maxc, np.float32)
            b = np.full((out, groups), -0.5, np.float32)
        codes.append(packed.reshape(-1))
        scales.append(s.reshape(-1))
        biases.append(b.reshape(-1))
        lines += ["[[linear]]", f"name = '{name}'", f"byte_offset = {byte}", f"scale_offset = {scale_off}",
                  f"bias_offset = {scale_off}", f"input_width = {inp}", f"output_width = {out}", f"bits = {bits}",
                  f"group_size = {group}", f"element_offset = {element}", f"perturb_whole = {whole}",
                  f"perturb_threshold = {threshold}", ""]
        byte += packed.size
        scale_off += s.size
        element += out * inp
    os.makedirs(directory, exist_ok=True)
    with open(os.path.join(directory, "model.toml"), "w") as f:
        f.write("\n".join(lines))
    np.concatenate(codes).astype(np.uint8).tofile(os.path.join(directory, "weights.bin"))
    np.concatenate(scales).astype("<f4").tofile(os.path.join(directory, "scales.bin"))
    np.concatenate(biases).astype("<f4").tofile(os.path.join(directory, "biases.bin"))
    return dict(cfg)
