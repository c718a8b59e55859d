"""ctypes binding of the C ABI in ``include/ennx_b200.h``.

The shared library is built in-tree (``ennx_b200/_lib/libennx_b200.so``) by
``ennx_b200.build``.  There is no CPU fallback: if the library is missing or
the device is not sm_100, every call raises.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libennx_b200.so"

OK, INVALID_ARGUMENT, OVERFLOW, CUDA_ERROR, TIMEOUT, UNSUPPORTED = range(6)
EPI_BF16, EPI_F32, EPI_SWIGLU, EPI_ROWSCALE, EPI_LSE = range(5)


class EnnxB200Error(RuntimeError):
    """A status other than ENNX_B200_OK returned by the C ABI."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class EnnxB200ValueError(EnnxB200Error, ValueError):
    """INVALID_ARGUMENT / OVERFLOW: the reference raises ValueError for these
    (rust/crates/ennx-py/src/py_weights.rs:27-29)."""


class DenseLeaf(ctypes.Structure):
    _fields_ = [("key", ctypes.c_uint64), ("offset", ctypes.c_size_t), ("len", ctypes.c_size_t),
                ("scale", ctypes.c_float)]


class DenseTerm(ctypes.Structure):
    _fields_ = [("seed", ctypes.c_uint64), ("coefficient", ctypes.c_float)]


class DenseView(ctypes.Structure):
    _fields_ = [("key", ctypes.c_uint64), ("start", ctypes.c_uint64), ("scale", ctypes.c_float)]


class Bf16Leaf(ctypes.Structure):
    """ennx_b200_bf16_leaf = Bf16Leaf (cuda/kernels/src/bf16.rs:5-13)."""
    _fields_ = [("key", ctypes.c_uint64), ("offset", ctypes.c_uint64), ("length", ctypes.c_uint64),
                ("scale", ctypes.c_float), ("weight", ctypes.c_float)]


class Selection(ctypes.Structure):
    _fields_ = [("index", ctypes.c_uint32), ("score", ctypes.c_float)]


class AskConfig(ctypes.Structure):
    _fields_ = [("neighbors", ctypes.c_uint32), ("acquisition", ctypes.c_uint32),
                ("epistemic_scale", ctypes.c_float), ("aleatoric_scale", ctypes.c_float),
                ("y_scale", ctypes.c_float), ("beta", ctypes.c_float)]


class TellSummary(ctypes.Structure):
    _fields_ = [("length", ctypes.c_double), ("best", ctypes.c_float), ("best_variance", ctypes.c_float),
                ("history", ctypes.c_uint32), ("restarts", ctypes.c_uint32), ("restarted", ctypes.c_uint32),
                ("status", ctypes.c_uint32)]


class GemmParams(ctypes.Structure):
    _fields_ = [("m", ctypes.c_int32), ("n", ctypes.c_int32), ("k", ctypes.c_int32),
                ("lda", ctypes.c_int64), ("ldb", ctypes.c_int64), ("ldc", ctypes.c_int64),
                ("groups", ctypes.c_int32), ("b_group_rows", ctypes.c_int32),
                ("group_offsets", ctypes.c_void_p), ("epilogue", ctypes.c_int32),
                ("alpha", ctypes.c_float), ("residual", ctypes.c_void_p), ("ldr", ctypes.c_int64),
                ("row_scale", ctypes.c_void_p), ("targets", ctypes.c_void_p),
                ("lse_partial", ctypes.c_void_p), ("target_logit", ctypes.c_void_p)]


class PackedLinear(ctypes.Structure):
    """ennx_b200_packed_linear: field order of KdaPackedLinear (forward_program.rs:224-235)."""
    _fields_ = [("byte_offset", ctypes.c_uint64), ("scale_offset", ctypes.c_uint64),
                ("bias_offset", ctypes.c_uint64), ("input_width", ctypes.c_uint64),
                ("output_width", ctypes.c_uint64), ("bits", ctypes.c_uint32), ("group_size", ctypes.c_uint32),
                ("element_offset", ctypes.c_uint64), ("perturb_whole", ctypes.c_uint32),
                ("perturb_threshold", ctypes.c_uint32)]


class KdaDecoderLayer(ctypes.Structure):
    """ennx_b200_kda_decoder_layer: the packed linears of one decoder layer."""
    _fields_ = [(n, PackedLinear) for n in ("qkv", "control", "output", "qkv_conv", "forget_b", "gate_b", "decay",
                                            "time_bias", "output_norm", "attention_norm", "moe_norm", "router")] + \
               [("expert_gate", ctypes.c_void_p), ("expert_up", ctypes.c_void_p), ("expert_down", ctypes.c_void_p)]


class KdaDecoderConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint32) for n in ("num_layers", "hidden", "heads", "head_width", "gate_rank",
                                               "num_experts", "top_k", "expert_width")] + \
               [("residual_scale", ctypes.c_float), ("rms_epsilon", ctypes.c_float),
                ("embedding_scale", ctypes.c_float)]


class PerturbSeed(ctypes.Structure):
    _fields_ = [("low", ctypes.c_uint32), ("high", ctypes.c_uint32), ("enabled", ctypes.c_uint32)]


class PackedKdaBlock(ctypes.Structure):
    """ennx_b200_packed_kda_block."""
    _fields_ = [(n, PackedLinear) for n in ("qkv", "control", "forget_b", "gate_b", "output", "decay", "time_bias",
                                            "output_norm")] + [
        ("heads", ctypes.c_int32), ("gate_rank", ctypes.c_int32), ("rms_eps", ctypes.c_float),
        ("residual_scale", ctypes.c_float)]


class ModelConfig(ctypes.Structure):
    _fields_ = [("layers", ctypes.c_int32), ("hidden", ctypes.c_int32), ("vocab", ctypes.c_int32),
                ("attn_period", ctypes.c_int32), ("q_heads", ctypes.c_int32), ("kv_heads", ctypes.c_int32),
                ("kda_heads", ctypes.c_int32), ("gate_rank", ctypes.c_int32), ("experts", ctypes.c_int32),
                ("top_k", ctypes.c_int32), ("expert_width", ctypes.c_int32), ("rms_eps", ctypes.c_float),
                ("rope_theta", ctypes.c_float), ("residual_scale", ctypes.c_float)]


LAYER_FIELDS = ("attn_norm", "w_qkv", "w_ctl", "w_forget", "w_ogate", "decay", "time_bias", "out_norm", "w_o",
                "moe_norm", "w_router", "w_gate_up", "w_down")


class LayerWeights(ctypes.Structure):
    _fields_ = [(f, ctypes.c_void_p) for f in LAYER_FIELDS]


class ModelWeights(ctypes.Structure):
    _fields_ = [("embedding", ctypes.c_void_p), ("final_norm", ctypes.c_void_p),
                ("layers", ctypes.POINTER(LayerWeights))]


_P = ctypes.c_void_p
_SZ = ctypes.c_size_t
_I32 = ctypes.c_int32
_U32 = ctypes.c_uint32
_U64 = ctypes.c_uint64
_F32 = ctypes.c_float

SIGNATURES = {
    "ennx_b200_abi_version": (_U32, []),
    "ennx_b200_last_error": (ctypes.c_char_p, []),
    "ennx_b200_device_check": (_I32, []),
    "ennx_b200_device_status": (_I32, [_P]),
    "ennx_b200_dense_apply_f32": (_I32, [_P, _SZ, _P, _SZ, _P, _SZ, _P, _P, _P]),
    "ennx_b200_dense_apply_bf16": (_I32, [_P, _SZ, _P, _SZ, _P, _SZ, _P, _P]),
    "ennx_b200_check_bf16": (_I32, [_P, _SZ, _P, _P]),
    "ennx_b200_dense_dist2": (_I32, [_P, _SZ, _P, _SZ, _P, _SZ, _P]),
    "ennx_b200_bf16_search_create": (_I32, [_P, _SZ, _P, _SZ, _SZ, _P, _P]),
    "ennx_b200_kda_decoder_create": (_I32, [_P, _SZ, _P, _SZ, _P, _SZ, _P, _P, _P, _P, _P, _P]),
    "ennx_b200_kda_decoder_destroy": (_I32, [_P]),
    "ennx_b200_kda_decoder_reset": (_I32, [_P]),
    "ennx_b200_kda_decoder_prepare": (_I32, [_P, _U64]),
    "ennx_b200_kda_decoder_decode_token": (_I32, [_P, _U32, _U64, _P]),
    "ennx_b200_kda_decoder_generate": (_I32, [_P, _P, _SZ, _SZ, _U64, _P]),
    "ennx_b200_kda_decoder_logits": (_I32, [_P, _P, _SZ]),
    "ennx_b200_bf16_search_destroy": (_I32, [_P]),
    "ennx_b200_bf16_search_init": (_I32, [_P, _F32, _F32, _SZ, ctypes.c_double, ctypes.c_double, ctypes.c_double]),
    "ennx_b200_bf16_search_copy_row": (_I32, [_P, _SZ, _SZ]),
    "ennx_b200_bf16_search_ask": (_I32, [_P, _SZ, _SZ, _P, _SZ, _P, _SZ, _F32, _U64, _P, _P]),
    "ennx_b200_bf16_search_ask_seeded": (_I32, [_P, _SZ, _P, _SZ, _SZ, _U64, _U64, _P]),
    "ennx_b200_bf16_search_tell": (_I32, [_P, _P, _SZ, _P, _P, _I32, _SZ, _SZ]),
    "ennx_b200_bf16_search_collect": (_I32, [_P, _SZ, _P, _P]),
    "ennx_b200_bf16_search_row": (_I32, [_P, _SZ, _P]),
    "ennx_b200_bf16_search_round": (_I32, [_P, _SZ, _P]),
    "ennx_b200_bf16_search_gather": (_I32, [_P, _P, _SZ, _P]),
    "ennx_b200_bf16_search_handoff": (_I32, [_P, _P, _I32]),
    "ennx_b200_bf16_search_last_scores": (_I32, [_P, _P, _SZ, _P, _SZ]),
    "ennx_b200_bf16_search_set_profiling": (_I32, [_P, _I32]),
    "ennx_b200_bf16_search_last_profile": (_I32, [_P, _P, _P]),
    "ennx_b200_dense_linear_f32": (_I32, [_P, _SZ, _P, _SZ, _P, DenseView, DenseView, _P, _SZ, _P, _P]),
    "ennx_b200_perturb_bf16": (_I32, [_P, _SZ, _U64, _U32, _U32, _F32, _P, _P, _P]),
    "ennx_b200_gemm_bf16": (_I32, [_P, _P, _P, _P, _P]),
    "ennx_b200_gemm_bf16_perturbed": (_I32, [_P, _P, _P, _P, _P, _P]),
    "ennx_b200_rmsnorm_bf16": (_I32, [_P, _P, ctypes.c_int64, _I32, _F32, _P, _P]),
    "ennx_b200_moe_route": (_I32, [_P, _P, ctypes.c_int64, _I32, _I32, _I32, _P, _P, _P, _P]),
    "ennx_b200_moe_workspace_size": (_SZ, [ctypes.c_int64, _I32, _I32, _I32, _I32]),
    "ennx_b200_moe_layer": (_I32, [_P, _P, _P, _P, ctypes.c_int64, _I32, _I32, _I32, _I32, _P, _P, _P, _P, _P,
                                   _SZ, _P]),
    "ennx_b200_gqa_attention": (_I32, [_P, _P, _P, _P, _I32, _I32, _I32, _I32, _F32, _P]),
    "ennx_b200_kda_workspace_size": (_SZ, [_I32, _I32, _I32]),
    "ennx_b200_kda_chunked": (_I32, [_P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _P, _SZ, _P]),
    "ennx_b200_kda_chunked_noalloc": (_I32, [_P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _P]),
    "ennx_b200_population_workspace_size": (_SZ, [_P, _I32, _I32]),
    "ennx_b200_population_forward": (_I32, [_P, _P, _U64, _F32, _I32, _I32, _P, _I32, _I32, _P, _P, _SZ, _P]),
    "ennx_b200_population_hidden": (_I32, [_P, _P, _U64, _F32, _I32, _I32, _P, _I32, _I32, _P, _P, _P, _SZ, _P]),
    "ennx_b200_set_perturbation_mode": (_I32, [_I32]),
    "ennx_b200_packed_kda_prefill_workspace_size": (_SZ, [_P, _I32, _I32, _I32]),
    "ennx_b200_packed_kda_prefill": (_I32, [_P, _P, _P, _P, PerturbSeed, _P, _P, _P, _I32, _I32, _I32, _P, _SZ, _P]),
    "ennx_b200_es_coefficients": (_I32, [_P, _I32, _I32, _F32, _F32, _P, _P]),
    "ennx_b200_es_update_bf16": (_I32, [_P, _SZ, _U64, _U32, _P, _U32, _U32, _P]),
    "ennx_b200_population_update": (_I32, [_P, _P, _U64, _P, _I32, _I32, _P]),
    "ennx_b200_l2norm_heads_bf16": (_I32, [_P, ctypes.c_int64, _I32, ctypes.c_int64, _P]),
    "ennx_b200_kda_gate_beta": (_I32, [_P, ctypes.c_int64, _P, ctypes.c_int64, _P, _P, ctypes.c_int64, _I32, _P, _P,
                                       _P]),
    "ennx_b200_kda_postprocess": (_I32, [_P, _P, ctypes.c_int64, _P, ctypes.c_int64, _I32, _F32, _P, _P]),
    "ennx_b200_kda_gated": (_I32, [_P, ctypes.c_int64, _P, ctypes.c_int64, _P, ctypes.c_int64, _P, _P, _P, _P, _I32,
                                   _I32, _I32, _P, _SZ, _P]),
    "ennx_b200_packed_dequantize_bf16": (_I32, [_P, _P, _P, _P, PerturbSeed, _P, _P]),
    "ennx_b200_packed_dequantize_f32": (_I32, [_P, _P, _P, _P, PerturbSeed, _P, _P]),
    "ennx_b200_packed_linear_workspace_size": (_SZ, [_P]),
    "ennx_b200_packed_linear_bf16": (_I32, [_P, ctypes.c_int64, _P, _P, _P, _P, PerturbSeed, _P, _P, _SZ, _P]),
    "ennx_b200_profile_begin": (_I32, []),
    "ennx_b200_profile_end": (_I32, [_P, _I32, _P]),
    "ennx_b200_launch_count": (_U64, []),
}

_lib = None


def lib() -> ctypes.CDLL:
    """Load the in-tree library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise EnnxB200Error(CUDA_ERROR, f"{LIB_PATH} is missing: run `python -m ennx_b200.build`")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name, None)
            if fn is None:
                continue
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int, what: str = "") -> None:
    if status == OK:
        return
    msg = lib().ennx_b200_last_error().decode(errors="replace")
    text = f"{what}: {msg}" if what else msg
    if status in (INVALID_ARGUMENT, OVERFLOW):
        raise EnnxB200ValueError(status, text)
    raise EnnxB200Error(status, text)


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)
