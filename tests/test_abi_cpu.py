"""CPU-side checks of the drop-in boundary: the library loads and exports
every entry point that include/*.h declares (no compute without a GPU)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(ennx_b200_\w+)\s*\(", text))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    from ennx_b200 import _abi
    lib = _abi.lib()
    names = declared_symbols()
    assert len(names) >= 10
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_abi_version_and_error_string():
    from ennx_b200 import _abi
    assert _abi.lib().ennx_b200_abi_version() == 1
    assert isinstance(_abi.lib().ennx_b200_last_error(), bytes)


def test_python_signatures_cover_header():
    from ennx_b200 import _abi
    assert set(declared_symbols()) <= set(_abi.SIGNATURES), set(declared_symbols()) - set(_abi.SIGNATURES)


def test_invalid_arguments_rejected_without_gpu():
    from ennx_b200 import _abi
    lib = _abi.lib()
    # null pointers are rejected on the host before any CUDA call
    st = lib.ennx_b200_dense_apply_f32(None, 0, None, 0, None, 0, None, None, None)
    assert st == _abi.INVALID_ARGUMENT
    assert b"empty" in lib.ennx_b200_last_error()
    p = _abi.GemmParams(m=128, n=128, k=100, lda=100, ldb=100, ldc=128, groups=1)
    st = lib.ennx_b200_gemm_bf16(ctypes.byref(p), ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), None)
    assert st == _abi.UNSUPPORTED and b"multiple of 64" in lib.ennx_b200_last_error()


def test_search_and_decoder_reject_bad_arguments_on_the_host():
    from ennx_b200 import _abi
    lib = _abi.lib()
    h = ctypes.c_void_p()
    leaves = (_abi.Bf16Leaf * 2)(_abi.Bf16Leaf(1, 0, 4, 1.0, 1.0), _abi.Bf16Leaf(2, 5, 4, 1.0, 1.0))
    st = lib.ennx_b200_bf16_search_create(None, 8, leaves, 2, 4, None, ctypes.byref(h))
    assert st == _abi.INVALID_ARGUMENT and b"requires a device base" in lib.ennx_b200_last_error()
    st = lib.ennx_b200_bf16_search_create(ctypes.c_void_p(16), 8, leaves, 2, 4, None, ctypes.byref(h))
    assert st == _abi.INVALID_ARGUMENT and b"contiguous non-empty layout" in lib.ennx_b200_last_error()
    st = lib.ennx_b200_bf16_search_create(ctypes.c_void_p(16), 8, leaves, 2, 1, None, ctypes.byref(h))
    assert st == _abi.INVALID_ARGUMENT and b"at least two row slots" in lib.ennx_b200_last_error()
    assert not h.value

    cfg = _abi.KdaDecoderConfig(2, 256, 2, 100, 16, 8, 2, 64, 0.5, 1e-6, 1.0)
    lin = _abi.PackedLinear(0, 0, 0, 256, 1, 8, 64, 0, 0, 0)
    layers = (_abi.KdaDecoderLayer * 2)()
    buf = (ctypes.c_uint8 * 16)()
    fl = (ctypes.c_float * 4)()
    args = (buf, 16, fl, 4, fl, 4)
    st = lib.ennx_b200_kda_decoder_create(*args, ctypes.byref(cfg), layers, ctypes.byref(lin), ctypes.byref(lin),
                                          None, ctypes.byref(h))
    assert st == _abi.INVALID_ARGUMENT and b"heads x head width" in lib.ennx_b200_last_error()
    cfg.head_width, cfg.top_k = 128, 9
    st = lib.ennx_b200_kda_decoder_create(*args, ctypes.byref(cfg), layers, ctypes.byref(lin), ctypes.byref(lin),
                                          None, ctypes.byref(h))
    assert st == _abi.INVALID_ARGUMENT and b"top_k must be in 1..=8" in lib.ennx_b200_last_error()
    cfg.top_k, cfg.num_layers = 2, 0
    st = lib.ennx_b200_kda_decoder_create(*args, ctypes.byref(cfg), layers, ctypes.byref(lin), ctypes.byref(lin),
                                          None, ctypes.byref(h))
    assert st == _abi.INVALID_ARGUMENT and b"has no layers" in lib.ennx_b200_last_error()
    assert not h.value
