"""ennx_b200 -- B200-native (sm_100a) model-evaluation hot path of ENNX.

The compute lives in the CUDA library ``ennx_b200/_lib/libennx_b200.so``
behind the C ABI of ``include/ennx_b200.h``; this package is the thin host
side that mirrors the reference's ``ennx.experimental`` operator surface.
"""
from ._abi import EnnxB200Error, EnnxB200ValueError, lib  # noqa: F401

__version__ = "0.1.0"
