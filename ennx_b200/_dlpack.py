"""DLPack export of a device buffer that this package owns, with a lease.

A buffer exported through ``__dlpack__`` stays leased until its consumer
releases the managed tensor (calls its deleter) or drops an unconsumed
capsule.  The owner refuses to overwrite a leased buffer, which is the
contract of the reference's exports (rust/crates/ennx-py/src/dlpack.rs:318-371,
py_weights.rs:62-66): a JAX or torch array made from a candidate never sees it
change underneath.

Both capsule kinds of the DLPack specification are produced: the versioned
``dltensor_versioned`` (flagged read-only) when the consumer offers
``max_version >= (1, 0)``, the legacy ``dltensor`` otherwise.  The structs
below are the DLPack 1.x C layout (dlpack.h), declared with ctypes.
"""
from __future__ import annotations

import ctypes
from typing import Callable

KDL_CPU, KDL_CUDA = 1, 2
KDL_FLOAT, KDL_BFLOAT = 2, 4
FLAG_READ_ONLY = 1

_LEGACY = b"dltensor"
_VERSIONED = b"dltensor_versioned"


class _Device(ctypes.Structure):
    _fields_ = [("device_type", ctypes.c_int32), ("device_id", ctypes.c_int32)]


class _DType(ctypes.Structure):
    _fields_ = [("code", ctypes.c_uint8), ("bits", ctypes.c_uint8), ("lanes", ctypes.c_uint16)]


class _Tensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("device", _Device), ("ndim", ctypes.c_int32), ("dtype", _DType),
                ("shape", ctypes.POINTER(ctypes.c_int64)), ("strides", ctypes.POINTER(ctypes.c_int64)),
                ("byte_offset", ctypes.c_uint64)]


_DELETER = ctypes.CFUNCTYPE(None, ctypes.c_void_p)


class _Managed(ctypes.Structure):
    _fields_ = [("dl_tensor", _Tensor), ("manager_ctx", ctypes.c_void_p), ("deleter", _DELETER)]


class _Version(ctypes.Structure):
    _fields_ = [("major", ctypes.c_uint32), ("minor", ctypes.c_uint32)]


class _ManagedVersioned(ctypes.Structure):
    _fields_ = [("version", _Version), ("manager_ctx", ctypes.c_void_p), ("deleter", _DELETER),
                ("flags", ctypes.c_uint64), ("dl_tensor", _Tensor)]


assert ctypes.sizeof(_Tensor) == 48 and ctypes.sizeof(_Managed) == 64 and ctypes.sizeof(_ManagedVersioned) == 80

# A private handle on the interpreter's C API: ctypes.pythonapi is shared by
# every module in the process, and others re-declare these prototypes on it.
_api = ctypes.PyDLL(None)
_api.PyCapsule_New.restype = ctypes.py_object
_api.PyCapsule_New.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_void_p]
_api.PyCapsule_IsValid.restype = ctypes.c_int
_api.PyCapsule_IsValid.argtypes = [ctypes.c_void_p, ctypes.c_char_p]
_api.PyCapsule_GetPointer.restype = ctypes.c_void_p
_api.PyCapsule_GetPointer.argtypes = [ctypes.c_void_p, ctypes.c_char_p]

# Everything a live export needs (the managed struct, its shape array, the
# owner object and the release callback), keyed by the managed struct's
# address.  An entry leaves when the export is released, exactly once.
_live: dict[int, tuple] = {}


def _release(address: int) -> None:
    entry = _live.pop(address, None)
    if entry is not None:
        entry[-1]()


@_DELETER
def _deleter(address):
    _release(address)


@ctypes.CFUNCTYPE(None, ctypes.c_void_p)
def _capsule_destructor(capsule):
    # A consumer renames the capsule to "used_..." and owns the release from
    # then on; a capsule still carrying its original name was never consumed.
    for name in (_LEGACY, _VERSIONED):
        if _api.PyCapsule_IsValid(capsule, name):
            _release(_api.PyCapsule_GetPointer(capsule, name))
            return


def live_exports() -> int:
    """Number of exports whose consumer has not released them yet."""
    return len(_live)


def export(owner: object, pointer: int, shape: tuple[int, ...], dtype_code: int, bits: int,
           device: tuple[int, int], release: Callable[[], None],
           max_version: tuple[int, int] | None = None) -> object:
    """Wrap ``pointer`` (contiguous, ``shape``) in a DLPack capsule.

    ``owner`` is kept alive until the consumer releases the tensor, then
    ``release()`` runs once.  If building the capsule fails, ``release()``
    runs before the exception propagates.
    """
    shape_arr = (ctypes.c_int64 * len(shape))(*shape)
    strides = [1] * len(shape)
    for i in range(len(shape) - 2, -1, -1):
        strides[i] = strides[i + 1] * shape[i + 1]
    strides_arr = (ctypes.c_int64 * len(shape))(*strides)
    tensor = _Tensor(ctypes.c_void_p(pointer), _Device(*device), len(shape), _DType(dtype_code, bits, 1),
                     shape_arr, strides_arr, 0)
    if max_version is not None and max_version[0] >= 1:
        minor = min(max_version[1], 3) if max_version[0] == 1 else 3
        managed = _ManagedVersioned(_Version(1, minor), None, _deleter, FLAG_READ_ONLY, tensor)
        name = _VERSIONED
    else:
        managed = _Managed(tensor, None, _deleter)
        name = _LEGACY
    address = ctypes.addressof(managed)
    _live[address] = (managed, shape_arr, strides_arr, owner, release)
    try:
        return _api.PyCapsule_New(ctypes.c_void_p(address), name,
                                  ctypes.cast(_capsule_destructor, ctypes.c_void_p))
    except BaseException:
        _release(address)
        raise
