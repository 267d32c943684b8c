"""ctypes binding of libveda_b200.so (the C ABI in include/veda_b200.h).

The library is loaded on first use. There is no fallback: if it is missing
or the device is not an sm_100 GPU, callers get an exception that says so.
"""

from __future__ import annotations

import ctypes
import os
import threading

LIBRARY = os.path.join(os.path.dirname(os.path.abspath(__file__)),
                       'libveda_b200.so')

VEDA_OK = 0
ERR_INVALID, ERR_CUDA, ERR_UNSUPPORTED = 1, 2, 3
STATUS_TIMEOUT = 1
STATUS_BAD_INDEX = 2
STATUS_OVERFLOW = 4
STATUS_BAD_COUNT = 8
STATUS_MISALIGNED = 16
BF16, F16, F32, FP8_E4M3 = 0, 1, 2, 3

_STATUS_NAMES = {STATUS_TIMEOUT: 'a bounded wait timed out',
                 STATUS_BAD_INDEX: 'a tile id was out of range',
                 STATUS_OVERFLOW: 'a row kept more tiles than the list width',
                 STATUS_BAD_COUNT: 'a tile count was out of range',
                 STATUS_MISALIGNED: 'shared memory was misaligned'}


class VedaError(RuntimeError):
    """A C-ABI call failed; `code` is its VEDA_ERR_* value."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


class LibraryMissing(VedaError):
    """libveda_b200.so has not been built."""


class DeviceStatusError(VedaError):
    """A kernel reported an error in the device status word."""


class ColumnBlock(ctypes.Structure):
    """veda_column_block."""

    _fields_ = [('start', ctypes.c_int32), ('stop', ctypes.c_int32),
                ('keeps_all', ctypes.c_int32), ('k_lo', ctypes.c_int32)]


_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64
_F = ctypes.c_float
_U64 = ctypes.c_uint64

# name -> argument types, in the order of include/veda_b200.h
SIGNATURES = {
    'veda_abi_version': [],
    'veda_last_error': [],
    'veda_device_supported': [_I],
    'veda_quantize': [_P, _I, _L, _L, _I, _I, _I, _I, _F, _P, _P, _P],
    'veda_quant_pool': [_P, _P, _I, _L, _L, _I, _I, _P, _I, _F, _P, _P, _P,
                        _P, _P, _P, _P],
    'veda_tile_logits': [_P, _P, _P, _P, _I, _I, _I, _I, _P, _P, _P],
    'veda_tile_logits_scaled': [_P, _P, _P, _P, _I, _P, _P, _I, _I, _I, _P,
                                _P, _P],
    'veda_tile_logits_static': [_P, _P, _P, _P, _I, _I, _I, _I, _P, _P],
    'veda_select': [_P, _L, _L, _I, _I, _I, _P, _I,
                    ctypes.POINTER(ColumnBlock), _P, _I, _P, _P, _P, _P],
    'veda_mask_to_index': [_P, _P, _I, _I, _I, _P, _P, _P, _P],
    'veda_sparse_attention': [_P, _P, _P, _P, _P, _I, _L, _L, _P, _I, _P, _P,
                              _I, _I, _P, _L, _L, _P, _P],
    'veda_sparse_attention_multicast': [_P, _P, _P, _P, _P, _I, _L, _L, _P,
                                        _I, _P, _P, _I, _I, _P, _P, _L, _L,
                                        _P, _P],
    'veda_quant_pool_packed': [_P, _P, _I, _L, _L, _L, _P, _I, _I, _P, _I,
                               _F, _P, _P, _P, _P, _P, _P, _P, _L, _L, _P,
                               _P, _P],
    'veda_sparse_attention_packed': [_P, _P, _P, _P, _P, _I, _L, _L, _P, _I,
                                     _P, _P, _I, _I, _P, _L, _L, _P, _L, _P,
                                     _P, _P],
    'veda_debug_sparse_attention': [_P, _P, _P, _P, _P, _I, _L, _L, _P, _I,
                                    _P, _P, _I, _I, _P, _L, _L, _U64, _I, _P,
                                    _P],
    'veda_gather_tiles': [_P, _I, _L, _L, _I, _I, _P, _I, _P, _I, _P, _P],
    'veda_scatter_tiles': [_P, _I, _P, _I, _P, _I, _I, _P, _L, _L, _I, _P],
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """The loaded library (built in-tree by `python -m veda_b200.build`)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIBRARY):
                raise LibraryMissing(
                    ERR_UNSUPPORTED,
                    f'{LIBRARY} is missing; build it with '
                    '`python -m veda_b200.build` (needs nvcc 12.8+)')
            lib = ctypes.CDLL(LIBRARY)
            for name, args in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = ctypes.c_char_p if name == 'veda_last_error' \
                    else ctypes.c_int
            _lib = lib
    return _lib


def call(name: str, *args) -> None:
    """Calls an entry point and raises VedaError on a non-zero return."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != VEDA_OK:
        message = lib.veda_last_error().decode(errors='replace')
        raise VedaError(rc, f'{name}: {message}')


def describe_status(word: int) -> str:
    return ', '.join(text for bit, text in _STATUS_NAMES.items()
                     if word & bit) or 'ok'
