"""ctypes binding of libtabbysample.so (include/tabby_sample.h).

The library is the product: there is no Python or CPU fallback. If the shared object is
missing or fails to load, ``lib()`` raises.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "lib", "libtabbysample.so")

TABBY_OK = 0
TABBY_EINVAL = 1
TABBY_ECUDA = 2
TABBY_ENOMEM = 3
TABBY_EINPUT = 4
TABBY_ETIMEOUT = 5
TABBY_EEMPTY = 6
TABBY_MAX_TOP_K_LIMIT = 1024
TABBY_DEFAULT_MAX_TOP_K = 64
TABBY_SHARD_TOP_K = 64
TABBY_NOALLOC_MAX_TOP_K = 256
TABBY_EXCHANGE_MAX_WORLD = 16
TABBY_EXCHANGE_HANDLE_BYTES = 64
SHARD_BLOCK_WORDS = 2 + 2 * TABBY_SHARD_TOP_K

# tabby_sampling_params (24 bytes) and tabby_sample_outcome (48 bytes).
PARAMS_DTYPE = np.dtype(
    [("temperature", "<f8"), ("top_p", "<f8"), ("top_k", "<i4"), ("reserved", "<i4")]
)
OUTCOME_DTYPE = np.dtype(
    [
        ("id", "<i4"),
        ("considered_count", "<i4"),
        ("probability", "<f8"),
        ("pool_mass", "<f8"),
        ("pool_exhausted", "<i4"),
        ("pool_size", "<i4"),
        ("max_logit", "<f4"),
        ("sum_exp", "<f4"),
        ("status", "<i4"),
        ("reserved", "<i4"),
    ]
)
assert PARAMS_DTYPE.itemsize == 24 and OUTCOME_DTYPE.itemsize == 48


class SamplerConfig(ctypes.Structure):
    _fields_ = [
        ("device", ctypes.c_int32),
        ("max_top_k", ctypes.c_int32),
        ("max_rows", ctypes.c_int32),
        ("max_vocab", ctypes.c_int32),
    ]


# Every symbol include/tabby_sample.h declares, with its ctypes signature.
_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_F32 = ctypes.c_float
_F64 = ctypes.c_double
SIGNATURES = {
    "tabby_abi_version": ([], _I32),
    "tabby_last_error": ([], ctypes.c_char_p),
    "tabby_pool_size": ([_F64, _I32, _I32], _I32),
    "tabby_sampler_create": ([ctypes.POINTER(SamplerConfig), ctypes.POINTER(_P)], ctypes.c_int),
    "tabby_sampler_destroy": ([_P], ctypes.c_int),
    "tabby_sample_rows_async": (
        [_P, _P, _I64, _I32, _I32, _P, _P, _P, _P, _P, _I32, _P], ctypes.c_int),
    "tabby_softmax_rows_async": ([_P, _I32, _I32, _I32, _I32, _P], ctypes.c_int),
    "tabby_sample_rows_rng_async": (
        [_P, _P, _I64, _I32, _I32, _P, _P, _P, _P, _P, _I32, _P], ctypes.c_int),
    "tabby_sample_rows_debug_async": (
        [_P, _P, _I64, _I32, _I32, _P, _P, _P, ctypes.c_uint32, _I32, _P], ctypes.c_int),
    "tabby_lmhead_create": ([_I32, _I32, _I32, _I32, ctypes.POINTER(_P)], ctypes.c_int),
    "tabby_lmhead_destroy": ([_P], ctypes.c_int),
    "tabby_lmhead_sample_async": (
        [_P, _P, _P, _I32, _P, _P, _P, _P, _P, _I32, _P, _P], ctypes.c_int),
    "tabby_sample_rows": ([_P, _P, _I64, _I32, _I32, _P, _P, _P, _P, _P, _I32], ctypes.c_int),
    "tabby_topk_rows_async": ([_P, _P, _I64, _I32, _I32, _I32, _P, _I32, _P], ctypes.c_int),
    "tabby_shard_local_async": ([_P, _P, _I64, _I32, _I32, _I64, _P, _I32, _P], ctypes.c_int),
    "tabby_shard_merge_async": (
        [_P, _P, _I32, _I32, _I32, _P, _P, _P, _P, _P, _I32, _P], ctypes.c_int),
    "tabby_exchange_create": ([_I32, _I32, _I32, _I32, ctypes.POINTER(_P)], ctypes.c_int),
    "tabby_exchange_ipc_handle": ([_P, _P], ctypes.c_int),
    "tabby_exchange_open": ([_P, _P], ctypes.c_int),
    "tabby_exchange_blocks": ([_P, ctypes.POINTER(_P), ctypes.POINTER(_I32)], ctypes.c_int),
    "tabby_exchange_merge_async": ([_P, _I32, _P, _P, _P, _P], ctypes.c_int),
    "tabby_exchange_destroy": ([_P], ctypes.c_int),
    "tabby_sample_from_topk": ([_P, _P, _I32, _F32, _F32, _P, _F64, _P], ctypes.c_int),
    "tabby_sample_rows_noalloc": (
        [_P, _I64, _I32, _I32, _I32, _P, _P, _P, _P, _P, _I32, _P], ctypes.c_int),
}

_lib = None


class TabbyError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"[tabby status {status}] {message}")
        self.status = status


def lib() -> ctypes.CDLL:
    """Load the shared library (raises if it is missing: no fallback exists)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing; build it with `python -m tabby_b200.build`"
            )
        l = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(l, name)
            fn.argtypes = args
            fn.restype = res
        _lib = l
    return _lib


def check(status: int) -> None:
    if status != TABBY_OK:
        raise TabbyError(status, lib().tabby_last_error().decode(errors="replace"))
