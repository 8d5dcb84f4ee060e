"""CPU: the C-ABI library loads, exports exactly what include/tabby_sample.h declares,
keeps the struct layouts the header documents, and validates arguments before it
touches a device (these calls need no GPU)."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "tabby_sample.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"TABBY_API\s+[\w\s\*]+?\b(tabby_\w+)\s*\(", text)))


def test_header_declares_the_entry_points():
    names = declared_symbols()
    assert len(names) == 24, names
    for n in ("tabby_sampler_create", "tabby_sample_rows_async", "tabby_topk_rows_async",
              "tabby_sample_rows_rng_async", "tabby_softmax_rows_async",
              "tabby_shard_local_async", "tabby_shard_merge_async", "tabby_sample_from_topk",
              "tabby_sample_rows_noalloc", "tabby_last_error", "tabby_sample_rows_debug_async",
              "tabby_exchange_create", "tabby_exchange_merge_async"):
        assert n in names


def test_library_exports_every_declared_symbol():
    from tabby_b200 import _lib

    L = _lib.lib()
    for name in declared_symbols():
        assert hasattr(L, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (tabby_\w+)", out))
    assert exported == set(declared_symbols()), exported ^ set(declared_symbols())


def test_struct_layouts():
    from tabby_b200 import _lib

    assert _lib.PARAMS_DTYPE.itemsize == 24
    assert _lib.OUTCOME_DTYPE.itemsize == 48
    assert ctypes.sizeof(_lib.SamplerConfig) == 16
    from oracle import oracle as o

    assert o.PARAMS_DTYPE == _lib.PARAMS_DTYPE
    assert o.OUTCOME_DTYPE == _lib.OUTCOME_DTYPE


def test_abi_version_and_pool_size():
    from tabby_b200 import _lib

    L = _lib.lib()
    assert L.tabby_abi_version() == 1
    assert L.tabby_pool_size(0.0, 40, 64) == 1
    assert L.tabby_pool_size(0.8, 0, 1024) == 1024


def test_argument_errors_without_a_device():
    from tabby_b200 import _lib

    L = _lib.lib()
    # A NULL config is rejected before any CUDA call.
    h = ctypes.c_void_p()
    assert L.tabby_sampler_create(None, ctypes.byref(h)) == _lib.TABBY_EINVAL
    assert L.tabby_last_error()
    # Caps beyond 1024 (TABBY_MAX_TOP_K_LIMIT) are rejected like forward.ts:348-351.
    cfg = _lib.SamplerConfig(0, 1025, 8, 1000)
    assert L.tabby_sampler_create(ctypes.byref(cfg), ctypes.byref(h)) == _lib.TABBY_EINVAL
    # Handle-free entry point: sizes beyond its fixed scratch are refused up front.
    rc = L.tabby_sample_rows_noalloc(ctypes.c_void_p(16), 100, 1, 100,
                                     _lib.TABBY_NOALLOC_MAX_TOP_K + 1, ctypes.c_void_p(16),
                                     ctypes.c_void_p(16), ctypes.c_void_p(16), None, None, 0,
                                     None)
    assert rc == _lib.TABBY_EINVAL and b"limit" in L.tabby_last_error()
    # Zero rows is a no-op.
    assert L.tabby_sample_rows_noalloc(None, 100, 0, 100, 64, None, None, None, None, None, 0,
                                       None) == _lib.TABBY_OK
    # Row softmax: shapes the shader would read past are refused before any CUDA call.
    assert L.tabby_softmax_rows_async(ctypes.c_void_p(16), 4, 8, 4, 5, None) == _lib.TABBY_EINVAL
    assert L.tabby_softmax_rows_async(ctypes.c_void_p(16), 4, 0, 0, 0, None) == _lib.TABBY_EINVAL
    assert L.tabby_softmax_rows_async(None, 0, 8, 0, 0, None) == _lib.TABBY_OK
    # Device-RNG entry point: a NULL handle is refused before any CUDA call.
    rc = L.tabby_sample_rows_rng_async(None, ctypes.c_void_p(16), 100, 1, 100,
                                       ctypes.c_void_p(16), ctypes.c_void_p(16),
                                       ctypes.c_void_p(16), None, None, 0, None)
    assert rc == _lib.TABBY_EINVAL and b"NULL" in L.tabby_last_error()


def test_sampler_create_without_gpu_fails_cleanly():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from tabby_b200 import Sampler
    from tabby_b200._lib import TabbyError

    with pytest.raises(TabbyError):
        Sampler(0, max_top_k=64, max_rows=4, max_vocab=1000)


def test_host_sample_from_topk_errors():
    from tabby_b200 import _lib

    L = _lib.lib()
    out = np.zeros(1, _lib.OUTCOME_DTYPE)
    p = np.zeros(1, _lib.PARAMS_DTYPE)
    ids = np.zeros(1, np.int32)
    vals = np.zeros(1, np.float32)
    rc = L.tabby_sample_from_topk(ids.ctypes.data, vals.ctypes.data, 0, 0.0, 1.0, p.ctypes.data,
                                  0.5, out.ctypes.data)
    assert rc == _lib.TABBY_EEMPTY
    assert b"empty candidate set" in L.tabby_last_error()


def test_product_never_imports_the_oracle():
    pkg = os.path.join(ROOT, "tabby_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h", ".cpp")):
                text = open(os.path.join(dirpath, f), errors="replace").read()
                assert "oracle" not in re.sub(r"#.*|//.*", "", text).lower() or f == "__init__.py", f


def test_exchange_rejects_bad_arguments_before_touching_the_device():
    """tabby_exchange_create validates world, rank and max_rows first (no GPU needed)."""
    import ctypes

    from tabby_b200 import _lib

    L = _lib.lib()
    h = ctypes.c_void_p()
    for world, rank, rows in ((0, 0, 8), (17, 0, 8), (2, 2, 8), (2, -1, 8), (2, 0, 0)):
        assert L.tabby_exchange_create(0, world, rank, rows, ctypes.byref(h)) == _lib.TABBY_EINVAL
        assert h.value is None
    assert L.tabby_exchange_create(0, 1, 0, 8, None) == _lib.TABBY_EINVAL
    assert L.tabby_exchange_merge_async(None, 1, None, None, None, None) == _lib.TABBY_EINVAL
    assert b"exchange" in L.tabby_last_error()
    assert L.tabby_exchange_destroy(None) == _lib.TABBY_OK
