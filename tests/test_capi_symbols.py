"""The C-ABI library loads and exports every entry point include/*.h declares
(no compute calls: runs without a GPU)."""
import ctypes
import glob
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = []
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        names += re.findall(r"^KRT_API\s+[\w\s\*]+?\b(krt_\w+)\s*\(", open(h).read(), flags=re.M)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = declared_symbols()
    for n in ("krt_qkv_rope_decode", "krt_qkv_rope_prefill", "krt_rowparallel_gemm_ar", "krt_comm_create",
              "krt_allreduce", "krt_last_error", "krt_fused_rmsnorm_qkv_rope"):
        assert n in names


def test_library_exports_every_declared_symbol():
    from python.kinetic_rt import _lib
    if not os.path.exists(_lib.LIB_PATH):
        pytest.skip("libkrt.so not built")
    lib = ctypes.CDLL(_lib.LIB_PATH)
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing
    # every declared symbol also has a ctypes signature in the binding
    assert set(declared_symbols()) <= set(_lib.SIGNATURES)


def test_version_and_error_strings():
    from python.kinetic_rt import _lib
    if not os.path.exists(_lib.LIB_PATH):
        pytest.skip("libkrt.so not built")
    h = _lib.lib()
    assert b"sm_100a" in h.krt_version()
    assert h.krt_comm_destroy(None) == 0   # a successful call clears this thread's message
    assert h.krt_last_error() == b""
