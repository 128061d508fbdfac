"""The C-ABI library loads, exports every symbol include/b200tx.h declares, and rejects bad
arguments before touching a device (no GPU needed: no compute call is made)."""

import ctypes
import re
from pathlib import Path

import pytest

from tiktoktechjam2026track3_b200 import _capi
from tiktoktechjam2026track3_b200.build import LIB_PATH, build

HEADER = Path(__file__).resolve().parents[1] / "include" / "b200tx.h"


@pytest.fixture(scope="module")
def lib():
    build()
    return _capi.load_library()


def declared_symbols():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(b2_\w+)\s*\(", text)))


def test_header_declares_bound_symbols():
    assert declared_symbols() == sorted(_capi.SIGNATURES)


def test_library_exports_every_declared_symbol(lib):
    raw = ctypes.CDLL(str(LIB_PATH))
    for name in declared_symbols():
        assert hasattr(raw, name), name


def test_abi_version(lib):
    assert lib.b2_abi_version() == 1


def test_linear_rejects_null_and_bad_shapes(lib):
    s = lib.b2_linear_fwd(None, None, None, 128, 128, 64, 0, None, 128, None, 0, None)
    assert s == 1
    assert b"null" in lib.b2_last_error()
    p = ctypes.c_void_p(16)
    assert lib.b2_linear_fwd(p, p, p, 128, 100, 64, 0, p, 128, None, 0, None) == 2
    assert b"multiple of 32" in lib.b2_last_error()
    assert lib.b2_linear_fwd(p, p, p, 128, 128, 60, 0, p, 128, None, 0, None) == 2
    assert lib.b2_linear_fwd(p, p, p, 128, 128, 64, 9, p, 128, None, 0, None) == 1
    assert lib.b2_linear_fwd(p, p, p, 128, 128, 64, 0, p, 128, None, 64, None) == 1
    assert lib.b2_linear_fwd(ctypes.c_void_p(8), p, p, 128, 128, 64, 0, p, 128, None, 0, None) == 2
    assert b"aligned" in lib.b2_last_error()


def test_attention_rejects_unsupported_head_dim(lib):
    p = ctypes.c_void_p(16)
    assert lib.b2_attention_fwd(p, 144, 0, 48, 96, 1, 8, 1, 48, None, 1, 0.1, p, 48, None) == 2
    assert b"head_dim" in lib.b2_last_error()
    # CUDA-core head dims need 8-element column alignment, tensor-core ones 64
    assert lib.b2_attention_fwd(p, 96, 0, 36, 64, 1, 8, 1, 32, None, 1, 0.1, p, 32, None) == 2
    assert b"multiples of 8" in lib.b2_last_error()
    assert lib.b2_attention_fwd(p, 192, 0, 32, 128, 1, 8, 1, 64, None, 1, 0.1, p, 64, None) == 2
    assert lib.b2_attention_fwd(None, 192, 0, 64, 128, 1, 8, 1, 64, None, 1, 0.1, p, 64, None) == 1


def test_layernorm_rejects_bad_arguments(lib):
    p = ctypes.c_void_p(16)
    assert lib.b2_layernorm_fwd(None, 0, p, p, 1e-5, p, None, None, 4, 8, None) == 1
    assert lib.b2_layernorm_fwd(p, 0, p, p, 0.0, p, None, None, 4, 8, None) == 1
    assert lib.b2_layernorm_fwd(p, 0, p, p, 1e-5, p, None, None, 0, 8, None) == 0  # empty is a no-op


def test_linear_ln_plan_depends_on_n_only(lib):
    for m in (1, 4096, 100000):
        assert _capi.linear_ln_plan(m, 768, 768, sm_count=148) == (192, 4, False)
    assert _capi.linear_ln_plan(4096, 1024, 4096, sm_count=148) == (256, 4, False)
    assert _capi.linear_ln_plan(4096, 2048, 8192, sm_count=148) == (256, 8, False)
    assert _capi.linear_ln_plan(64, 96, 64, sm_count=148) == (128, 1, False)
    assert _capi.linear_ln_plan(64, 640, 64, sm_count=148) == (128, 5, False)
    assert _capi.linear_ln_plan(64, 2560, 64, sm_count=148) is None  # 10 CTAs per row
    assert _capi.linear_ln_plan(64, 48, 64, sm_count=148) is None


def test_linear_ln_rejects_bad_arguments(lib):
    p = ctypes.c_void_p(16)
    f = lib.b2_linear_ln_fwd
    assert f(None, p, p, 128, 768, 768, 0, p, None, p, p, 1e-5, p, None) == 1
    assert f(p, p, p, 128, 768, 768, 0, p, None, p, p, 0.0, p, None) == 1
    assert f(p, p, p, 128, 2560, 768, 0, p, None, p, p, 1e-5, p, None) == 2
    assert b"plan" in lib.b2_last_error()
    assert f(p, p, p, 128, 768, 60, 0, p, None, p, p, 1e-5, p, None) == 2
    assert f(ctypes.c_void_p(8), p, p, 128, 768, 768, 0, p, None, p, p, 1e-5, p, None) == 2
    assert b"aligned" in lib.b2_last_error()
    assert f(p, p, p, 0, 768, 768, 0, p, None, p, p, 1e-5, p, None) == 0  # empty is a no-op
