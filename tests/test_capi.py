"""The C-ABI library loads on a CPU host and exports every declared entry point.

No compute runs here: only the host-side guards that return before any
device work (unsupported configurations, bad arguments) are exercised.
"""

from __future__ import annotations

import ctypes
import os
import re

import pytest

from mxflashattn_b200 import _lib, build

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "mxfa_b200.h")


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(mxfa_[a-z0-9_]+)\s*\(", text)))


def test_header_and_binding_agree():
    assert declared_symbols() == sorted(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_abi_version_and_error_string(lib):
    assert lib.mxfa_abi_version() == 1
    assert isinstance(lib.mxfa_last_error(), bytes)


@pytest.mark.parametrize("hq,hkv,d,np_", [(12, 4, 128, 2), (8, 4, 96, 2), (8, 3, 128, 1), (8, 4, 128, 0),
                                          (32, 2, 64, 1)])
def test_reference_split_entry_guards_match_reference(lib, hq, hkv, d, np_):
    """D in {64,128}, HQ % HKV == 0, GQ in {2,4,8}, NP >= 1 -> else -1 (m1_kernel.cpp:1212-1215)."""
    rc = lib.mxfa_paged_decode_split_launch(None, None, None, None, None, None, None, None, 0.1, 1, hq, hkv, d,
                                            16, 4, 1, np_, 16, 2, None)
    assert rc == _lib.MXFA_ERR_UNSUPPORTED
    assert "unsupported" in lib.mxfa_last_error().decode() or "HQ" in lib.mxfa_last_error().decode()


def test_invalid_arguments_return_invalid(lib):
    rc = lib.mxfa_kvcache_attention_launch(None, None, None, None, None, None, None, None, 0, 1, 1, 8, 2, 128, 16,
                                           4, 10, 0, 0, 0, 0, 1, 0.1, None)
    assert rc == _lib.MXFA_ERR_INVALID
    rc = lib.mxfa_varlen_fwd_launch(None, None, None, None, None, None, None, 1, 4, 4, 4, 4, 8, 2, 80, 1, 1, 0.1,
                                    None)
    assert rc == _lib.MXFA_ERR_UNSUPPORTED


def test_workspace_and_plan_are_host_only(lib):
    assert lib.mxfa_split_workspace_bytes(10, 128, 3) == 10 * 3 * 130 * 4
    assert lib.mxfa_split_workspace_bytes(0, 128, 3) == 0
    np_, cl = ctypes.c_int(0), ctypes.c_int(0)
    assert lib.mxfa_kvcache_plan(1, 1, 32, 8, 128, 16384, ctypes.byref(np_), ctypes.byref(cl)) == 0
    assert np_.value > 1 and cl.value % 16 == 0 and np_.value * cl.value >= 16384
    assert lib.mxfa_kvcache_plan(128, 1, 32, 8, 128, 1280, ctypes.byref(np_), ctypes.byref(cl)) == 0
    assert np_.value == 1 and cl.value >= 1280


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(_lib.NativeLibraryError, match="not built"):
        _lib.load(str(tmp_path / "libmxfa_b200.so"))
