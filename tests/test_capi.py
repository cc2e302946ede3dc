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


def _prototypes():
    """name -> (return type, [parameter types]) parsed from the header's declarations."""
    text = re.sub(r"/\*.*?\*/|//[^\n]*", " ", open(HEADER).read(), flags=re.S)
    text = re.sub(r"^\s*#.*$", ";", text, flags=re.M)  # preprocessor lines end a declaration
    text = re.sub(r'extern\s+"C"\s*\{|\}', ";", text)
    protos = {}
    for ret, name, params in re.findall(r"(?<=;)\s*([A-Za-z_][\w\s]*?\**)\s*\b(mxfa_[a-z0-9_]+)\s*\(([^)]*)\)\s*;",
                                        text):
        params = " ".join(params.split())
        types = [] if params in ("", "void") else [re.sub(r"\s*\b\w+$", "", a.strip()) for a in params.split(",")]
        protos[name] = (" ".join(ret.split()), types)
    return protos


def _kind(c_type: str) -> str:
    if "*" in c_type:
        return "pointer"
    return {"int": "int", "float": "float", "size_t": "size_t"}[c_type.replace("const ", "").strip()]


def _ctypes_kind(t) -> str:
    if t in (ctypes.c_void_p, ctypes.c_char_p) or hasattr(t, "_type_") and isinstance(t._type_, type):
        return "pointer"
    return {ctypes.c_int: "int", ctypes.c_float: "float", ctypes.c_size_t: "size_t"}[t]


def test_binding_argument_lists_match_the_header_prototypes():
    """Every ctypes signature has the header's parameter count and kinds (pointer / int / float / size_t) and
    return kind, so an argument added on one side only cannot shift the others."""
    protos = _prototypes()
    assert sorted(protos) == declared_symbols()
    for name, (restype, argtypes) in _lib.SIGNATURES.items():
        ret, params = protos[name]
        assert [_kind(p) for p in params] == [_ctypes_kind(a) for a in argtypes], name
        assert _kind(ret) == _ctypes_kind(restype), name


def test_status_codes_and_flags_match_the_header():
    text = open(HEADER).read()
    defines = {k: int(v.rstrip("u"), 0) for k, v in re.findall(r"#define (MXFA_\w+) \(?(-?\w+)\)?", text)
               if re.fullmatch(r"-?(0x[0-9a-fA-F]+|\d+)u?", v)}
    for name in ("MXFA_OK", "MXFA_ERR_UNSUPPORTED", "MXFA_ERR_INVALID", "MXFA_ERR_CUDA"):
        assert getattr(_lib, name) == defines[name], name
    for name in ("PAGE_OUT_OF_RANGE", "TABLE_TOO_NARROW", "WAIT_TIMEOUT", "DENSE_OVERFLOW", "BAD_ORDER"):
        assert getattr(_lib, f"FLAG_{name}") == defines[f"MXFA_FLAG_{name}"], name


def test_integration_guide_names_every_declared_symbol():
    guide = open(os.path.join(os.path.dirname(HEADER), os.pardir, "INTEGRATION.md")).read()
    assert [name for name in declared_symbols() if name not in guide] == []


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


def test_guards_refuse_bad_geometry_and_alignment_before_any_device_work(lib):
    """Every entry refuses, on the host, what its kernels could not address: a zero page size or an
    unaligned operand on the context-parallel decode, query rows past 2^31-1, an unaligned output on
    the prefill (written in 16-byte stores) and unaligned combine operands. The addresses are never
    dereferenced: each call returns before it touches a device."""
    A = 1 << 20  # a 16-byte aligned stand-in address
    inv, uns = _lib.MXFA_ERR_INVALID, _lib.MXFA_ERR_UNSUPPORTED

    def cp(q=A, ps=16, btw=4, pages=10, local=None):
        args = [q, A, A, A, A, A, A, A, 1 << 30, A, A]
        if local is not None:
            args.append(local)
        args += [0, 2, 4, 32, 8, 128, ps, btw, pages, 0, 0, 1, 0.1, None]
        fn = lib.mxfa_cp_attention_launch if local is not None else lib.mxfa_cp_decode_launch
        return fn(*args)

    assert cp(ps=0) == inv
    assert cp(pages=0) == inv
    assert cp(btw=0) == inv
    assert cp(q=A + 8) == inv
    assert cp(local=A + 8) == inv
    rc = lib.mxfa_kvcache_attention_launch(A, A, A, A, A, A, A, A, 1 << 30, 1 << 16, 256, 256, 32, 128, 16, 4, 10,
                                           0, 0, 0, 0, 1, 0.1, None)
    assert rc == uns and b"2^31-1" in lib.mxfa_last_error()
    rc = lib.mxfa_kvcache_attention_launch(A, A, A, A, A, A, A, A, 1 << 30, 1, 1, 32, 8, 128, 4096, 1 << 20, 10,
                                           0, 0, 0, 0, 1, 0.1, None)
    assert rc == uns and b"capacity" in lib.mxfa_last_error()
    rc = lib.mxfa_kvcache_attention_noalloc_launch(A, A, A, A, A, A, A, 1, 1, 32, 8, 128, 4096, 1 << 20, 10, 0, 0,
                                                   0, 0, 1, 0.1, None)
    assert rc == uns and b"capacity" in lib.mxfa_last_error()
    rc = lib.mxfa_varlen_fwd_launch(A, A, A, None, None, A + 8, None, 2, 64, 64, 128, 128, 8, 2, 128, 1, 1, 0.1,
                                    None)
    assert rc == inv and b"aligned" in lib.mxfa_last_error()
    assert lib.mxfa_split_combine_launch(A, A + 2, A, None, None, 4, 128, 2, 1, None) == inv
    assert lib.mxfa_split_combine_launch(A, A, A + 2, None, None, 4, 128, 2, 1, None) == inv
    assert lib.mxfa_lse_merge_launch(A + 2, A, None, 2, 4, 128, 1, None) == inv
    assert lib.mxfa_cp_buffer_bytes(2, 1 << 20, 1 << 12, 8, 128) == 0
    assert lib.mxfa_cp_merge_launch(A, A, None, 2, 1 << 20, 1 << 12, 8, 128, 1, None) == uns


def test_split_plan_invariants(lib):
    """mxfa_kvcache_plan over random shapes: at least one split, chunks a multiple of the 16-token tile, the
    splits cover the cache capacity with no empty trailing split, at most 1024 splits, and one split when the
    capacity is 256 positions or fewer (host-only; the SM count falls back to 148 without a device)."""
    from hypothesis import given, settings
    from hypothesis import strategies as st

    @settings(max_examples=300, deadline=None)
    @given(b=st.integers(1, 4096), sq=st.integers(1, 16), hkv=st.sampled_from([1, 2, 4, 8, 16]),
           gq=st.sampled_from([1, 2, 4, 8]), max_len=st.integers(0, 1 << 20))
    def check(b, sq, hkv, gq, max_len):
        np_, cl = ctypes.c_int(0), ctypes.c_int(0)
        assert lib.mxfa_kvcache_plan(b, sq, hkv * gq, hkv, 128, max_len, ctypes.byref(np_), ctypes.byref(cl)) == 0
        n, c = np_.value, cl.value
        cap = max(max_len, 1)
        assert n >= 1 and c >= 16 and c % 16 == 0
        assert n * c >= cap and (n - 1) * c < cap
        assert n <= 1024
        if cap <= 256:
            assert n == 1
        rows = b * sq * hkv * gq
        assert lib.mxfa_split_workspace_bytes(rows, 128, n) == rows * n * 130 * 4

    check()
