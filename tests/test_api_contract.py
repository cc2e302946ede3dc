"""Public API and dispatch contract on the CPU (no GPU): guards, errors, records.

Mirrors the reference's CPU suite (tests/test_api.py, tests/test_dispatch.py)
for everything that does not compute: validation runs before dispatch, and
dispatch either records the CUDA backend or raises BackendUnavailableError
with the reason.  The reference's CPU fallback is intentionally absent.
"""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

import mxflashattn_b200.dispatch as dispatch
from mxflashattn_b200 import (
    BackendUnavailableError,
    flash_attn_func,
    flash_attn_varlen_func,
    flash_attn_with_kvcache,
    get_last_dispatch_info,
)


def tensors(batch=1, q_len=2, kv_len=3, q_heads=2, kv_heads=1, head_dim=64, dtype=torch.float16):
    q = torch.randn(batch, q_len, q_heads, head_dim).to(dtype)
    k = torch.randn(batch, kv_len, kv_heads, head_dim).to(dtype)
    return q, k, torch.randn_like(k)


def test_cpu_tensors_raise_with_actionable_reason(monkeypatch):
    q, k, v = tensors()
    monkeypatch.delenv("MXFLASHATTN_ALLOW_FALLBACK", raising=False)
    with pytest.raises(BackendUnavailableError, match="native_backend_requires_accelerator_tensor"):
        flash_attn_func(q, k, v)
    assert get_last_dispatch_info() is None


def test_allow_fallback_is_reported_as_ignored(monkeypatch):
    q, k, v = tensors()
    monkeypatch.setenv("MXFLASHATTN_ALLOW_FALLBACK", "1")
    with pytest.raises(BackendUnavailableError, match="no CPU reference path"):
        flash_attn_func(q, k, v, causal=True)


def test_varlen_rejects_cumulative_lengths_that_do_not_cover_tokens():
    q = torch.randn(2, 1, 64)
    k = torch.randn(2, 1, 64)
    cu = torch.tensor([0, 1], dtype=torch.int32)
    with pytest.raises(ValueError, match="cover all tokens"):
        flash_attn_varlen_func(q, k, k, cu, cu, max_seqlen_q=1, max_seqlen_k=1)


def test_varlen_rejects_empty_key_sequences():
    q = torch.randn(2, 1, 64)
    k = torch.randn(1, 1, 64)
    cu_q = torch.tensor([0, 1, 2], dtype=torch.int32)
    cu_k = torch.tensor([0, 0, 1], dtype=torch.int32)
    with pytest.raises(ValueError, match="key/value sequences must be non-empty"):
        flash_attn_varlen_func(q, k, k, cu_q, cu_k, max_seqlen_q=1, max_seqlen_k=1)


def test_varlen_rejects_cumulative_lengths_on_a_different_device():
    q = torch.randn(1, 1, 64)
    k = torch.randn(1, 1, 64)
    cu = torch.tensor([0, 1], device="meta", dtype=torch.int32)
    with pytest.raises(ValueError, match="same device as q"):
        flash_attn_varlen_func(q, k, k, cu, cu, max_seqlen_q=1, max_seqlen_k=1)


def test_varlen_rejects_sequence_longer_than_max():
    q = torch.randn(3, 2, 64)
    cu = torch.tensor([0, 3], dtype=torch.int32)
    with pytest.raises(ValueError, match="longer than max_seqlen"):
        flash_attn_varlen_func(q, q[:, :1], q[:, :1], cu, cu, max_seqlen_q=2, max_seqlen_k=3)


def test_kvcache_rejects_zero_page_size():
    q = torch.randn(1, 1, 1, 64)
    k_cache = torch.empty(1, 0, 1, 64)
    with pytest.raises(ValueError, match="page size must be positive"):
        flash_attn_with_kvcache(q, k_cache, torch.empty_like(k_cache),
                                cache_seqlens=torch.tensor([1], dtype=torch.int32),
                                block_table=torch.tensor([[0]], dtype=torch.int32))


@pytest.mark.parametrize("kwargs,exc,match", [
    ({"rotary_cos": torch.zeros(1)}, NotImplementedError, "rotary"),
    ({"return_softmax_lse": True}, NotImplementedError, "return_softmax_lse"),
    ({"window_size": (4, 0)}, NotImplementedError, "local window"),
    ({"softcap": 1.0}, NotImplementedError, "soft-capping"),
    ({"alibi_slopes": torch.zeros(2)}, NotImplementedError, "alibi"),
    ({"cache_seqlens": None}, ValueError, "cache_seqlens is required"),
    ({"cache_seqlens": torch.tensor([1.0])}, TypeError, "int32 or int64"),
    ({"block_table": torch.tensor([[0.0]])}, TypeError, "int32 or int64"),
    ({"softmax_scale": float("inf")}, ValueError, "softmax_scale must be finite"),
])
def test_kvcache_guards(kwargs, exc, match):
    q = torch.randn(1, 1, 2, 64, dtype=torch.float16)
    kc = torch.randn(2, 16, 1, 64, dtype=torch.float16)
    args = {"cache_seqlens": torch.tensor([3], dtype=torch.int32), "block_table": torch.tensor([[0]], dtype=torch.int32)}
    args.update(kwargs)
    with pytest.raises(exc, match=match):
        flash_attn_with_kvcache(q, kc, kc.clone(), **args)


def test_kvcache_rejects_k_without_v():
    q = torch.randn(1, 1, 2, 64)
    kc = torch.randn(1, 4, 1, 64)
    with pytest.raises(ValueError, match="both be provided"):
        flash_attn_with_kvcache(q, kc, kc, k=torch.randn(1, 1, 1, 64), cache_seqlens=torch.tensor([1]))


def test_unsupported_flash_attention_options_fail_clearly():
    q, k, v = tensors()
    with pytest.raises(NotImplementedError, match="dropout"):
        flash_attn_func(q, k, v, dropout_p=0.1)
    with pytest.raises(NotImplementedError, match="deterministic"):
        flash_attn_func(q, k, v, deterministic=True)


def test_head_dim_and_gqa_guards():
    q, k, v = tensors(head_dim=96)
    with pytest.raises(ValueError, match="head dimension"):
        flash_attn_func(q, k, v)
    q, k, v = tensors(q_heads=3, kv_heads=2)
    with pytest.raises(ValueError, match="divisible"):
        flash_attn_func(q, k, v)


def test_nan_scale_is_rejected():
    q, k, v = tensors()
    with pytest.raises(ValueError, match="softmax_scale must be finite"):
        flash_attn_func(q, k, v, softmax_scale=float("nan"))


def _cuda_like(dtype=torch.float16):
    return SimpleNamespace(device=SimpleNamespace(type="cuda"), dtype=dtype)


def test_dispatch_records_cuda_backend_with_a_fake_extension(monkeypatch):
    calls = []
    ext = SimpleNamespace(is_available=lambda: True,
                          flash_attn_func=lambda *args: calls.append(args) or "result")
    monkeypatch.setattr(dispatch, "_native_extension", lambda: ext)
    tensor = _cuda_like()
    assert dispatch.dispatch("flash_attn_func", tensor, (tensor, 0.0)) == "result"
    assert calls == [(tensor, 0.0)]
    info = dispatch.get_last_dispatch_info()
    assert info.backend == "cuda_sm100" and info.operation == "flash_attn_func" and info.fallback_reason is None


@pytest.mark.parametrize("ext,reason", [
    (None, "native_extension_not_built_or_not_importable"),
    (SimpleNamespace(is_available=lambda: False), "native_extension_reports_unavailable_runtime"),
    (SimpleNamespace(is_available=lambda: True), "native_extension_does_not_implement_flash_attn_func"),
])
def test_dispatch_reasons(monkeypatch, ext, reason):
    monkeypatch.setattr(dispatch, "_native_extension", lambda: ext)
    assert dispatch.native_unavailable_reason(_cuda_like(), "flash_attn_func") == reason
    with pytest.raises(BackendUnavailableError, match=reason):
        dispatch.dispatch("flash_attn_func", _cuda_like(), ())


def test_dispatch_rejects_float32_before_touching_the_extension(monkeypatch):
    monkeypatch.setattr(dispatch, "_native_extension", lambda: pytest.fail("must not import"))
    assert dispatch.native_unavailable_reason(_cuda_like(torch.float32), "flash_attn_func") == (
        "native_backend_supports_only_float16_and_bfloat16")


def test_native_library_failure_becomes_backend_unavailable(monkeypatch):
    from mxflashattn_b200._lib import NativeLibraryError

    def boom(*args):
        raise NativeLibraryError("mxfa_varlen_fwd_launch: unsupported configuration: head dim")

    ext = SimpleNamespace(is_available=lambda: True, flash_attn_func=boom)
    monkeypatch.setattr(dispatch, "_native_extension", lambda: ext)
    with pytest.raises(BackendUnavailableError, match="native_call_failed"):
        dispatch.dispatch("flash_attn_func", _cuda_like(), ())


def test_availability_check_failure_is_reported(monkeypatch):
    def broken():
        raise OSError("driver gone")

    monkeypatch.setattr(dispatch, "_native_extension", lambda: SimpleNamespace(is_available=broken))
    assert dispatch.native_unavailable_reason(_cuda_like(), "flash_attn_func").startswith(
        "native_availability_check_failed:OSError")


# ------------------------------------------------ FP8 (e4m3) cache extension

def _fp8_paged(head_dim=128, q_dtype=torch.bfloat16):
    q = torch.randn(2, 1, 4, head_dim).to(q_dtype)
    kc = torch.randn(6, 16, 2, head_dim).to(torch.float8_e4m3fn)
    vc = torch.randn(6, 16, 2, head_dim).to(torch.float8_e4m3fn)
    return q, kc, vc, torch.tensor([3, 5], dtype=torch.int32), torch.zeros((2, 3), dtype=torch.int32)


@pytest.mark.parametrize("kwargs,match", [
    (dict(k_scale=0.0), "k_scale must be a positive finite number"),
    (dict(v_scale=float("nan")), "v_scale must be a positive finite number"),
])
def test_fp8_cache_rejects_bad_scales(kwargs, match):
    q, kc, vc, sl, bt = _fp8_paged()
    with pytest.raises(ValueError, match=match):
        flash_attn_with_kvcache(q, kc, vc, cache_seqlens=sl, block_table=bt, **kwargs)


def test_fp8_cache_guards():
    q, kc, vc, sl, bt = _fp8_paged(head_dim=64)
    with pytest.raises(ValueError, match="head dimension 128"):
        flash_attn_with_kvcache(q, kc, vc, cache_seqlens=sl, block_table=bt)
    q, kc, vc, sl, bt = _fp8_paged(q_dtype=torch.float32)
    with pytest.raises(TypeError, match="float16 or bfloat16 query"):
        flash_attn_with_kvcache(q, kc, vc, cache_seqlens=sl, block_table=bt)
    q, kc, vc, sl, bt = _fp8_paged()
    with pytest.raises(ValueError, match="same dtype"):
        flash_attn_with_kvcache(q, kc, vc.to(torch.bfloat16), cache_seqlens=sl, block_table=bt)
    k_new = torch.randn(2, 1, 2, 128).to(torch.bfloat16)
    with pytest.raises(ValueError, match="must be float8_e4m3fn"):
        flash_attn_with_kvcache(q, kc, vc, k=k_new, v=k_new, cache_seqlens=sl, block_table=bt)


def test_scales_are_rejected_for_16_bit_caches():
    q, k, v = tensors(head_dim=128)
    with pytest.raises(ValueError, match="float8_e4m3fn caches only"):
        flash_attn_with_kvcache(q, k, v, cache_seqlens=torch.tensor([3], dtype=torch.int32), k_scale=0.5)


def test_fp8_scales_reach_the_backend(monkeypatch):
    calls = []
    ext = SimpleNamespace(is_available=lambda: True,
                          flash_attn_with_kvcache=lambda *args: calls.append(args) or "result")
    monkeypatch.setattr(dispatch, "_native_extension", lambda: ext)
    monkeypatch.setattr(dispatch, "native_unavailable_reason", lambda tensor, op: None)
    q, kc, vc, sl, bt = _fp8_paged()
    assert flash_attn_with_kvcache(q, kc, vc, cache_seqlens=sl, block_table=bt, k_scale=0.5, v_scale=2.0) == "result"
    assert calls[0][-2:] == (0.5, 2.0)


def test_out_buffer_is_validated_and_passed_to_the_backend(monkeypatch):
    calls = []
    ext = SimpleNamespace(is_available=lambda: True,
                          flash_attn_with_kvcache=lambda *args: calls.append(args) or args[-1])
    monkeypatch.setattr(dispatch, "_native_extension", lambda: ext)
    monkeypatch.setattr(dispatch, "native_unavailable_reason", lambda tensor, op: None)
    q, k, v = tensors()
    sl = torch.tensor([3], dtype=torch.int32)
    with pytest.raises(ValueError, match="out must be"):
        flash_attn_with_kvcache(q, k, v, cache_seqlens=sl, out=torch.empty(1, 1, 2, 64, dtype=q.dtype))
    with pytest.raises(ValueError, match="out must be"):
        flash_attn_with_kvcache(q, k, v, cache_seqlens=sl, out=torch.empty_like(q, dtype=torch.bfloat16))
    assert not calls
    out = torch.empty_like(q)
    assert flash_attn_with_kvcache(q, k, v, cache_seqlens=sl, out=out) is out
    assert calls[0][-3:-1] == (1.0, 1.0) and calls[0][-1] is out
    # without `out` the backend receives the reference's nine positional arguments
    flash_attn_with_kvcache(q, k, v, cache_seqlens=sl)
    assert len(calls[1]) == 9


def test_length_order_is_validated_and_passed_to_the_backend(monkeypatch):
    calls = []
    ext = SimpleNamespace(is_available=lambda: True,
                          flash_attn_with_kvcache=lambda *args: calls.append(args) or args[0])
    monkeypatch.setattr(dispatch, "_native_extension", lambda: ext)
    monkeypatch.setattr(dispatch, "native_unavailable_reason", lambda tensor, op: None)
    q, k, v = tensors()
    sl = torch.tensor([3], dtype=torch.int32)
    for bad in (torch.zeros(1, dtype=torch.int64), torch.zeros(2, dtype=torch.int32), [0]):
        with pytest.raises(ValueError, match="length_order must be"):
            flash_attn_with_kvcache(q, k, v, cache_seqlens=sl, length_order=bad)
    assert not calls
    order = torch.zeros(1, dtype=torch.int32)
    flash_attn_with_kvcache(q, k, v, cache_seqlens=sl, length_order=order)
    # scales, out (None) and the order follow the reference's nine positional arguments
    assert len(calls[0]) == 13 and calls[0][-2] is None and calls[0][-1] is order


def test_length_order_helper_guards():
    from mxflashattn_b200 import kvcache_length_order

    with pytest.raises(TypeError, match="torch.Tensor"):
        kvcache_length_order([1, 2])
    with pytest.raises(ValueError, match="one-dimensional"):
        kvcache_length_order(torch.zeros(2, 2, dtype=torch.int32))
    with pytest.raises(ValueError, match="CUDA device"):
        kvcache_length_order(torch.zeros(4, dtype=torch.int32))


def test_public_signatures_are_the_references():
    """Each public function takes the reference's parameters in its order, with its kinds and defaults, and each
    exported record has its fields and defaults (tests/golden/api_signatures.json, read from the reference
    package); additions to the functions are keyword-only."""
    import dataclasses
    import inspect
    import json
    import os

    import mxflashattn_b200
    import mxflashattn_b200.api as api

    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "api_signatures.json")
    with open(path) as f:
        reference = json.load(f)
    records = reference.pop("records")
    for name, ref_fields in records.items():
        ours = [[f.name, None if f.default is dataclasses.MISSING else repr(f.default)]
                for f in dataclasses.fields(getattr(mxflashattn_b200, name))]
        assert ours == ref_fields, name
    for name, ref_params in reference.items():
        ours = [[n, p.kind.name, repr(p.default)] for n, p in inspect.signature(getattr(api, name)).parameters.items()]
        assert ours[:len(ref_params)] == ref_params, name
        assert all(kind == "KEYWORD_ONLY" for _, kind, _ in ours[len(ref_params):]), name


def _reference_errors():
    import json
    import os

    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "api_errors.json")
    with open(path) as f:
        return json.load(f)


@pytest.mark.parametrize("case", sorted(_reference_errors()))
def test_invalid_calls_raise_what_the_reference_raises(case, monkeypatch):
    """Exception type and message on the reference's invalid calls (tests/golden/api_errors.json, recorded by
    running the reference's API on tests/golden/api_error_cases.py)."""
    import api_error_cases

    import mxflashattn_b200

    fn_name, build, strict = api_error_cases.cases()[case]
    monkeypatch.setenv("MXFLASHATTN_STRICT_VALIDATION", "1" if strict else "0")
    monkeypatch.delenv("MXFLASHATTN_ALLOW_FALLBACK", raising=False)
    args, kwargs = build()
    expected_type, expected_message = _reference_errors()[case]
    with pytest.raises(Exception) as info:
        getattr(mxflashattn_b200, fn_name)(*args, **kwargs)
    assert [type(info.value).__name__, str(info.value)] == [expected_type, expected_message]


@pytest.mark.parametrize("env,um", [(None, 2), ("0", 0), ("1", 1), ("2", 2), (" 1", 1), ("1.5", 1), ("abc", 0),
                                    ("-1", 2), ("+1", 1), ("", 0), ("7", 2)])
def test_m1_softmax_variant_is_read_like_the_reference_binding(env, um, monkeypatch):
    """MXFA_M1_UM parsed as C atoi, 0 and 1 honoured, else 2 (m1_binding.cpp:100-105)."""
    from mxflashattn_b200 import m1

    if env is None:
        monkeypatch.delenv("MXFA_M1_UM", raising=False)
    else:
        monkeypatch.setenv("MXFA_M1_UM", env)
    assert m1.softmax_variant_from_env() == um
