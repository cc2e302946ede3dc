"""The reference's device-conditional API tests (tests/test_c500.py), on B200.

Same inputs, seeds and assertions as the reference's C500 suite, with the
backend label set extended by this build's ``cuda_sm100``; tolerances are the
reference's 0.04 plus the tighter north-star bars where they apply.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from helpers import host

pytestmark = pytest.mark.gpu

NATIVE_BACKENDS = {"vendor_direct", "mxmac_aten_correctness", "mxmac_flash_attn", "mxmac_aten_extension",
                   "cuda_sm100"}


def _assert_native_dispatch():
    from mxflashattn_b200 import get_last_dispatch_info

    info = get_last_dispatch_info()
    assert info is not None and info.backend in NATIVE_BACKENDS


@pytest.mark.parametrize("dtype_name", ["float16", "bfloat16"])
def test_batched_gqa_causal_matches_reference(dtype_name, cuda_device):
    import torch

    from mxflashattn_b200 import flash_attn_func

    dtype = getattr(torch, dtype_name)
    torch.manual_seed(21)
    q = torch.randn((2, 4, 8, 64), device=cuda_device, dtype=dtype)
    k = torch.randn((2, 7, 2, 64), device=cuda_device, dtype=dtype)
    v = torch.randn_like(k)
    actual = flash_attn_func(q, k, v, causal=True)
    _assert_native_dispatch()
    expected = oracle.attention_batched(host(q), host(k), host(v), causal=True)
    np.testing.assert_allclose(host(actual), expected, rtol=0.04, atol=0.04)


@pytest.mark.parametrize("dtype_name", ["float16", "bfloat16"])
def test_native_backend_preserves_zero_scale(dtype_name, cuda_device):
    import torch

    from mxflashattn_b200 import flash_attn_func

    dtype = getattr(torch, dtype_name)
    torch.manual_seed(24)
    q = torch.randn((1, 2, 4, 64), device=cuda_device, dtype=dtype)
    k = torch.randn((1, 5, 2, 64), device=cuda_device, dtype=dtype)
    v = torch.randn_like(k)
    actual = flash_attn_func(q, k, v, softmax_scale=0.0)
    _assert_native_dispatch()
    expected = oracle.attention_batched(host(q), host(k), host(v), softmax_scale=0.0)
    np.testing.assert_allclose(host(actual), expected, rtol=0.04, atol=0.04)


@pytest.mark.parametrize("dtype_name", ["float16", "bfloat16"])
def test_varlen_gqa_matches_reference(dtype_name, cuda_device):
    import torch

    from mxflashattn_b200 import flash_attn_varlen_func

    dtype = getattr(torch, dtype_name)
    torch.manual_seed(22)
    q = torch.randn((5, 4, 64), device=cuda_device, dtype=dtype)
    k = torch.randn((8, 2, 64), device=cuda_device, dtype=dtype)
    v = torch.randn_like(k)
    cu_q = torch.tensor([0, 2, 5], device=cuda_device, dtype=torch.int32)
    cu_k = torch.tensor([0, 3, 8], device=cuda_device, dtype=torch.int32)
    actual = flash_attn_varlen_func(q, k, v, cu_q, cu_k, max_seqlen_q=3, max_seqlen_k=5)
    _assert_native_dispatch()
    expected = oracle.attention_varlen(host(q), host(k), host(v), [0, 2, 5], [0, 3, 8])
    np.testing.assert_allclose(host(actual), expected, rtol=0.04, atol=0.04)


@pytest.mark.parametrize("dtype_name", ["float16", "bfloat16"])
def test_paged_kv_append_matches_reference(dtype_name, cuda_device):
    import torch

    from mxflashattn_b200 import flash_attn_with_kvcache

    dtype = getattr(torch, dtype_name)
    torch.manual_seed(23)
    q = torch.randn((1, 1, 4, 64), device=cuda_device, dtype=dtype)
    k_cache = torch.randn((3, 4, 2, 64), device=cuda_device, dtype=dtype)
    v_cache = torch.randn_like(k_cache)
    new_k = torch.randn((1, 1, 2, 64), device=cuda_device, dtype=dtype)
    new_v = torch.randn_like(new_k)
    block_table = torch.tensor([[2, 0]], device=cuda_device, dtype=torch.int32)
    cache_seqlens = torch.tensor([5], device=cuda_device, dtype=torch.int32)

    actual_k, actual_v, actual_sl = k_cache.clone(), v_cache.clone(), cache_seqlens.clone()
    actual = flash_attn_with_kvcache(q, actual_k, actual_v, k=new_k, v=new_v, cache_seqlens=actual_sl,
                                     block_table=block_table)
    _assert_native_dispatch()
    exp_k, exp_v, exp_sl = host(k_cache), host(v_cache), cache_seqlens.cpu().numpy()
    expected = oracle.attention_kvcache(host(q), exp_k, exp_v, cache_seqlens=exp_sl,
                                        block_table=block_table.cpu().numpy(), k=host(new_k), v=host(new_v))
    np.testing.assert_allclose(host(actual), expected, rtol=0.04, atol=0.04)
    np.testing.assert_array_equal(host(actual_k), exp_k)
    np.testing.assert_array_equal(host(actual_v), exp_v)
    assert actual_sl.tolist() == exp_sl.tolist() == [6]


def test_paged_kv_cache_reads_blocks_in_table_order(cuda_device):
    """reference test_api.py:136-155 on the device."""
    import torch

    from mxflashattn_b200 import flash_attn_func, flash_attn_with_kvcache

    torch.manual_seed(5)
    q = torch.randn(1, 1, 2, 64, device=cuda_device, dtype=torch.float16)
    k_cache = torch.randn(2, 2, 1, 64, device=cuda_device, dtype=torch.float16)
    v_cache = torch.randn_like(k_cache)
    block_table = torch.tensor([[1, 0]], dtype=torch.int32, device=cuda_device)
    cache_seqlens = torch.tensor([3], dtype=torch.int32, device=cuda_device)
    out = flash_attn_with_kvcache(q, k_cache, v_cache, cache_seqlens=cache_seqlens, block_table=block_table)
    expected_k = torch.cat((k_cache[1], k_cache[0, :1]), dim=0).unsqueeze(0)
    expected_v = torch.cat((v_cache[1], v_cache[0, :1]), dim=0).unsqueeze(0)
    expected = flash_attn_func(q, expected_k, expected_v)
    torch.testing.assert_close(out, expected, rtol=0, atol=2e-3)


def test_out_buffer_receives_the_same_result(cuda_device):
    """The keyword-only ``out`` extension writes the result in place, bit for bit."""
    import torch

    from mxflashattn_b200 import flash_attn_with_kvcache

    torch.manual_seed(6)
    q = torch.randn(3, 1, 8, 128, device=cuda_device, dtype=torch.bfloat16)
    kc = torch.randn(40, 16, 2, 128, device=cuda_device, dtype=torch.bfloat16)
    vc = torch.randn_like(kc)
    bt = torch.randperm(39, device=cuda_device).to(torch.int32).reshape(3, 13)
    sl = torch.tensor([200, 17, 1], dtype=torch.int32, device=cuda_device)
    ref = flash_attn_with_kvcache(q, kc, vc, cache_seqlens=sl, block_table=bt)
    out = torch.full_like(q, float("nan"))
    got = flash_attn_with_kvcache(q, kc, vc, cache_seqlens=sl, block_table=bt, out=out)
    torch.cuda.synchronize()
    assert got is out
    assert torch.equal(out, ref)


def test_strict_validation_rejects_out_of_range_page(monkeypatch, cuda_device):
    import torch

    from mxflashattn_b200 import flash_attn_with_kvcache

    monkeypatch.setenv("MXFLASHATTN_STRICT_VALIDATION", "1")
    q = torch.randn(1, 1, 2, 64, device=cuda_device, dtype=torch.float16)
    kc = torch.randn(2, 2, 1, 64, device=cuda_device, dtype=torch.float16)
    with pytest.raises(ValueError, match="out-of-range page"):
        flash_attn_with_kvcache(q, kc, kc.clone(), cache_seqlens=torch.tensor([3], device=cuda_device, dtype=torch.int32),
                                block_table=torch.tensor([[0, 5]], device=cuda_device, dtype=torch.int32))


def test_float32_inputs_are_rejected_without_fallback(cuda_device):
    import torch

    from mxflashattn_b200 import BackendUnavailableError, flash_attn_func

    q = torch.randn(1, 2, 2, 64, device=cuda_device)
    with pytest.raises(BackendUnavailableError, match="float16_and_bfloat16"):
        flash_attn_func(q, q[:, :, :1], q[:, :, :1])
