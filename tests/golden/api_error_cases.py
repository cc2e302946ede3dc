"""Invalid calls of the public API, shared by ``make_api_errors.py`` and the contract test.

Each case names the public function and builds its arguments from CPU
tensors, deterministically.  Every call is rejected by argument validation
before any dispatch, so the exception type and message are the API's own
contract, the same whichever backend would have run.  ``strict`` cases run
with ``MXFLASHATTN_STRICT_VALIDATION=1`` (the host-syncing checks).
"""

from __future__ import annotations

import torch

BF16 = torch.bfloat16


def _qkv(q_heads=4, kv_heads=2, dim=64, q_len=3, k_len=5, batch=2, dtype=BF16):
    g = torch.Generator().manual_seed(7)
    q = torch.randn(batch, q_len, q_heads, dim, generator=g).to(dtype)
    k = torch.randn(batch, k_len, kv_heads, dim, generator=g).to(dtype)
    return q, k, k.clone()


def _packed(q_tokens=6, k_tokens=8, q_heads=4, kv_heads=2, dim=64, dtype=BF16):
    g = torch.Generator().manual_seed(8)
    q = torch.randn(q_tokens, q_heads, dim, generator=g).to(dtype)
    k = torch.randn(k_tokens, kv_heads, dim, generator=g).to(dtype)
    return q, k, k.clone()


def _cu(*offsets, dtype=torch.int32):
    return torch.tensor(offsets, dtype=dtype)


def _func(**kw):
    q, k, v = _qkv()
    return (q, k, v), kw


def _varlen(q=None, k=None, v=None, cu_q=None, cu_k=None, max_q=4, max_k=5, **kw):
    pq, pk, pv = _packed()
    q = pq if q is None else q
    k = pk if k is None else k
    v = pv if v is None else v
    cu_q = _cu(0, 2, 6) if cu_q is None else cu_q
    cu_k = _cu(0, 3, 8) if cu_k is None else cu_k
    return (q, k, v, cu_q, cu_k, max_q, max_k), kw


def _paged(q_heads=4, kv_heads=2, dim=64, batch=2, page_size=4, pages=6, dtype=BF16):
    g = torch.Generator().manual_seed(9)
    q = torch.randn(batch, 1, q_heads, dim, generator=g).to(dtype)
    kc = torch.randn(pages, page_size, kv_heads, dim, generator=g).to(dtype)
    return q, kc, kc.clone()


def _kv(q=None, kc=None, vc=None, **kw):
    pq, pkc, pvc = _paged()
    q = pq if q is None else q
    kc = pkc if kc is None else kc
    vc = pvc if vc is None else vc
    kw.setdefault("cache_seqlens", torch.tensor([3, 5], dtype=torch.int32))
    kw.setdefault("block_table", torch.tensor([[0, 1, 2], [3, 4, 5]], dtype=torch.int32))
    return (q, kc, vc), kw


def cases():
    """name -> (public function name, builder returning (args, kwargs), strict validation on?)."""
    q, k, v = _qkv()
    pq, pk, pv = _packed()
    c = {
        # flash_attn_func
        "func_q_not_a_tensor": ("flash_attn_func", lambda: ((q.tolist(), k, v), {}), False),
        "func_q_rank3": ("flash_attn_func", lambda: ((q[0], k, v), {}), False),
        "func_dtype_mismatch": ("flash_attn_func", lambda: ((q, k.half(), v), {}), False),
        "func_float64": ("flash_attn_func", lambda: ((q.double(), k.double(), v.double()), {}), False),
        "func_head_dim_96": ("flash_attn_func", lambda: (_qkv(dim=96), {}), False),
        "func_heads_not_divisible": ("flash_attn_func", lambda: (_qkv(q_heads=6, kv_heads=4), {}), False),
        "func_batch_mismatch": ("flash_attn_func", lambda: ((q, k[:1], v[:1]), {}), False),
        "func_kv_shape_mismatch": ("flash_attn_func", lambda: ((q, k, v[:, :4]), {}), False),
        "func_empty_keys": ("flash_attn_func", lambda: ((q, k[:, :0], v[:, :0]), {}), False),
        "func_scale_nan": ("flash_attn_func", lambda: _func(softmax_scale=float("nan")), False),
        "func_scale_not_a_number": ("flash_attn_func", lambda: _func(softmax_scale="x"), False),
        "func_dropout": ("flash_attn_func", lambda: _func(dropout_p=0.1), False),
        "func_window": ("flash_attn_func", lambda: _func(window_size=(4, 0)), False),
        "func_softcap": ("flash_attn_func", lambda: _func(softcap=5.0), False),
        "func_alibi": ("flash_attn_func", lambda: _func(alibi_slopes=torch.ones(4)), False),
        "func_deterministic": ("flash_attn_func", lambda: _func(deterministic=True), False),
        "func_return_attn_probs": ("flash_attn_func", lambda: _func(return_attn_probs=True), False),
        # flash_attn_varlen_func
        "varlen_q_rank4": ("flash_attn_varlen_func", lambda: _varlen(q=pq[None]), False),
        "varlen_kv_shape_mismatch": ("flash_attn_varlen_func", lambda: _varlen(v=pv[:7]), False),
        "varlen_dtype_mismatch": ("flash_attn_varlen_func", lambda: _varlen(k=pk.half(), v=pv.half()), False),
        "varlen_float64": ("flash_attn_varlen_func",
                           lambda: _varlen(q=pq.double(), k=pk.double(), v=pv.double()), False),
        "varlen_heads_not_multiple": ("flash_attn_varlen_func",
                                      lambda: _varlen(*_packed(q_heads=3, kv_heads=2)), False),
        "varlen_head_dim_96": ("flash_attn_varlen_func", lambda: _varlen(*_packed(dim=96)), False),
        "varlen_cu_not_a_tensor": ("flash_attn_varlen_func", lambda: _varlen(cu_q=[0, 2, 6]), False),
        "varlen_cu_float": ("flash_attn_varlen_func", lambda: _varlen(cu_q=_cu(0, 2, 6, dtype=torch.float32)),
                            False),
        "varlen_cu_2d": ("flash_attn_varlen_func", lambda: _varlen(cu_k=_cu(0, 3, 8)[None]), False),
        "varlen_cu_not_covering": ("flash_attn_varlen_func", lambda: _varlen(cu_q=_cu(0, 2, 5)), False),
        "varlen_cu_not_from_zero": ("flash_attn_varlen_func", lambda: _varlen(cu_q=_cu(1, 2, 6)), False),
        "varlen_cu_decreasing": ("flash_attn_varlen_func", lambda: _varlen(cu_k=_cu(0, 5, 3, 8), cu_q=_cu(0, 2, 4, 6)),
                                 False),
        "varlen_max_too_small": ("flash_attn_varlen_func", lambda: _varlen(max_q=3), False),
        "varlen_empty_key_sequence": ("flash_attn_varlen_func", lambda: _varlen(cu_k=_cu(0, 0, 8)), False),
        "varlen_batch_mismatch": ("flash_attn_varlen_func", lambda: _varlen(cu_k=_cu(0, 3, 5, 8)), False),
        "varlen_dropout": ("flash_attn_varlen_func", lambda: _varlen(dropout_p=0.5), False),
        "varlen_scale_inf": ("flash_attn_varlen_func", lambda: _varlen(softmax_scale=float("inf")), False),
        # flash_attn_with_kvcache
        "kv_rotary": ("flash_attn_with_kvcache", lambda: _kv(rotary_cos=torch.ones(1)), False),
        "kv_return_lse": ("flash_attn_with_kvcache", lambda: _kv(return_softmax_lse=True), False),
        "kv_window": ("flash_attn_with_kvcache", lambda: _kv(window_size=(2, 2)), False),
        "kv_softcap": ("flash_attn_with_kvcache", lambda: _kv(softcap=1.0), False),
        "kv_scale_nan": ("flash_attn_with_kvcache", lambda: _kv(softmax_scale=float("nan")), False),
        "kv_k_without_v": ("flash_attn_with_kvcache", lambda: _kv(k=torch.zeros(2, 1, 2, 64, dtype=BF16)), False),
        "kv_q_rank3": ("flash_attn_with_kvcache", lambda: _kv(q=_paged()[0][:, 0]), False),
        "kv_cache_shape_mismatch": ("flash_attn_with_kvcache", lambda: _kv(vc=_paged()[2][:5]), False),
        "kv_dtype_mismatch": ("flash_attn_with_kvcache", lambda: _kv(q=_paged()[0].half()), False),
        "kv_float64": ("flash_attn_with_kvcache",
                       lambda: _kv(*(t.double() for t in _paged())), False),
        "kv_dense_batch_mismatch": ("flash_attn_with_kvcache",
                                    lambda: _kv(*_paged(pages=3), block_table=None,
                                                cache_seqlens=torch.tensor([1, 2], dtype=torch.int32)), False),
        "kv_head_dim_96": ("flash_attn_with_kvcache", lambda: _kv(*_paged(dim=96)), False),
        "kv_heads_not_divisible": ("flash_attn_with_kvcache", lambda: _kv(*_paged(q_heads=3, kv_heads=2)), False),
        "kv_page_size_zero": ("flash_attn_with_kvcache", lambda: _kv(*_paged(page_size=0)), False),
        "kv_append_shapes_differ": ("flash_attn_with_kvcache",
                                    lambda: _kv(k=torch.zeros(2, 1, 2, 64, dtype=BF16),
                                                v=torch.zeros(2, 2, 2, 64, dtype=BF16)), False),
        "kv_append_batch_mismatch": ("flash_attn_with_kvcache",
                                     lambda: _kv(k=torch.zeros(1, 1, 2, 64, dtype=BF16),
                                                 v=torch.zeros(1, 1, 2, 64, dtype=BF16)), False),
        "kv_append_dtype_mismatch": ("flash_attn_with_kvcache",
                                     lambda: _kv(k=torch.zeros(2, 1, 2, 64, dtype=torch.float16),
                                                 v=torch.zeros(2, 1, 2, 64, dtype=torch.float16)), False),
        "kv_no_seqlens": ("flash_attn_with_kvcache", lambda: _kv(cache_seqlens=None), False),
        "kv_seqlens_not_a_tensor": ("flash_attn_with_kvcache", lambda: _kv(cache_seqlens=[3, 5]), False),
        "kv_seqlens_wrong_count": ("flash_attn_with_kvcache",
                                   lambda: _kv(cache_seqlens=torch.tensor([3], dtype=torch.int32)), False),
        "kv_seqlens_float": ("flash_attn_with_kvcache", lambda: _kv(cache_seqlens=torch.tensor([3.0, 5.0])), False),
        "kv_table_not_a_tensor": ("flash_attn_with_kvcache", lambda: _kv(block_table=[[0, 1, 2], [3, 4, 5]]),
                                  False),
        "kv_table_wrong_rows": ("flash_attn_with_kvcache",
                                lambda: _kv(block_table=torch.tensor([[0, 1, 2]], dtype=torch.int32)), False),
        "kv_table_float": ("flash_attn_with_kvcache",
                           lambda: _kv(block_table=torch.tensor([[0.0, 1.0, 2.0], [3.0, 4.0, 5.0]])), False),
        # host-syncing checks (MXFLASHATTN_STRICT_VALIDATION=1)
        "kv_strict_negative_length": ("flash_attn_with_kvcache",
                                      lambda: _kv(cache_seqlens=torch.tensor([-1, 5], dtype=torch.int32)), True),
        "kv_strict_no_tokens": ("flash_attn_with_kvcache",
                                lambda: _kv(cache_seqlens=torch.tensor([0, 5], dtype=torch.int32)), True),
        "kv_strict_dense_overflow": ("flash_attn_with_kvcache",
                                     lambda: _kv(*_paged(pages=2), block_table=None,
                                                 cache_seqlens=torch.tensor([4, 5], dtype=torch.int32)), True),
        "kv_strict_table_too_short": ("flash_attn_with_kvcache",
                                      lambda: _kv(cache_seqlens=torch.tensor([3, 13], dtype=torch.int32)), True),
        "kv_strict_page_out_of_range": ("flash_attn_with_kvcache",
                                        lambda: _kv(block_table=torch.tensor([[0, 1, 2], [3, 9, 5]],
                                                                             dtype=torch.int32)), True),
    }
    return c
