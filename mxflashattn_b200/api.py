"""FlashAttention-compatible public API (drop-in for mxflashattn/api.py).

Signatures, guard order, exception types and messages follow the reference
(mxflashattn/api.py:34-286).  Each call validates cheaply on the host and
hands the resolved arguments to ``dispatch``, whose only backend is the
sm_100a CUDA library.
"""

from __future__ import annotations

import math
import os

import torch

from .dispatch import dispatch
from .validation import validate_cumulative_lengths, validate_options, validate_qkv, validate_softmax_scale


def _resolved_scale(head_dim: int, softmax_scale: float | None) -> float:
    # an explicit 0.0 is kept (uniform attention); None means 1/sqrt(D)
    return float(softmax_scale) if softmax_scale is not None else float(head_dim ** -0.5)


def flash_attn_func(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    dropout_p: float = 0.0,
    softmax_scale: float | None = None,
    causal: bool = False,
    window_size: tuple[int, int] = (-1, -1),
    softcap: float = 0.0,
    alibi_slopes: torch.Tensor | None = None,
    deterministic: bool = False,
    return_attn_probs: bool = False,
) -> torch.Tensor:
    """Dense attention forward, q [B, Sq, HQ, D], k/v [B, Sk, HKV, D] (api.py:34-66)."""
    validate_qkv(q, k, v)
    validate_softmax_scale(softmax_scale)
    validate_options(dropout_p=dropout_p, window_size=window_size, softcap=softcap, alibi_slopes=alibi_slopes,
                     deterministic=deterministic, return_attn_probs=return_attn_probs)
    return dispatch("flash_attn_func", q, (q, k, v, causal, _resolved_scale(q.shape[-1], softmax_scale)))


def flash_attn_varlen_func(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    cu_seqlens_q: torch.Tensor,
    cu_seqlens_k: torch.Tensor,
    max_seqlen_q: int,
    max_seqlen_k: int,
    dropout_p: float = 0.0,
    softmax_scale: float | None = None,
    causal: bool = False,
    window_size: tuple[int, int] = (-1, -1),
    softcap: float = 0.0,
    alibi_slopes: torch.Tensor | None = None,
    deterministic: bool = False,
    return_attn_probs: bool = False,
) -> torch.Tensor:
    """Packed variable-length forward, q [Tq, HQ, D], k/v [Tk, HKV, D] (api.py:69-148)."""
    validate_softmax_scale(softmax_scale)
    for name, tensor in (("q", q), ("k", k), ("v", v)):
        if not isinstance(tensor, torch.Tensor) or tensor.ndim != 3:
            raise ValueError(f"{name} must have rank 3 with layout [total_tokens, heads, dim]")
    if k.shape != v.shape:
        raise ValueError("k and v must have identical shapes")
    if q.device != k.device or q.device != v.device:
        raise ValueError("q, k, and v must be on the same device")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise ValueError("q, k, and v must have the same dtype")
    if q.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise TypeError("supported dtypes are float16, bfloat16, and float32 for reference execution")
    if q.shape[1] <= 0 or k.shape[1] <= 0 or q.shape[1] % k.shape[1]:
        raise ValueError("q heads must be a positive multiple of kv heads")
    if q.shape[2] not in (64, 128) or k.shape[2] != q.shape[2]:
        raise ValueError("head dimension must be 64 or 128 and match across q, k, and v")
    if not isinstance(cu_seqlens_q, torch.Tensor) or not isinstance(cu_seqlens_k, torch.Tensor):
        raise TypeError("cu_seqlens_q and cu_seqlens_k must be torch.Tensor values")
    if cu_seqlens_q.device != q.device or cu_seqlens_k.device != q.device:
        raise ValueError("cu_seqlens_q and cu_seqlens_k must be on the same device as q")
    validate_options(dropout_p=dropout_p, window_size=window_size, softcap=softcap, alibi_slopes=alibi_slopes,
                     deterministic=deterministic, return_attn_probs=return_attn_probs)
    q_offsets = validate_cumulative_lengths(cu_seqlens_q, total_tokens=q.shape[0], max_seqlen=max_seqlen_q,
                                            name="cu_seqlens_q")
    k_offsets = validate_cumulative_lengths(cu_seqlens_k, total_tokens=k.shape[0], max_seqlen=max_seqlen_k,
                                            name="cu_seqlens_k", require_non_empty=True)
    if len(q_offsets) != len(k_offsets):
        raise ValueError("cu_seqlens_q and cu_seqlens_k must describe the same batch size")
    return dispatch(
        "flash_attn_varlen_func",
        q,
        (q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, causal,
         _resolved_scale(q.shape[-1], softmax_scale)),
    )


def _strict_kvcache_checks(k_cache, k, cache_seqlens, block_table) -> None:
    """Host-syncing deep checks, enabled by MXFLASHATTN_STRICT_VALIDATION=1 (api.py:228-247)."""
    appended = 0 if k is None else k.shape[1]
    lengths = [int(x) for x in cache_seqlens.detach().cpu().tolist()]
    if any(n < 0 for n in lengths):
        raise ValueError("cache sequence lengths must be non-negative")
    if any(n + appended == 0 for n in lengths):
        raise ValueError("attention requires at least one cached or appended key/value token")
    page_size = k_cache.shape[1]
    if block_table is None:
        if any(n + appended > page_size for n in lengths):
            raise ValueError("cache sequence length exceeds dense cache capacity")
        return
    rows = block_table.detach().cpu().tolist()
    for n, row in zip(lengths, rows):
        used = (n + appended + page_size - 1) // page_size
        if used > block_table.shape[1]:
            raise ValueError("block_table does not contain enough pages for cache sequence")
        if any(int(pg) < 0 or int(pg) >= k_cache.shape[0] for pg in row[:used]):
            raise ValueError("block_table contains an out-of-range page index")


def flash_attn_with_kvcache(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    k: torch.Tensor | None = None,
    v: torch.Tensor | None = None,
    cache_seqlens: torch.Tensor | None = None,
    block_table: torch.Tensor | None = None,
    softmax_scale: float | None = None,
    causal: bool = False,
    window_size: tuple[int, int] = (-1, -1),
    softcap: float = 0.0,
    alibi_slopes: torch.Tensor | None = None,
    rotary_cos: torch.Tensor | None = None,
    rotary_sin: torch.Tensor | None = None,
    return_softmax_lse: bool = False,
    *,
    k_scale: float | None = None,
    v_scale: float | None = None,
    out: torch.Tensor | None = None,
    length_order: torch.Tensor | None = None,
) -> torch.Tensor:
    """Paged or dense KV-cache attention with optional append (api.py:151-286).

    Appending ``k``/``v`` writes the caches and advances ``cache_seqlens`` in
    place on the device, like the reference.

    Extensions beyond the reference (keyword-only, so every reference call is
    unchanged): ``k_cache``/``v_cache`` may be ``torch.float8_e4m3fn`` (head
    dim 128, q in fp16/bf16); the attended values are ``k_cache * k_scale``
    and ``v_cache * v_scale`` (default 1.0), and appended ``k``/``v`` must
    then already be e4m3 with the same scales.  ``out`` (contiguous, q's
    shape, dtype and device) receives the result instead of a new tensor and
    is returned.  ``length_order`` (int32 [B] on q's device, from
    ``kvcache_length_order(cache_seqlens)``, computed once per step and
    passed to every layer) schedules the sequences longest first without the
    ranking each launch otherwise does; it only orders the work, so the
    result is the same with or without it.
    """
    validate_softmax_scale(softmax_scale)
    if rotary_cos is not None or rotary_sin is not None:
        raise NotImplementedError("rotary embeddings are not supported")
    if return_softmax_lse:
        raise NotImplementedError("return_softmax_lse is not supported")
    validate_options(dropout_p=0.0, window_size=window_size, softcap=softcap, alibi_slopes=alibi_slopes,
                     deterministic=False, return_attn_probs=False)
    if (k is None) != (v is None):
        raise ValueError("k and v must either both be provided or both be omitted")
    if q.ndim != 4 or k_cache.ndim != 4 or v_cache.shape != k_cache.shape:
        raise ValueError("q and cache tensors must have rank 4 and matching k/v cache shapes")
    if q.device != k_cache.device or q.device != v_cache.device:
        raise ValueError("q and cache tensors must be on the same device")
    fp8_cache = k_cache.dtype == _FP8
    if fp8_cache:
        _validate_fp8_cache(q, k_cache, v_cache, k, v, k_scale, v_scale)
    elif k_scale is not None or v_scale is not None:
        raise ValueError("k_scale / v_scale apply to float8_e4m3fn caches only")
    elif q.dtype != k_cache.dtype or q.dtype != v_cache.dtype:
        raise ValueError("q and cache tensors must have the same dtype")
    if q.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise TypeError("supported dtypes are float16, bfloat16, and float32 for reference execution")
    if q.shape[0] != k_cache.shape[0] and block_table is None:
        raise ValueError("dense cache batch dimension must match q")
    if q.shape[2] <= 0 or k_cache.shape[2] <= 0:
        raise ValueError("q and kv cache head counts must be positive")
    if k_cache.shape[1] <= 0:
        raise ValueError("cache page size must be positive")
    if q.shape[3] not in (64, 128) or k_cache.shape[3] != q.shape[3]:
        raise ValueError("head dimension must be 64 or 128 and match across q and caches")
    if q.shape[2] % k_cache.shape[2]:
        raise ValueError("q heads must be divisible by kv cache heads")
    if k is not None and (k.shape != v.shape or k.ndim != 4):
        raise ValueError("appended k and v must have identical rank-4 shapes")
    if k is not None and (k.shape[0] != q.shape[0] or k.shape[2:] != k_cache.shape[2:]):
        raise ValueError("appended k/v must match batch, kv heads, and head dimension")
    if k is not None and not fp8_cache and (k.device != q.device or k.dtype != q.dtype or v.device != q.device
                                            or v.dtype != q.dtype):
        raise ValueError("appended k/v must match the query device and dtype")
    if cache_seqlens is None:
        raise ValueError("cache_seqlens is required for dense and paged caches")
    if not isinstance(cache_seqlens, torch.Tensor):
        raise TypeError("cache_seqlens must be a torch.Tensor")
    if cache_seqlens.ndim != 1 or cache_seqlens.numel() != q.shape[0]:
        raise ValueError("cache_seqlens must be one-dimensional with one value per batch item")
    if cache_seqlens.dtype not in (torch.int32, torch.int64):
        raise TypeError("cache_seqlens must use int32 or int64")
    if cache_seqlens.device != q.device:
        raise ValueError("cache_seqlens must be on the same device as q")
    if block_table is not None:
        if not isinstance(block_table, torch.Tensor):
            raise TypeError("block_table must be a torch.Tensor")
        if block_table.ndim != 2 or block_table.shape[0] != q.shape[0]:
            raise ValueError("block_table must have one row per batch item")
        if block_table.dtype not in (torch.int32, torch.int64):
            raise TypeError("block_table must use int32 or int64")
        if block_table.device != q.device:
            raise ValueError("block_table must be on the same device as q")
    elif k_cache.shape[0] != q.shape[0]:
        raise ValueError("dense cache batch dimension must match q")
    if out is not None and (not isinstance(out, torch.Tensor) or out.shape != q.shape or out.dtype != q.dtype
                            or out.device != q.device or not out.is_contiguous()):
        raise ValueError("out must be a contiguous tensor with q's shape, dtype and device")
    if length_order is not None and (not isinstance(length_order, torch.Tensor) or length_order.dtype != torch.int32
                                     or length_order.shape != (q.shape[0],) or length_order.device != q.device):
        raise ValueError("length_order must be an int32 tensor with one entry per batch item on q's device")
    if os.getenv("MXFLASHATTN_STRICT_VALIDATION", "0") == "1":
        _strict_kvcache_checks(k_cache, k, cache_seqlens, block_table)
    args = (q, k_cache, v_cache, k, v, cache_seqlens, block_table, _resolved_scale(q.shape[-1], softmax_scale),
            causal)
    if fp8_cache or out is not None or length_order is not None:
        args += (1.0 if k_scale is None else float(k_scale), 1.0 if v_scale is None else float(v_scale))
    if out is not None or length_order is not None:
        args += (out,)
    if length_order is not None:
        args += (length_order,)
    return dispatch("flash_attn_with_kvcache", q, args)


def kvcache_length_order(cache_seqlens: torch.Tensor) -> torch.Tensor | None:
    """The batch's longest-first order for ``flash_attn_with_kvcache(..., length_order=)``.

    No reference counterpart (an extension of this package).  One small
    kernel writes int32 [B] (order[rank] = sequence index, ties by index) on
    the device; call it once per decode step, after the lengths are final,
    and pass the result to every layer.  None for batches of one or of more
    than 512 sequences, which need no order.
    """
    if not isinstance(cache_seqlens, torch.Tensor):
        raise TypeError("cache_seqlens must be a torch.Tensor")
    if cache_seqlens.ndim != 1 or cache_seqlens.dtype not in (torch.int32, torch.int64):
        raise ValueError("cache_seqlens must be a one-dimensional int32 or int64 tensor")
    if cache_seqlens.device.type != "cuda":
        raise ValueError("cache_seqlens must be on a CUDA device")
    from . import backend

    return backend.kvcache_length_order(cache_seqlens)


_FP8 = getattr(torch, "float8_e4m3fn", None)


def _validate_fp8_cache(q, k_cache, v_cache, k, v, k_scale, v_scale) -> None:
    """Guards of the e4m3 cache extension (no reference counterpart)."""
    if v_cache.dtype != k_cache.dtype:
        raise ValueError("k_cache and v_cache must have the same dtype")
    if q.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError("float8_e4m3fn caches need a float16 or bfloat16 query")
    if q.shape[3] != 128:
        raise ValueError("float8_e4m3fn caches need head dimension 128")
    for name, value in (("k_scale", k_scale), ("v_scale", v_scale)):
        if value is not None and not (math.isfinite(float(value)) and float(value) > 0.0):
            raise ValueError(f"{name} must be a positive finite number")
    if k is not None and (k.dtype != k_cache.dtype or v.dtype != k_cache.dtype or k.device != q.device
                          or v.device != q.device):
        raise ValueError("appended k/v for a float8_e4m3fn cache must be float8_e4m3fn on the query device")
