"""vLLM paged decoder metadata -> ``flash_attn_with_kvcache`` (integrations/vllm/decoder_adapter.py:117-286).

Converts vLLM's packed query ``[tokens, heads, dim]``, its
``[2, blocks, block_size, kv_heads, dim]`` cache and the attention metadata
into one paged ``flash_attn_with_kvcache`` call on the B200 backend.  Only
one-token decode is owned; prefill, cascade and other layouts raise
``DecoderAdapterBlocked`` so the caller can hand them back to vLLM.

The environment switches keep the reference's meaning:
``MXFLASHATTN_GRAPH_DECODE`` (static-shape decode for CUDA-graph capture),
``MXFLASHATTN_TRANSPARENT`` (minimal checks) and ``MXFLASHATTN_STRICT_LAYOUT``
(host-syncing layout inspection, off by default because it reads device
metadata back every layer).
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Any

import torch

from mxflashattn_b200 import flash_attn_with_kvcache, kvcache_length_order

STRICT_LAYOUT = os.getenv("MXFLASHATTN_STRICT_LAYOUT", "0") == "1"
_REQUIRED = ("num_actual_tokens", "max_query_len", "query_start_loc", "max_seq_len", "seq_lens", "block_table",
             "scheduler_metadata", "causal", "use_cascade")


def _transparent_enabled() -> bool:
    return os.getenv("MXFLASHATTN_TRANSPARENT", "0") == "1"


@dataclass(frozen=True, slots=True)
class DecoderLayout:
    num_actual_tokens: int
    batch_size: int
    query_lens: tuple[int, ...]
    max_query_len: int
    seq_lens: tuple[int, ...]
    query_start_loc: tuple[int, ...]
    block_table_shape: tuple[int, int]
    kv_cache_shape: tuple[int, int, int, int, int]
    scheduler_metadata_present: bool


class DecoderAdapterBlocked(RuntimeError):
    """Raised when vLLM metadata is outside the adapter's verified contract."""


def _check_shapes(query: torch.Tensor, kv_cache: torch.Tensor, attn_metadata: Any) -> None:
    missing = [name for name in _REQUIRED if not hasattr(attn_metadata, name)]
    if missing:
        raise DecoderAdapterBlocked(f"metadata_missing_fields:{','.join(missing)}")
    if query.ndim != 3:
        raise DecoderAdapterBlocked(f"query_rank:{query.ndim},expected:3")
    if kv_cache.ndim != 5 or kv_cache.shape[0] != 2:
        raise DecoderAdapterBlocked(
            f"kv_cache_shape:{tuple(kv_cache.shape)},expected:[2,blocks,block_size,kv_heads,head_dim]")


def inspect_layout(query: torch.Tensor, kv_cache: torch.Tensor, attn_metadata: Any) -> DecoderLayout:
    """Full layout record; reads query_start_loc and seq_lens back to the host."""
    _check_shapes(query, kv_cache, attn_metadata)
    starts = tuple(int(x) for x in attn_metadata.query_start_loc.detach().cpu().tolist())
    seq_lens = tuple(int(x) for x in attn_metadata.seq_lens.detach().cpu().tolist())
    if len(starts) != len(seq_lens) + 1 or starts[0] != 0 or starts[-1] != int(attn_metadata.num_actual_tokens):
        raise DecoderAdapterBlocked("query_start_loc_does_not_cover_num_actual_tokens")
    block_table = attn_metadata.block_table
    if block_table.ndim != 2 or block_table.shape[0] != len(seq_lens):
        raise DecoderAdapterBlocked("block_table_rows_do_not_match_batch")
    return DecoderLayout(
        num_actual_tokens=int(attn_metadata.num_actual_tokens),
        batch_size=len(seq_lens),
        query_lens=tuple(b - a for a, b in zip(starts, starts[1:])),
        max_query_len=int(attn_metadata.max_query_len),
        seq_lens=seq_lens,
        query_start_loc=starts,
        block_table_shape=(int(block_table.shape[0]), int(block_table.shape[1])),
        kv_cache_shape=tuple(int(x) for x in kv_cache.shape),
        scheduler_metadata_present=attn_metadata.scheduler_metadata is not None,
    )


def fast_layout(query: torch.Tensor, kv_cache: torch.Tensor, attn_metadata: Any) -> DecoderLayout:
    """Layout record without any device-to-host synchronisation."""
    _check_shapes(query, kv_cache, attn_metadata)
    block_table = attn_metadata.block_table
    if block_table.ndim != 2:
        raise DecoderAdapterBlocked("block_table_rows_do_not_match_batch")
    batch = int(block_table.shape[0])
    max_query_len = int(attn_metadata.max_query_len)
    return DecoderLayout(
        num_actual_tokens=int(attn_metadata.num_actual_tokens),
        batch_size=batch,
        query_lens=tuple([max_query_len] * batch),
        max_query_len=max_query_len,
        seq_lens=(),
        query_start_loc=(),
        block_table_shape=(batch, int(block_table.shape[1])),
        kv_cache_shape=tuple(int(x) for x in kv_cache.shape),
        scheduler_metadata_present=attn_metadata.scheduler_metadata is not None,
    )


def _step_length_order(attn_metadata, cache_seqlens: torch.Tensor):
    """The batch's longest-first order, computed by the step's first layer and reused by the others.

    vLLM hands one metadata object per step to every attention layer, so the
    order (one small kernel) is kept on it.  The order only schedules the
    work: a metadata object reused with other lengths costs speed, never
    correctness.  Objects that take no new attributes recompute per layer.
    None off the GPU (the order is a launch option of the CUDA backend).
    """
    if not cache_seqlens.is_cuda:
        return None
    order = getattr(attn_metadata, "_mxfa_length_order", None)
    if order is None or order.shape[0] != cache_seqlens.shape[0] or order.device != cache_seqlens.device:
        order = kvcache_length_order(cache_seqlens)
        try:
            attn_metadata._mxfa_length_order = order
        except (AttributeError, TypeError):  # frozen or slotted metadata
            pass
    return order


def _as_device_i32(t: torch.Tensor, device) -> torch.Tensor:
    # vLLM already keeps these int32 on the device; convert only when it does not
    return t if (t.device == device and t.dtype == torch.int32) else t.to(device=device, dtype=torch.int32)


def decode_forward(
    query: torch.Tensor,
    kv_cache: torch.Tensor,
    attn_metadata: Any,
    *,
    softmax_scale: float,
    causal: bool = True,
) -> tuple[torch.Tensor, DecoderLayout | None]:
    """One-token paged decode through the public API.

    vLLM writes the new token's K/V into the cache before attention, so no
    k/v is appended here and ``seq_lens`` already counts it.  Returns the
    output ``[num_tokens, heads * dim]`` and the layout record (None on the
    transparent and graph paths).
    """
    if os.getenv("MXFLASHATTN_GRAPH_DECODE", "0") == "1":
        has_padded_decode = (
            attn_metadata.seq_lens.ndim == 1
            and attn_metadata.block_table.ndim == 2
            and attn_metadata.seq_lens.numel() == attn_metadata.block_table.shape[0]
            and attn_metadata.seq_lens.numel() < query.shape[0]
        )
        has_split_decode = (
            int(getattr(attn_metadata, "num_decode_tokens", 0) or 0) > 0
            and int(getattr(attn_metadata, "num_decodes", 0) or 0) > 0
            and getattr(attn_metadata, "decode_seq_lens", None) is not None
            and getattr(attn_metadata, "decode_block_table", None) is not None
        )
        if int(getattr(attn_metadata, "max_query_len", 0)) != 1 and not has_padded_decode and not has_split_decode:
            raise DecoderAdapterBlocked(
                f"only_single_token_decode_supported:max_query_len={int(getattr(attn_metadata, 'max_query_len', 0))}")
        return _decode_forward_graph(query, kv_cache, attn_metadata, softmax_scale=softmax_scale, causal=causal)
    if _transparent_enabled():
        if int(attn_metadata.max_query_len) != 1:
            raise DecoderAdapterBlocked(
                f"only_single_token_decode_supported:max_query_len={int(attn_metadata.max_query_len)}")
        key_cache, value_cache = kv_cache.unbind(0)
        n = int(attn_metadata.num_actual_tokens)
        q = query[:n].reshape(n, 1, query.shape[1], query.shape[2])
        seq_lens = _as_device_i32(attn_metadata.seq_lens.reshape(-1), query.device)  # capture metadata may be [1, batch]
        result = flash_attn_with_kvcache(
            q, key_cache, value_cache, cache_seqlens=seq_lens,
            block_table=_as_device_i32(attn_metadata.block_table, query.device), softmax_scale=softmax_scale,
            causal=causal, length_order=_step_length_order(attn_metadata, seq_lens))
        return result.reshape(n, -1), None
    layout = inspect_layout(query, kv_cache, attn_metadata) if STRICT_LAYOUT else fast_layout(
        query, kv_cache, attn_metadata)
    if not bool(attn_metadata.causal) and causal:
        raise DecoderAdapterBlocked("metadata_causal_flag_is_false")
    if bool(attn_metadata.use_cascade):
        raise DecoderAdapterBlocked("cascade_attention_not_supported_by_adapter")
    if layout.max_query_len != 1:
        raise DecoderAdapterBlocked(f"only_single_token_decode_supported:max_query_len={layout.max_query_len}")
    if kv_cache.dtype not in (torch.float16, torch.bfloat16):
        raise DecoderAdapterBlocked(f"kv_cache_dtype_not_supported:{kv_cache.dtype}")
    if query.shape[1] % kv_cache.shape[3]:
        raise DecoderAdapterBlocked("query_and_kv_head_counts_are_not_gqa_compatible")
    key_cache, value_cache = kv_cache.unbind(0)
    batch = layout.batch_size
    q = query[: layout.num_actual_tokens].reshape(batch, 1, query.shape[1], query.shape[2])
    seq_lens = _as_device_i32(attn_metadata.seq_lens, query.device)
    result = flash_attn_with_kvcache(
        q, key_cache, value_cache, cache_seqlens=seq_lens,
        block_table=_as_device_i32(attn_metadata.block_table, query.device), softmax_scale=softmax_scale,
        causal=causal, length_order=_step_length_order(attn_metadata, seq_lens))
    return result.reshape(layout.num_actual_tokens, -1), layout


def _decode_forward_graph(query, kv_cache, attn_metadata, *, softmax_scale: float, causal: bool = True):
    """Static-shape decode for CUDA-graph capture (decoder_adapter.py:236-286).

    Uses the decode subset of the metadata when present; otherwise one query
    row per metadata row (capture padding of q is left out).
    """
    key_cache, value_cache = kv_cache.unbind(0)
    decode_n = int(getattr(attn_metadata, "num_decode_tokens", 0) or 0)
    decode_batch = int(getattr(attn_metadata, "num_decodes", 0) or 0)
    decode_seq = getattr(attn_metadata, "decode_seq_lens", None)
    decode_bt = getattr(attn_metadata, "decode_block_table", None)
    if decode_n > 0 and decode_batch > 0 and decode_seq is not None and decode_bt is not None:
        if decode_n % decode_batch:
            raise DecoderAdapterBlocked("decode_tokens_not_divisible_by_num_decodes")
        q = query[:decode_n].reshape(decode_batch, decode_n // decode_batch, query.shape[1],
                                     query.shape[2]).contiguous()
        cache_seqlens = decode_seq.reshape(-1)
        block_table = decode_bt
        batch = decode_batch
    else:
        raw_seq = attn_metadata.seq_lens.reshape(-1)
        batch = int(raw_seq.numel()) if raw_seq.numel() < query.shape[0] else query.shape[0]
        q = query[:batch].reshape(batch, 1, query.shape[1], query.shape[2]).contiguous()
        cache_seqlens = raw_seq
        block_table = attn_metadata.block_table
    cache_seqlens = _as_device_i32(cache_seqlens, query.device).contiguous()
    block_table = _as_device_i32(block_table, query.device).contiguous()
    if cache_seqlens.numel() != batch or block_table.shape[0] != batch:
        raise DecoderAdapterBlocked("decode_metadata_batch_mismatch")
    result = flash_attn_with_kvcache(q, key_cache, value_cache, cache_seqlens=cache_seqlens,
                                     block_table=block_table, softmax_scale=softmax_scale, causal=causal,
                                     length_order=_step_length_order(attn_metadata, cache_seqlens))
    return result.reshape(q.shape[0] * q.shape[1], -1), None
