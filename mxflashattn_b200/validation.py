"""Argument guards of the public API.

Same checks, exception types and messages as the reference's guards
(mxflashattn/validation.py:14-100), so callers and tests that match on
them keep working; the messages are part of the drop-in contract.
"""

from __future__ import annotations

import math
from collections.abc import Sequence

import torch

SUPPORTED_HEAD_DIMS = (64, 128)
REFERENCE_DTYPES = (torch.float16, torch.bfloat16, torch.float32)
NATIVE_DTYPES = (torch.float16, torch.bfloat16)


def validate_softmax_scale(softmax_scale: float | None) -> None:
    """None or a finite number (0.0 is a legal scale; validation.py:14-22)."""
    if softmax_scale is None:
        return
    try:
        value = float(softmax_scale)
    except (TypeError, ValueError) as error:
        raise TypeError("softmax_scale must be a finite number or None") from error
    if not math.isfinite(value):
        raise ValueError("softmax_scale must be finite")


def validate_qkv(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
    """Rank-4 [batch, seq, heads, dim] triple with GQA-compatible heads (validation.py:25-53)."""
    for name, tensor in (("q", q), ("k", k), ("v", v)):
        if not isinstance(tensor, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
        if tensor.ndim != 4:
            raise ValueError(f"{name} must have rank 4 with layout [batch, seq, heads, dim]")
    if q.device != k.device or q.device != v.device:
        raise ValueError("q, k, and v must be on the same device")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise ValueError("q, k, and v must have the same dtype")
    if q.dtype not in REFERENCE_DTYPES:
        raise TypeError("supported dtypes are float16, bfloat16, and float32 for reference execution")
    batch, q_len, q_heads, head_dim = q.shape
    kv_batch, kv_len, kv_heads, kv_dim = k.shape
    if v.shape != k.shape:
        raise ValueError("k and v must have identical shapes")
    if batch != kv_batch:
        raise ValueError("q, k, and v batch dimensions must match")
    if q_heads <= 0 or kv_heads <= 0:
        raise ValueError("q and kv head counts must be positive")
    if q_heads % kv_heads:
        raise ValueError("the number of q heads must be divisible by the number of kv heads")
    if head_dim != kv_dim or head_dim not in SUPPORTED_HEAD_DIMS:
        raise ValueError(
            f"head dimension must be one of {SUPPORTED_HEAD_DIMS} and match across q, k, and v")
    if q_len < 0 or kv_len <= 0:
        raise ValueError("q must have a non-negative sequence length and k/v must be non-empty")


_UNSUPPORTED_OPTIONS = (
    ("dropout_p", lambda v: v != 0, "dropout is not supported in the forward-only implementation"),
    ("window_size", lambda v: tuple(v) != (-1, -1), "local window attention is not supported"),
    ("softcap", lambda v: v != 0, "soft-capping is not supported"),
    ("alibi_slopes", lambda v: v is not None, "alibi_slopes are not supported"),
    ("return_attn_probs", bool, "return_attn_probs is not supported"),
    ("deterministic", bool, "deterministic mode is not currently supported"),
)


def validate_options(
    *,
    dropout_p: float,
    window_size: Sequence[int],
    softcap: float,
    alibi_slopes: torch.Tensor | None,
    return_attn_probs: bool,
    deterministic: bool,
) -> None:
    """Reject the FlashAttention options this forward path does not implement (validation.py:56-76)."""
    values = {
        "dropout_p": dropout_p,
        "window_size": window_size,
        "softcap": softcap,
        "alibi_slopes": alibi_slopes,
        "return_attn_probs": return_attn_probs,
        "deterministic": deterministic,
    }
    for name, rejected, message in _UNSUPPORTED_OPTIONS:
        if rejected(values[name]):
            raise NotImplementedError(message)


def validate_cumulative_lengths(
    cu_seqlens: torch.Tensor,
    *,
    total_tokens: int,
    max_seqlen: int,
    name: str,
    require_non_empty: bool = False,
) -> list[int]:
    """Host check of a cu_seqlens vector; returns it as a list (validation.py:79-100).

    This reads the tensor back to the host (one synchronisation), exactly as
    the reference API does for the varlen entry point.
    """
    if not isinstance(cu_seqlens, torch.Tensor) or cu_seqlens.ndim != 1:
        raise TypeError(f"{name} must be a one-dimensional torch.Tensor")
    if cu_seqlens.dtype not in (torch.int32, torch.int64):
        raise TypeError(f"{name} must use int32 or int64")
    offsets = [int(x) for x in cu_seqlens.detach().cpu().tolist()]
    if len(offsets) < 2 or offsets[0] != 0 or offsets[-1] != total_tokens:
        raise ValueError(f"{name} must start at zero and cover all tokens")
    lengths = [b - a for a, b in zip(offsets, offsets[1:])]
    if any(n < 0 for n in lengths):
        raise ValueError(f"{name} must be monotonically non-decreasing")
    if require_non_empty and any(n == 0 for n in lengths):
        raise ValueError("key/value sequences must be non-empty")
    if max_seqlen < 0 or max(lengths) > max_seqlen:
        raise ValueError(f"{name} contains a sequence longer than max_seqlen")
    return offsets
