"""The single CUDA backend behind ``dispatch``: torch tensors -> libmxfa_b200.

It exposes the extension contract the reference's dispatcher calls
(``getattr(ext, operation)(*extension_args)`` guarded by ``is_available()``,
mxflashattn/dispatch.py:131-137) with the positional argument lists the
reference's public API builds (mxflashattn/api.py:53, :122-133, :251-262):

* ``flash_attn_func(q, k, v, causal, scale)``
* ``flash_attn_varlen_func(q, k, v, cu_q, cu_k, max_q, max_k, causal, scale)``
* ``flash_attn_with_kvcache(q, k_cache, v_cache, k, v, cache_seqlens, block_table, scale, causal)``

PyTorch is used for device buffers and the current stream only; all math
runs in the sm_100a kernels.  Every call is asynchronous on the current
stream and reads nothing back to the host.
"""

from __future__ import annotations

import contextlib

import torch

from . import _lib

SUPPORTED_DTYPES = (torch.float16, torch.bfloat16)


_AVAILABLE: dict[int, bool] = {}


_CUDA_OK: list[bool] = []


def is_available() -> bool:
    """True when the current CUDA device is sm_100 and the library is usable (cached per device)."""
    if not _CUDA_OK:
        if not torch.cuda.is_available():
            return False
        _CUDA_OK.append(True)
    dev = torch.cuda.current_device()
    cached = _AVAILABLE.get(dev)
    if cached is not None:
        return cached
    try:
        ok = bool(_L().mxfa_is_available())
    except _lib.NativeLibraryError:
        ok = False
    _AVAILABLE[dev] = ok
    return ok


def _bf16(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return 1
    if t.dtype == torch.float16:
        return 0
    raise TypeError(f"the CUDA backend supports float16 and bfloat16, got {t.dtype}")


def _i32(t: torch.Tensor) -> torch.Tensor:
    return t if (t.dtype == torch.int32 and t.is_contiguous()) else t.to(torch.int32).contiguous()


def _contig(t: torch.Tensor) -> torch.Tensor:
    return t if t.is_contiguous() else t.contiguous()


_NULL_CTX = contextlib.nullcontext()


def _on(t: torch.Tensor):
    """Device context for a launch: a no-op when ``t`` already lives on the current device."""
    idx = t.device.index
    return _NULL_CTX if idx == torch.cuda.current_device() else torch.cuda.device(idx)


_LIB: list = []


def _L():
    """The loaded library (cached)."""
    if not _LIB:
        _LIB.append(_lib.load())
    return _LIB[0]


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


# ------------------------------------------------------------------ prefill

def flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, causal,
                           softmax_scale, *, return_lse: bool = False, exact_p: bool = False):
    """Packed varlen forward: q [Tq, HQ, D], k/v [Tk, HKV, D] -> out [Tq, HQ, D].

    ``exact_p``: keep P at ~16 significant bits in the P.V product
    (``mxfa_varlen_fwd_exact_launch``, 1.5x the tensor work) instead of
    rounding it once to the input type.
    """
    q, k, v = _contig(q), _contig(k), _contig(v)
    out = torch.empty_like(q)
    lse = torch.empty((q.shape[0], q.shape[1]), device=q.device, dtype=torch.float32) if return_lse else None
    cu_q, cu_k = _i32(cu_seqlens_q), _i32(cu_seqlens_k)
    batch = cu_q.numel() - 1
    name = "mxfa_varlen_fwd_exact_launch" if exact_p else "mxfa_varlen_fwd_launch"
    with _on(q):
        rc = getattr(_L(), name)(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), cu_q.data_ptr(), cu_k.data_ptr(), out.data_ptr(),
            _lib.ptr(lse), batch, int(max_seqlen_q), int(max_seqlen_k), q.shape[0], k.shape[0], q.shape[1],
            k.shape[1], q.shape[2], int(bool(causal)), _bf16(q), float(softmax_scale), _stream(q))
    _lib.check(rc, name)
    return (out, lse) if return_lse else out


def flash_attn_func(q, k, v, causal, softmax_scale, *, return_lse: bool = False, exact_p: bool = False):
    """Dense batched forward: q [B, Sq, HQ, D], k/v [B, Sk, HKV, D] -> out [B, Sq, HQ, D]."""
    q, k, v = _contig(q), _contig(k), _contig(v)
    out = torch.empty_like(q)
    B, Sq, HQ, D = q.shape
    lse = torch.empty((B, Sq, HQ), device=q.device, dtype=torch.float32) if return_lse else None
    name = "mxfa_varlen_fwd_exact_launch" if exact_p else "mxfa_varlen_fwd_launch"
    with _on(q):
        rc = getattr(_L(), name)(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), None, None, out.data_ptr(), _lib.ptr(lse), B, Sq,
            k.shape[1], B * Sq, B * k.shape[1], HQ, k.shape[2], D, int(bool(causal)), _bf16(q),
            float(softmax_scale), _stream(q))
    _lib.check(rc, name)
    return (out, lse) if return_lse else out


# ------------------------------------------------------------------ decode

_PLANS: dict[tuple, tuple[int, int]] = {}


def kvcache_plan(batch: int, q_len: int, q_heads: int, kv_heads: int, head_dim: int, max_len: int):
    """(num_splits, chunk_len) the library picks for this shape on the current device (cached)."""
    import ctypes

    key = (torch.cuda.current_device() if (_CUDA_OK or torch.cuda.is_available()) else -1, batch, q_len, q_heads,
           kv_heads, head_dim, max_len)
    plan = _PLANS.get(key)
    if plan is None:
        np_, cl = ctypes.c_int(0), ctypes.c_int(0)
        _lib.check(_L().mxfa_kvcache_plan(batch, q_len, q_heads, kv_heads, head_dim, max_len,
                                                  ctypes.byref(np_), ctypes.byref(cl)), "mxfa_kvcache_plan")
        plan = _PLANS[key] = (int(np_.value), int(cl.value))
    return plan


_COUNTERS: dict[tuple, "torch.Tensor"] = {}


def split_counters(device, stream_handle: int, nbytes: int):
    """Zeroed counter array for single-launch splits on one (device, stream).

    Every counted launch leaves its counters at zero again, so one array per
    stream is reused by all launches ordered on that stream; it only grows.
    """
    key = (device, stream_handle)
    buf = _COUNTERS.get(key)
    n = max(nbytes // 4, 1)
    if buf is None or buf.numel() < n:
        buf = _COUNTERS[key] = torch.zeros((max(n, 4096),), device=device, dtype=torch.int32)
    return buf


def kvcache_length_order(cache_seqlens):
    """Longest-first order of the batch (int32 [B]: order[rank] = sequence), for ``length_order=``.

    Computed on the device (``mxfa_kvcache_length_order_launch``) once per
    step and passed to every layer's ``kvcache_attention``, it replaces the
    ranking each CTA otherwise does on every layer.  Batches of one or of more
    than 512 sequences need none (None is returned)."""
    seq = _i32(cache_seqlens)
    B = seq.shape[0]
    if B <= 1 or B > 512:
        return None
    order = torch.empty((B,), device=seq.device, dtype=torch.int32)
    with _on(seq):
        rc = _L().mxfa_kvcache_length_order_launch(seq.data_ptr(), B, order.data_ptr(), _stream(seq))
    _lib.check(rc, "mxfa_kvcache_length_order_launch")
    return order


def kvcache_attention(q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale, causal, *,
                      append_len: int = 0, return_lse: bool = False, num_splits: int = 0, chunk_len: int = 0,
                      out=None, k_new=None, v_new=None, single_launch: bool = True, k_scale: float = 1.0,
                      v_scale: float = 1.0, length_order=None):
    """Attention of q [B, Sq, HQ, D] over the cached tokens (+ ``append_len``).

    ``cache_seqlens`` holds the lengths before the append.  Without
    ``k_new``/``v_new`` nothing is written to the caches (the appended rows
    must already be there); with them the same launch writes those rows into
    the caches first (``mxfa_kvcache_append_attention_launch``).
    ``num_splits``/``chunk_len`` 0 = library plan.  A split plan runs as one
    launch (the last split CTA of each unit merges) unless ``single_launch``
    is False, which keeps the separate combine kernel.  ``torch.float8_e4m3fn``
    caches attend to ``k_cache * k_scale`` and ``v_cache * v_scale``.
    ``length_order`` (from ``kvcache_length_order``) schedules the sequences
    without the per-CTA ranking; it is ignored by the fused append.
    """
    B, Sq, HQ, D = q.shape
    q = _contig(q)
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("the CUDA backend requires contiguous k_cache / v_cache")
    seq = _i32(cache_seqlens)
    bt = None if block_table is None else _i32(block_table)
    PS = k_cache.shape[1]
    HKV = k_cache.shape[2]
    if bt is not None:
        btw, pages = bt.shape[1], k_cache.shape[0]
        max_len = btw * PS
    else:
        btw, pages = 0, k_cache.shape[0]
        max_len = PS
    if out is None:
        out = torch.empty_like(q)
    lse = torch.empty((B, Sq, HQ), device=q.device, dtype=torch.float32) if return_lse else None
    lib = _L()
    if num_splits <= 0 or chunk_len <= 0:
        num_splits, chunk_len = kvcache_plan(B, Sq, HQ, HKV, D, max_len)
    ws = None
    ws_bytes = 0
    if num_splits > 1:
        ws_bytes = int(lib.mxfa_split_workspace_bytes(B * Sq * HQ, D, num_splits))
        ws = torch.empty((ws_bytes // 4,), device=q.device, dtype=torch.float32)
    with _on(q):
        stream = _stream(q)
        counters = None
        if num_splits > 1 and single_launch:
            counters = split_counters(q.device, stream, int(lib.mxfa_split_counter_bytes(B, Sq, HQ, HKV)))
        if length_order is not None and k_new is None:
            order = _i32(length_order)
            if order.shape != (B,) or order.device != q.device:
                raise ValueError(f"length_order must be int32 [{B}] on {q.device}")
            fp8 = _is_fp8(k_cache)
            name = "mxfa_kvcache_attention_ordered_launch"
            rc = lib.mxfa_kvcache_attention_ordered_launch(
                q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), _lib.ptr(bt), seq.data_ptr(), order.data_ptr(),
                out.data_ptr(), _lib.ptr(lse), _lib.ptr(ws), ws_bytes, _lib.ptr(counters), B, Sq, HQ, HKV, D, PS,
                btw, pages, int(append_len), num_splits, chunk_len, int(bool(causal)), _bf16(q),
                float(softmax_scale), int(fp8), float(k_scale), float(v_scale), stream)
        elif _is_fp8(k_cache):
            if k_new is not None:
                raise ValueError("the fused append does not take float8_e4m3fn rows; append with kv_append first")
            name = "mxfa_kvcache_attention_fp8_launch"
            rc = lib.mxfa_kvcache_attention_fp8_launch(
                q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), _lib.ptr(bt), seq.data_ptr(),
                out.data_ptr(), _lib.ptr(lse), _lib.ptr(ws), ws_bytes, _lib.ptr(counters), B, Sq, HQ, HKV, D, PS,
                btw, pages, int(append_len), num_splits, chunk_len, int(bool(causal)), _bf16(q),
                float(softmax_scale), float(k_scale), float(v_scale), stream)
        elif k_new is None:
            if counters is None:
                name = "mxfa_kvcache_attention_launch"
                rc = lib.mxfa_kvcache_attention_launch(
                    q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), _lib.ptr(bt), seq.data_ptr(),
                    out.data_ptr(), _lib.ptr(lse), _lib.ptr(ws), ws_bytes, B, Sq, HQ, HKV, D, PS, btw, pages,
                    int(append_len), num_splits, chunk_len, int(bool(causal)), _bf16(q), float(softmax_scale),
                    stream)
            else:
                name = "mxfa_kvcache_attention_counted_launch"
                rc = lib.mxfa_kvcache_attention_counted_launch(
                    q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), _lib.ptr(bt), seq.data_ptr(),
                    out.data_ptr(), _lib.ptr(lse), _lib.ptr(ws), ws_bytes, counters.data_ptr(), B, Sq, HQ, HKV,
                    D, PS, btw, pages, int(append_len), num_splits, chunk_len, int(bool(causal)), _bf16(q),
                    float(softmax_scale), stream)
        else:
            name = "mxfa_kvcache_append_attention_launch"
            k_new, v_new = _contig(k_new), _contig(v_new)
            rc = lib.mxfa_kvcache_append_attention_launch(
                q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), _lib.ptr(bt), seq.data_ptr(),
                out.data_ptr(), _lib.ptr(lse), _lib.ptr(ws), ws_bytes, _lib.ptr(counters), k_new.data_ptr(),
                v_new.data_ptr(), B, Sq, HQ, HKV, D, PS, btw, pages, int(k_new.shape[1]), num_splits, chunk_len,
                int(bool(causal)), _bf16(q), float(softmax_scale), stream)
    _lib.check(rc, name)
    return (out, lse) if return_lse else out


def _is_fp8(t) -> bool:
    return t.dtype == getattr(torch, "float8_e4m3fn", None)


def fused_append_supported(q, k_cache, k) -> bool:
    """True when one launch can append ``k``/``v`` and attend (up to 16 query rows per KV head)."""
    B, Sq, HQ, D = q.shape
    HKV = k_cache.shape[2]
    return (k is not None and k.shape[1] > 0 and HQ % HKV == 0 and Sq * (HQ // HKV) <= 16
            and k.dtype == k_cache.dtype and not _is_fp8(k_cache))


def kv_append(k_cache, v_cache, k, v, cache_seqlens, block_table) -> None:
    """Write k/v [B, Sk, HKV, D] at positions cache_seqlens[b] + i (no length update)."""
    k, v = _contig(k), _contig(v)
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("the CUDA backend requires contiguous k_cache / v_cache")
    seq = _i32(cache_seqlens)
    bt = None if block_table is None else _i32(block_table)
    B, Sk, HKV, D = k.shape
    with _on(k):
        rc = _L().mxfa_kv_append_launch(
            k.data_ptr(), v.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), _lib.ptr(bt), seq.data_ptr(), B,
            Sk, HKV, D, k_cache.shape[1], 0 if bt is None else bt.shape[1], k_cache.shape[0], k.element_size(),
            _stream(k))
    _lib.check(rc, "mxfa_kv_append_launch")


def seqlens_add_(cache_seqlens: torch.Tensor, delta: int) -> None:
    """In-place ``cache_seqlens += delta`` on the device (int32 or int64)."""
    if cache_seqlens.dtype not in (torch.int32, torch.int64) or not cache_seqlens.is_contiguous():
        cache_seqlens.add_(delta)
        return
    with _on(cache_seqlens):
        rc = _L().mxfa_seqlens_add_launch(
            cache_seqlens.data_ptr(), int(cache_seqlens.dtype == torch.int64), cache_seqlens.numel(), int(delta),
            _stream(cache_seqlens))
    _lib.check(rc, "mxfa_seqlens_add_launch")


def flash_attn_with_kvcache(q, k_cache, v_cache, k, v, cache_seqlens, block_table, softmax_scale, causal,
                            k_scale: float = 1.0, v_scale: float = 1.0, out=None, length_order=None):
    """``flash_attn_with_kvcache`` semantics of the reference (reference.py:88-139).

    Appends ``k``/``v`` (when given) at the current lengths, attends over the
    grown cache, then advances ``cache_seqlens`` in place -- all on the
    current stream, with no host synchronisation.  ``out`` (optional, q's
    shape and dtype, contiguous) receives the result.  ``length_order``
    (optional, from ``kvcache_length_order``) schedules the sequences without
    the per-launch ranking.
    """
    if q.shape[1] == 0:
        if k is not None:
            kv_append(k_cache, v_cache, k, v, cache_seqlens, block_table)
            seqlens_add_(cache_seqlens, k.shape[1])
        return out if out is not None else torch.empty_like(q)
    append_len = 0
    if k is not None and fused_append_supported(q, k_cache, k):
        # decode shapes: the attention kernel writes the new rows itself (one launch fewer)
        append_len = k.shape[1]
        out = kvcache_attention(q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale, causal,
                                append_len=append_len, k_new=k, v_new=v, out=out)
        seqlens_add_(cache_seqlens, append_len)
        return out
    if k is not None:
        kv_append(k_cache, v_cache, k, v, cache_seqlens, block_table)
        append_len = k.shape[1]
    out = kvcache_attention(q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale, causal,
                            append_len=append_len, k_scale=k_scale, v_scale=v_scale, out=out,
                            length_order=length_order)
    if k is not None:
        seqlens_add_(cache_seqlens, append_len)
    return out


def kvcache_attention_packed(q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale, *,
                             num_splits: int = 0, chunk_len: int = 0, out=None):
    """Local half of a context-split decode: packed f32 [B*HQ, D+1] = (normalised O, LSE) per row."""
    B, Sq, HQ, D = q.shape
    if Sq != 1:
        raise ValueError("packed local attention takes one query token per sequence")
    q = _contig(q)
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("the CUDA backend requires contiguous k_cache / v_cache")
    seq = _i32(cache_seqlens)
    bt = None if block_table is None else _i32(block_table)
    PS, HKV = k_cache.shape[1], k_cache.shape[2]
    btw = 0 if bt is None else bt.shape[1]
    max_len = btw * PS if bt is not None else PS
    if num_splits <= 0 or chunk_len <= 0:
        num_splits, chunk_len = kvcache_plan(B, 1, HQ, HKV, D, max_len)
    lib = _L()
    ws_bytes = int(lib.mxfa_split_workspace_bytes(B * HQ, D, num_splits))
    ws = torch.empty((max(ws_bytes, 16) // 4,), device=q.device, dtype=torch.float32)
    if out is None:
        out = torch.empty((B * HQ, D + 1), device=q.device, dtype=torch.float32)
    with _on(q):
        rc = lib.mxfa_kvcache_attention_packed_launch(
            q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), _lib.ptr(bt), seq.data_ptr(), out.data_ptr(),
            ws.data_ptr(), ws_bytes, B, HQ, HKV, D, PS, btw, k_cache.shape[0], num_splits, chunk_len, _bf16(q),
            float(softmax_scale), _stream(q))
    _lib.check(rc, "mxfa_kvcache_attention_packed_launch")
    return out


# ------------------------------------------------------ combine / merge

def split_combine(ows, mdws, rows: int, head_dim: int, num_splits: int, dtype, *, lse: bool = False,
                  out=None):
    """LSE-merge split partials ows [rows, NP, D], mdws [rows, NP, 2] -> out [rows, D]."""
    if out is None:
        out = torch.empty((rows, head_dim), device=ows.device, dtype=dtype)
    lse_t = torch.empty((rows,), device=ows.device, dtype=torch.float32) if lse else None
    with _on(ows):
        rc = _L().mxfa_split_combine_launch(
            ows.data_ptr(), mdws.data_ptr(), out.data_ptr(), None, _lib.ptr(lse_t), rows, head_dim, num_splits,
            int(dtype == torch.bfloat16), _stream(ows))
    _lib.check(rc, "mxfa_split_combine_launch")
    return (out, lse_t) if lse else out


def lse_merge(packed, rows: int, head_dim: int, dtype, *, lse: bool = False, out=None):
    """Merge per-rank (O, LSE): packed f32 [N, rows, D + 1] -> out [rows, D] (and LSE)."""
    n_ranks = packed.shape[0]
    if out is None:
        out = torch.empty((rows, head_dim), device=packed.device, dtype=dtype)
    lse_t = torch.empty((rows,), device=packed.device, dtype=torch.float32) if lse else None
    with _on(packed):
        rc = _L().mxfa_lse_merge_launch(
            packed.data_ptr(), out.data_ptr(), _lib.ptr(lse_t), n_ranks, rows, head_dim,
            int(dtype == torch.bfloat16), _stream(packed))
    _lib.check(rc, "mxfa_lse_merge_launch")
    return (out, lse_t) if lse else out
