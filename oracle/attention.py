"""numpy restatement of the reference oracle (test infrastructure only).

All arrays are numpy.  Inputs hold values already rounded to the caller's
storage dtype (bf16/fp16 grids, see ``mxflashattn_b200.synthetic``); the math
runs in float32 like the reference (``q.float()``, ``reference.py:26-28``) or
in float64 when ``precision=np.float64`` is passed (the cross-check style of
the reference's ``csrc_native/test_ext.py:42-60``).
"""

from __future__ import annotations

import math

import numpy as np

LOG2E = 1.4426950408889634
LN2 = 0.6931471805599453


def _scale(head_dim: int, softmax_scale: float | None) -> float:
    # reference.py:24 -- None means 1/sqrt(head_dim); 0.0 is kept as 0.0.
    return softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(head_dim)


def attention_single(
    q: np.ndarray,
    k: np.ndarray,
    v: np.ndarray,
    *,
    softmax_scale: float | None = None,
    causal: bool = False,
    precision=np.float32,
    return_lse: bool = False,
):
    """softmax(q k^T * scale) v for [seq, heads, dim] inputs (reference.py:8-40).

    GQA repeats each KV head over ``q_heads // kv_heads`` consecutive query
    heads (``repeat_interleave``, reference.py:27-28).  Causal masking is
    bottom-right aligned: query row i sees keys j <= i + (key_len - query_len)
    (reference.py:31-35).  Rows with no visible key produce 0 (the NaN->0 of
    reference.py:38).  Returns float arrays in ``precision``; cast with
    ``synthetic.round_dtype`` to emulate the final ``.to(q.dtype)``.
    """
    query_len, query_heads, head_dim = q.shape
    key_len, kv_heads, _ = k.shape
    if query_len == 0:
        out = np.zeros_like(q, dtype=precision)
        return (out, np.zeros((query_heads, 0), precision)) if return_lse else out
    if key_len == 0:
        raise ValueError("attention requires at least one key/value token")
    scale = precision(_scale(head_dim, softmax_scale))
    groups = query_heads // kv_heads
    qf = q.astype(precision).transpose(1, 0, 2)                       # [H, Sq, D]
    kf = np.repeat(k.astype(precision), groups, axis=1).transpose(1, 0, 2)
    vf = np.repeat(v.astype(precision), groups, axis=1).transpose(1, 0, 2)
    scores = np.matmul(qf, kf.transpose(0, 2, 1)) * scale               # [H, Sq, Sk]
    if causal:
        q_pos = np.arange(query_len) + (key_len - query_len)
        k_pos = np.arange(key_len)
        blocked = k_pos[None, :] > q_pos[:, None]
        scores = np.where(blocked[None], -np.inf, scores).astype(precision)
    with np.errstate(invalid="ignore", over="ignore"):
        row_max = scores.max(axis=-1, keepdims=True)
        e = np.exp(scores - row_max)
        denom = e.sum(axis=-1, keepdims=True)
        probs = e / denom
    probs = np.nan_to_num(probs, nan=0.0, posinf=0.0, neginf=0.0).astype(precision)
    out = np.matmul(probs, vf).transpose(1, 0, 2)                     # [Sq, H, D]
    if not return_lse:
        return out
    with np.errstate(divide="ignore", invalid="ignore"):
        lse = (row_max[..., 0] + np.log(denom[..., 0])).astype(precision)  # [H, Sq]
    lse = np.where(np.isfinite(row_max[..., 0]), lse, -np.inf).astype(precision)
    return out, lse


def attention_batched(q, k, v, *, softmax_scale=None, causal=False, precision=np.float32):
    """Per-batch loop over ``attention_single`` (reference.py:43-57)."""
    outs = [
        attention_single(q[b], k[b], v[b], softmax_scale=softmax_scale, causal=causal, precision=precision)
        for b in range(q.shape[0])
    ]
    if not outs:
        return np.zeros_like(q, dtype=precision)
    return np.stack(outs, axis=0)


def attention_varlen(q, k, v, cu_q, cu_k, *, softmax_scale=None, causal=False, precision=np.float32,
                     return_lse=False):
    """Packed variable-length attention (reference.py:60-85)."""
    outs, lses = [], []
    for i in range(len(cu_q) - 1):
        qs, qe = int(cu_q[i]), int(cu_q[i + 1])
        ks, ke = int(cu_k[i]), int(cu_k[i + 1])
        res = attention_single(q[qs:qe], k[ks:ke], v[ks:ke], softmax_scale=softmax_scale,
                               causal=causal, precision=precision, return_lse=return_lse)
        if return_lse:
            outs.append(res[0])
            lses.append(res[1])
        else:
            outs.append(res)
    out = np.concatenate(outs, axis=0) if outs else np.zeros_like(q[:0], dtype=precision)
    if return_lse:
        return out, (np.concatenate(lses, axis=1) if lses else np.zeros((q.shape[1], 0), precision))
    return out


def gather_paged_kv(cache: np.ndarray, block_row, length: int) -> np.ndarray:
    """Logical [length, heads, dim] view of one sequence of a paged cache.

    Pages are taken in block-table order and the last page is truncated
    (reference.py:123-126).
    """
    page_size = cache.shape[1]
    n_pages = (length + page_size - 1) // page_size
    pages = [cache[int(block_row[p])] for p in range(n_pages)]
    if not pages:
        return cache[:0, 0]
    return np.concatenate(pages, axis=0)[:length]


def attention_kvcache(
    q,
    k_cache,
    v_cache,
    *,
    cache_seqlens,
    block_table=None,
    k=None,
    v=None,
    softmax_scale=None,
    causal=False,
    precision=np.float32,
    return_lse=False,
):
    """KV-cache attention with optional append (reference.py:88-139).

    Mutates ``k_cache``/``v_cache`` (append into the slot of logical position
    ``old_len + i``, page ``block_table[b, pos // page_size]``, offset
    ``pos % page_size``; reference.py:115-122) and ``cache_seqlens``
    (``+= k.shape[1]``, reference.py:137-138) in place, like the reference.
    """
    lengths = [int(x) for x in np.asarray(cache_seqlens).tolist()]
    batch = q.shape[0]
    outs, lses = [], []
    append_len = 0 if k is None else k.shape[1]
    for b in range(batch):
        old_len = lengths[b]
        total = old_len + append_len
        if block_table is None:
            if append_len:
                k_cache[b, old_len:total] = k[b]
                v_cache[b, old_len:total] = v[b]
            cur_k = k_cache[b, :total]
            cur_v = v_cache[b, :total]
        else:
            page_size = k_cache.shape[1]
            row = [int(x) for x in np.asarray(block_table[b]).tolist()]
            for t in range(append_len):
                logical = old_len + t
                page_index, offset = divmod(logical, page_size)
                phys = row[page_index]
                k_cache[phys, offset] = k[b, t]
                v_cache[phys, offset] = v[b, t]
            cur_k = gather_paged_kv(k_cache, row, total)
            cur_v = gather_paged_kv(v_cache, row, total)
        res = attention_single(q[b], cur_k, cur_v, softmax_scale=softmax_scale, causal=causal,
                               precision=precision, return_lse=return_lse)
        if return_lse:
            outs.append(res[0])
            lses.append(res[1])
        else:
            outs.append(res)
    if k is not None:
        cache_seqlens += append_len
    out = np.stack(outs, axis=0) if outs else np.zeros_like(q, dtype=precision)
    if return_lse:
        return out, np.stack(lses, axis=0)
    return out


def split_partials(q_row, keys, values, scale, num_splits, chunk_len):
    """Per-chunk split-KV partial state of one query row (m1_kernel.cpp:563-577, :846-853).

    ``q_row`` [D]; ``keys``/``values`` [L, D] float arrays of one KV head.
    Chunk z covers positions [z*chunk_len, (z+1)*chunk_len) of the sequence.
    Returns ``o`` [NP, D] (unnormalised sum of p*v), ``m`` [NP] (max of the
    log2-domain score s*scale*log2(e)) and ``d`` [NP] (sum of 2^(s-m));
    empty chunks give m=-inf, d=0, o=0 -- the partial-state contract of the
    reference's split kernel and its combine.
    """
    length = keys.shape[0]
    d_model = q_row.shape[0]
    o = np.zeros((num_splits, d_model), np.float64)
    m = np.full((num_splits,), -np.inf, np.float64)
    d = np.zeros((num_splits,), np.float64)
    s_all = (keys.astype(np.float64) @ q_row.astype(np.float64)) * (scale * LOG2E)
    for z in range(num_splits):
        lo, hi = z * chunk_len, min((z + 1) * chunk_len, length)
        if hi <= lo:
            continue
        s = s_all[lo:hi]
        m[z] = s.max()
        p = np.exp2(s - m[z])
        d[z] = p.sum()
        o[z] = p @ values[lo:hi].astype(np.float64)
    return o, m, d


def merge_partials(o, m, d):
    """LSE merge of split partials (split_combine, m1_kernel.cpp:862-888).

    Returns the normalised output [D] and the natural-log LSE.  All-empty
    input gives zeros and -inf.
    """
    finite = np.isfinite(m)
    if not finite.any():
        return np.zeros(o.shape[1]), -np.inf
    mm = m[finite].max()
    w = np.where(finite, np.exp2(np.where(finite, m, mm) - mm), 0.0)
    den = (w * d).sum()
    out = (w[:, None] * o).sum(axis=0) / den if den > 0 else np.zeros(o.shape[1])
    lse = (mm + math.log2(den)) * LN2 if den > 0 else -np.inf
    return out, lse


def attention_chunked(q, k, v, *, chunk_size=256, softmax_scale=None, causal=False):
    """Online-softmax attention over key chunks, float32 (prefill.py:11-81).

    ``q`` [B, Sq, HQ, D], ``k``/``v`` [B, Sk, HKV, D] (GQA: each KV head serves
    ``HQ // HKV`` consecutive query heads).  Keys are visited in chunks of
    ``chunk_size``; each row keeps a running maximum ``m``, normaliser ``l``
    and unnormalised output ``o``, and a chunk rescales them by
    ``exp(m_old - m_new)`` before adding its own ``exp(s - m_new)`` terms.
    Causal masking is bottom-right aligned like the direct oracle; a row whose
    keys are all masked so far contributes nothing, and a row that never sees
    a key outputs 0.  The second oracle for the online softmax the kernels
    run: it must agree with ``attention_batched`` to float32 rounding.
    """
    if not isinstance(chunk_size, (int, np.integer)) or chunk_size <= 0:
        raise ValueError("chunk_size must be a positive integer")
    B, Sq, HQ, D = q.shape
    Sk, HKV = k.shape[1], k.shape[2]
    scale = np.float32(_scale(D, softmax_scale))
    G = HQ // HKV
    qf = q.astype(np.float32).transpose(0, 2, 1, 3)                          # [B, HQ, Sq, D]
    kf = np.repeat(k.astype(np.float32).transpose(0, 2, 1, 3), G, axis=1)   # [B, HQ, Sk, D]
    vf = np.repeat(v.astype(np.float32).transpose(0, 2, 1, 3), G, axis=1)
    o = np.zeros((B, HQ, Sq, D), np.float32)
    l = np.zeros((B, HQ, Sq, 1), np.float32)
    m = np.full((B, HQ, Sq, 1), -np.inf, np.float32)
    row_pos = np.arange(Sq) + (Sk - Sq)  # the last key each query row may see
    for lo in range(0, Sk, chunk_size):
        hi = min(lo + chunk_size, Sk)
        s = (qf @ kf[:, :, lo:hi].transpose(0, 1, 3, 2)) * scale          # [B, HQ, Sq, hi-lo]
        if causal:
            s = np.where(np.arange(lo, hi)[None, :] > row_pos[:, None], np.float32(-np.inf), s)
        m_new = np.maximum(m, s.max(axis=-1, keepdims=True))
        seen = np.isfinite(m_new)
        keep = np.where(np.isfinite(m), np.exp(m - np.where(seen, m_new, 0.0)), 0.0).astype(np.float32)
        p = np.where(np.isfinite(s), np.exp(s - np.where(seen, m_new, 0.0)), 0.0).astype(np.float32)
        l = l * keep + p.sum(axis=-1, keepdims=True)
        o = o * keep + p @ vf[:, :, lo:hi]
        m = m_new
    out = np.where(l > 0, o / np.where(l > 0, l, 1.0), 0.0).astype(np.float32)
    return out.transpose(0, 2, 1, 3)


def attention_chunked_fallback(q, k, v, *, chunk_size=256, softmax_scale=None, causal=False):
    """The direct oracle when one chunk covers every key, else the chunked one (prefill.py:84-108)."""
    if chunk_size >= k.shape[1]:
        return attention_batched(q, k, v, softmax_scale=softmax_scale, causal=causal)
    return attention_chunked(q, k, v, chunk_size=chunk_size, softmax_scale=softmax_scale, causal=causal)
