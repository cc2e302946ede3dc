"""Decode across GPUs: batch / KV-head sharding and long-context splitting.

Two partitionings of the decode path, one process per GPU:

* **Batch or KV-head groups** (``shard_batch`` / ``shard_kv_heads``): every
  (sequence, KV head) unit is independent, so each rank decodes its share
  with no communication at all.
* **Context split** for long sequences (``context_parallel_decode``): each
  rank holds a contiguous, page-aligned range of every sequence's positions
  in its own HBM, computes attention over that range as fp32 (O, LSE) with
  ``mxfa_kvcache_attention_packed_launch``, the ranks exchange those records
  with ONE all-gather of ``[rows, D + 1]`` fp32 per layer, and every rank
  merges them locally with ``mxfa_lse_merge_launch``.  Only those small
  records cross NVLink; KV pages never leave the GPU that owns them.

The reference runs on one device only; this module is new.  The exchange
(``gather_partials``) is a plain ``torch.distributed`` collective, so the
host logic runs unchanged on a CPU ``gloo`` group in tests.
"""

from __future__ import annotations

import numpy as np


# ------------------------------------------------------------------ sharding

def shard_batch(batch: int, world_size: int, rank: int) -> range:
    """Contiguous slice of sequences owned by ``rank`` (sizes differ by at most one)."""
    base, extra = divmod(batch, world_size)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def shard_kv_heads(kv_heads: int, world_size: int, rank: int) -> range:
    """KV heads owned by ``rank``; its query heads are those heads' GQA groups."""
    if kv_heads % world_size:
        raise ValueError(f"{kv_heads} KV heads do not divide over {world_size} ranks")
    per = kv_heads // world_size
    return range(rank * per, (rank + 1) * per)


def shard_ranges(lengths, world_size: int, page_size: int) -> np.ndarray:
    """Position range [start, end) of every sequence on every rank, page-aligned.

    Sequence b's ``ceil(len/page_size)`` pages are divided into ``world_size``
    contiguous groups whose sizes differ by at most one page; rank r owns the
    positions of its group.  Returns int64 ``[world_size, B, 2]``.  Every
    position belongs to exactly one rank.
    """
    lengths = np.asarray(lengths, dtype=np.int64)
    out = np.zeros((world_size, lengths.shape[0], 2), dtype=np.int64)
    for b, length in enumerate(lengths):
        pages = -(-int(length) // page_size)
        for r in range(world_size):
            p0 = (r * pages) // world_size
            p1 = ((r + 1) * pages) // world_size
            out[r, b, 0] = min(p0 * page_size, length)
            out[r, b, 1] = min(p1 * page_size, length)
    return out


def local_view(lengths, block_table, world_size: int, rank: int, page_size: int):
    """Rank-local lengths and block table for the context split.

    ``block_table`` [B, W] maps a sequence's logical pages to physical pages.
    Rank ``rank`` keeps the pages of its position range; the returned table
    lists them in order (padded with the row's first kept page, never read)
    and the lengths count only the local positions.
    """
    block_table = np.asarray(block_table)
    ranges = shard_ranges(lengths, world_size, page_size)[rank]
    local_len = (ranges[:, 1] - ranges[:, 0]).astype(np.int32)
    pages = [(-(-int(e) // page_size) - int(s) // page_size) if e > s else 0 for s, e in ranges]
    width = max(max(pages, default=0), 1)
    table = np.zeros((block_table.shape[0], width), dtype=np.int32)
    for b, (s, e) in enumerate(ranges):
        if e > s:
            p0 = int(s) // page_size
            n = pages[b]
            table[b, :n] = block_table[b, p0:p0 + n]
            table[b, n:] = block_table[b, p0]
    return local_len, table


# ------------------------------------------------------------------ exchange

def gather_partials(packed_local, group=None):
    """All-gather the per-rank packed (O, LSE) records: [rows, D+1] -> [world, rows, D+1].

    One collective per layer; on GPUs it runs over NCCL (NVLink/NVSwitch), on
    CPU tensors over gloo.
    """
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rows = packed_local.shape[0]
    flat = torch.empty((world * rows,) + tuple(packed_local.shape[1:]), dtype=packed_local.dtype,
                       device=packed_local.device)
    dist.all_gather_into_tensor(flat, packed_local.contiguous(), group=group)
    return flat.view((world, rows) + tuple(packed_local.shape[1:]))


def context_parallel_decode(q, k_cache, v_cache, local_seqlens, local_block_table, softmax_scale=None, *,
                            group=None, num_splits: int = 0, chunk_len: int = 0, return_lse: bool = False):
    """Single-token decode with every sequence's context split across the ranks of ``group``.

    ``k_cache``/``v_cache``/``local_block_table``/``local_seqlens`` describe
    this rank's pages only (see ``local_view``).  Returns the merged output
    ``[B, 1, HQ, D]`` on every rank (and the merged natural-log LSE
    ``[B, HQ]`` when ``return_lse``).
    """
    from . import backend

    B, Sq, HQ, D = q.shape
    if Sq != 1:
        raise ValueError("context-parallel decode takes one query token per sequence")
    scale = softmax_scale if softmax_scale is not None else D ** -0.5
    packed = backend.kvcache_attention_packed(q, k_cache, v_cache, local_seqlens, local_block_table, scale,
                                              num_splits=num_splits, chunk_len=chunk_len)
    gathered = gather_partials(packed, group)
    merged = backend.lse_merge(gathered, B * HQ, D, q.dtype, lse=return_lse)
    if return_lse:
        out, lse = merged
        return out.reshape(B, 1, HQ, D), lse.reshape(B, HQ)
    return merged.reshape(B, 1, HQ, D)
