"""Decode across GPUs: batch / KV-head sharding and long-context splitting.

Partitionings of the attention path, one process per GPU:

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
* **Prefill by KV-head groups** (``prefill_local_heads``): each rank runs the
  varlen forward over its KV heads and the query heads that read them; heads
  are independent, so there is no communication.

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


def prefill_local_heads(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, *, world_size: int,
                        rank: int, causal: bool = True, softmax_scale=None, return_lse: bool = False):
    """This rank's share of a varlen prefill: KV heads ``shard_kv_heads(HKV, world, rank)``.

    ``q`` is ``[Tq, HQ, D]`` and ``k``/``v`` are ``[Tk, HKV, D]`` with every head.
    The output (and LSE) cover query heads ``[hk0*GQ, hk1*GQ)`` only, where
    GQ = HQ / HKV, because query head h reads KV head h // GQ.  Concatenating
    the ranks' outputs along the head axis gives the full result bit for
    bit.  A tensor-parallel model that already holds only its own heads calls
    ``backend.flash_attn_varlen_func`` on them directly.
    """
    from . import backend

    hq, hkv, d = q.shape[1], k.shape[1], q.shape[2]
    if hq % hkv:
        raise ValueError(f"{hq} query heads are not a multiple of {hkv} KV heads")
    heads = shard_kv_heads(hkv, world_size, rank)
    gq = hq // hkv
    qs = q[:, heads.start * gq:heads.stop * gq].contiguous()
    ks = k[:, heads.start:heads.stop].contiguous()
    vs = v[:, heads.start:heads.stop].contiguous()
    scale = softmax_scale if softmax_scale is not None else d ** -0.5
    return backend.flash_attn_varlen_func(qs, ks, vs, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                                          causal, scale, return_lse=return_lse)


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


# ------------------------------------------------- fused exchange (peer memory)


_IPC_HANDLE_BYTES = 64  # sizeof(cudaIpcMemHandle_t)


def map_exchange_buffers(lib, nbytes: int, world: int, rank: int, group=None):
    """Allocate this rank's exchange buffer, export it and map every peer's (collective, current device).

    Every rank takes the same collective steps whatever fails: the exported
    handles are all-gathered (None from a rank whose allocation or export
    failed), then every rank's import status.  A failure on any rank makes
    every rank unmap and free what it holds and raise, instead of leaving the
    other ranks blocked in their next collective.
    Returns (this rank's buffer address, the peer mappings it opened, the
    buffer address of every rank in rank order).
    """
    import ctypes

    import torch.distributed as dist

    from . import _lib

    def status(rc, what):
        if rc != _lib.MXFA_OK:
            raise _lib.NativeLibraryError(f"{what}: status {rc}: {lib.mxfa_last_error().decode(errors='replace')}")

    local, handle, error = None, None, None
    try:
        addr = ctypes.c_void_p()
        status(lib.mxfa_peer_alloc(nbytes, ctypes.byref(addr)), "mxfa_peer_alloc")
        local = addr.value
        buf = (ctypes.c_char * _IPC_HANDLE_BYTES)()
        status(lib.mxfa_peer_export(local, buf), "mxfa_peer_export")
        handle = bytes(buf)
    except Exception as exc:  # reported to every rank below
        error = exc
    handles = [None] * world
    dist.all_gather_object(handles, handle, group=group)
    imported, ptrs = [], []
    if error is None and all(h is not None for h in handles):
        try:
            for r, h in enumerate(handles):
                if r == rank:
                    ptrs.append(local)
                    continue
                peer = ctypes.c_void_p()
                status(lib.mxfa_peer_import((ctypes.c_char * _IPC_HANDLE_BYTES).from_buffer_copy(h),
                                            ctypes.byref(peer)), "mxfa_peer_import")
                imported.append(peer.value)
                ptrs.append(peer.value)
        except Exception as exc:
            error = exc
    oks = [None] * world
    dist.all_gather_object(oks, error is None, group=group)
    if all(oks):
        return local, imported, ptrs
    for p in imported:
        lib.mxfa_peer_close(p)
    dist.barrier(group=group)  # no rank still maps a buffer that is about to be freed
    if local is not None:
        lib.mxfa_peer_free(local)
    failed = [r for r, ok in enumerate(oks) if not ok]
    raise RuntimeError(f"context-parallel exchange buffers could not be mapped: failed on rank(s) {failed}"
                       + (f" ({error})" if error is not None else "")) from error


class FusedContextParallelDecode:
    """Context-split decode with the (O, LSE) exchange fused into the kernels.

    Same result as ``context_parallel_decode`` without the NCCL all-gather:
    each rank's decode publishes its records straight into every rank's
    exchange buffer over NVLink (plain stores to CUDA-IPC-mapped memory);
    the same kernel then waits for all ranks' records of each unit and merges
    it (``one_launch``, when the grid's units fit on the GPU at once), or a
    small merge kernel on each rank does (``one_launch=False``, and the
    library's own choice for larger grids).
    One instance serves a fixed geometry (batch, heads, head dim) for any
    number of calls and layers; every rank must make the same calls in the
    same order.  ``close()`` (collective) releases the mappings.
    """

    def __init__(self, batch: int, q_heads: int, kv_heads: int, head_dim: int, *, group=None, device=None,
                 one_launch: bool = True):
        import torch
        import torch.distributed as dist

        from . import _lib

        self._lib = lib = _lib.load()
        self.group = group
        self.one_launch = one_launch
        self.launches_per_call = 0  # kernels the last call launched (1: merged inside the decode kernel)
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.geometry = (batch, q_heads, kv_heads, head_dim)
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        nbytes = int(lib.mxfa_cp_buffer_bytes(self.world, batch, q_heads, kv_heads, head_dim))
        if nbytes == 0:
            raise ValueError(f"unsupported context-parallel geometry {self.geometry}")
        with torch.cuda.device(self.device):
            self._local, self._imported, ptrs = map_exchange_buffers(lib, nbytes, self.world, self.rank, group)
            # device array of the peers' buffer addresses (uint64 stored as int64)
            self.peer_table = torch.tensor([p - (1 << 64) if p >= (1 << 63) else p for p in ptrs],
                                           dtype=torch.int64, device=self.device)
        dist.barrier(group=group)

    def __call__(self, q, k_cache, v_cache, local_seqlens, local_block_table, softmax_scale=None, *,
                 num_splits: int = 0, chunk_len: int = 0, return_lse: bool = False):
        import torch

        from . import _lib, backend

        B, Sq, HQ, D = q.shape
        if any(t.device != self.device for t in (q, k_cache, v_cache, local_seqlens, local_block_table)):
            raise ValueError(f"every tensor must be on {self.device}, the device this exchange was built on")
        if (B, HQ, k_cache.shape[2], D) != self.geometry or Sq != 1:
            raise ValueError(f"call geometry {(B, HQ, k_cache.shape[2], D)} (Sq={Sq}) does not match "
                             f"{self.geometry} with one query token")
        scale = softmax_scale if softmax_scale is not None else D ** -0.5
        q = q.contiguous()
        seq = local_seqlens.to(torch.int32).contiguous()
        bt = local_block_table.to(torch.int32).contiguous()
        PS, HKV = k_cache.shape[1], k_cache.shape[2]
        btw = bt.shape[1]
        if num_splits <= 0 or chunk_len <= 0:
            num_splits, chunk_len = backend.kvcache_plan(B, 1, HQ, HKV, D, btw * PS)
        lib = self._lib
        ws_bytes = int(lib.mxfa_split_workspace_bytes(B * HQ, D, num_splits))
        out = torch.empty_like(q)
        lse = torch.empty((B, HQ), device=q.device, dtype=torch.float32) if return_lse else None
        with torch.cuda.device(q.device):
            stream = torch.cuda.current_stream(q.device).cuda_stream
            ws = torch.empty((max(ws_bytes, 16) // 4,), device=q.device, dtype=torch.float32)
            counters = backend.split_counters(q.device, stream, int(lib.mxfa_split_counter_bytes(B, 1, HQ, HKV)))
            bf16 = int(q.dtype == torch.bfloat16)
            if self.one_launch:
                rc = lib.mxfa_cp_attention_launch(
                    q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), bt.data_ptr(), seq.data_ptr(),
                    out.data_ptr(), _lib.ptr(lse), ws.data_ptr(), ws_bytes, counters.data_ptr(),
                    self.peer_table.data_ptr(), self._local, self.rank, self.world, B, HQ, HKV, D, PS, btw,
                    k_cache.shape[0], num_splits, chunk_len, bf16, float(scale), stream)
                _lib.check(rc, "mxfa_cp_attention_launch")
                self.launches_per_call = 1 if lib.mxfa_cp_last_merged_in_place() else 2
            else:
                rc = lib.mxfa_cp_decode_launch(
                    q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), bt.data_ptr(), seq.data_ptr(),
                    out.data_ptr(), None, ws.data_ptr(), ws_bytes, counters.data_ptr(), self.peer_table.data_ptr(),
                    self.rank, self.world, B, HQ, HKV, D, PS, btw, k_cache.shape[0], num_splits, chunk_len, bf16,
                    float(scale), stream)
                _lib.check(rc, "mxfa_cp_decode_launch")
                rc = lib.mxfa_cp_merge_launch(self._local, out.data_ptr(), _lib.ptr(lse), self.world, B, HQ, HKV,
                                              D, bf16, stream)
                _lib.check(rc, "mxfa_cp_merge_launch")
                self.launches_per_call = 2
        return (out, lse) if return_lse else out

    def close(self) -> None:
        """Collective: every rank stops using the buffers, then mappings and memory are released."""
        import torch
        import torch.distributed as dist

        from . import _lib

        if self._local is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for p in self._imported:
                _lib.check(self._lib.mxfa_peer_close(p), "mxfa_peer_close")
            self._imported = []
            dist.barrier(group=self.group)  # no rank still maps this rank's buffer
            _lib.check(self._lib.mxfa_peer_free(self._local), "mxfa_peer_free")
        self._local = None
