"""Context-split decode host logic on CPU ranks (gloo, world size 2 and 3).

Each rank takes its page-aligned slice of every sequence (``local_view``),
computes its (O, LSE) record with the oracle, the ranks exchange records
with the product's ``gather_partials`` (a real all-gather over gloo) and the
LSE merge of the gathered records must equal attention over the whole
context.  No GPU is used: the CUDA halves are covered by the -m gpu tests.
"""

from __future__ import annotations

import ctypes
import datetime
import math
import socket

import numpy as np
import pytest

import oracle
from mxflashattn_b200 import context_split as cs
from mxflashattn_b200 import synthetic as syn


def test_shard_ranges_cover_every_position_once():
    lengths = [1, 15, 16, 17, 100, 1000, 0, 33]
    for world in (1, 2, 3, 4, 8):
        r = cs.shard_ranges(lengths, world, 16)
        for b, length in enumerate(lengths):
            covered = np.zeros(length, dtype=int)
            for k in range(world):
                s, e = r[k, b]
                assert s % 16 == 0 and 0 <= s <= e <= length
                covered[s:e] += 1
            assert (covered == 1).all()


def test_batch_and_head_shards_partition():
    for world in (1, 2, 3, 8):
        seen = [i for k in range(world) for i in cs.shard_batch(128, world, k)]
        assert seen == list(range(128))
    assert [list(cs.shard_kv_heads(8, 4, k)) for k in range(4)] == [[0, 1], [2, 3], [4, 5], [6, 7]]
    with pytest.raises(ValueError):
        cs.shard_kv_heads(8, 3, 0)


def _rank_record(case, world, rank):
    """Oracle (O, LSE) packed record of one rank's positions: [B*HQ, D+1] float32."""
    B, _, HQ, D = case.q.shape
    lengths = case.cache_seqlens
    local_len, table = cs.local_view(lengths, case.block_table, world, rank, case.k_cache.shape[1])
    rec = np.zeros((B * HQ, D + 1), np.float32)
    for b in range(B):
        if local_len[b] == 0:
            rec[b * HQ:(b + 1) * HQ, D] = -np.inf
            continue
        k = oracle.gather_paged_kv(case.k_cache, table[b], int(local_len[b]))
        v = oracle.gather_paged_kv(case.v_cache, table[b], int(local_len[b]))
        out, lse = oracle.attention_single(case.q[b], k, v, softmax_scale=case.softmax_scale, return_lse=True)
        rec[b * HQ:(b + 1) * HQ, :D] = out[0]
        rec[b * HQ:(b + 1) * HQ, D] = lse[:, 0]
    return rec


def _merge(gathered):
    """Host LSE merge of [N, rows, D+1] records (the algebra mxfa_lse_merge_launch runs)."""
    o, lse = gathered[..., :-1].astype(np.float64), gathered[..., -1].astype(np.float64)
    m = np.max(np.where(np.isfinite(lse), lse, -np.inf), axis=0)
    w = np.where(np.isfinite(lse), np.exp(lse - m[None]), 0.0)
    return (w[..., None] * o).sum(0) / w.sum(0)[:, None], m + np.log(w.sum(0))


def _worker(rank, world, port, result):
    import torch
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        case = syn.paged_case(77, batch=3, q_heads=8, kv_heads=2, head_dim=64, dtype="bf16", page_size=16,
                              lengths=[1000, 17, 40])
        rec = torch.from_numpy(_rank_record(case, world, rank))
        gathered = cs.gather_partials(rec).numpy()
        out, lse = _merge(gathered)
        full, full_lse = oracle.attention_kvcache(case.q, case.k_cache.copy(), case.v_cache.copy(),
                                                  cache_seqlens=case.cache_seqlens.copy(),
                                                  block_table=case.block_table,
                                                  softmax_scale=case.softmax_scale, return_lse=True)
        err = float(np.max(np.abs(out - full.reshape(-1, 64))))
        lerr = float(np.max(np.abs(lse - full_lse.reshape(-1))))
        result[rank] = (err, lerr, gathered.shape)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 3])
def test_context_split_exchange_and_merge_over_gloo(world):
    import torch.multiprocessing as mp

    manager = mp.Manager()
    result = manager.dict()
    mp.spawn(_worker, args=(world, _free_port(), result), nprocs=world, join=True)
    assert sorted(result.keys()) == list(range(world))
    for rank in range(world):
        err, lerr, shape = result[rank]
        assert shape == (world, 3 * 8, 65)
        assert err < 1e-5 and lerr < 1e-5 and math.isfinite(err)


class _FakePeerLib:
    """The library's peer-memory entries for CPU ranks: addresses are integers, a handle carries the exporting
    rank's address, and `fail_at` = (rank, step) makes that rank's step return a CUDA error status."""

    def __init__(self, rank, fail_at):
        self.rank, self.fail_at = rank, fail_at
        self.log = []

    def _fails(self, step):
        return self.fail_at == (self.rank, step)

    def mxfa_last_error(self):
        return b"injected failure"

    def mxfa_peer_alloc(self, nbytes, out):
        if self._fails("alloc"):
            return 3
        out._obj.value = 0x100000 * (self.rank + 1)
        self.log.append(("alloc", out._obj.value))
        return 0

    def mxfa_peer_export(self, ptr, handle):
        if self._fails("export"):
            return 3
        ctypes.memmove(handle, int(ptr).to_bytes(8, "little") + bytes(56), 64)
        return 0

    def mxfa_peer_import(self, handle, out):
        if self._fails("import"):
            return 3
        out._obj.value = int.from_bytes(bytes(handle)[:8], "little") + 0x1000  # this rank's mapping of it
        self.log.append(("import", out._obj.value))
        return 0

    def mxfa_peer_close(self, ptr):
        self.log.append(("close", ptr))
        return 0

    def mxfa_peer_free(self, ptr):
        self.log.append(("free", ptr))
        return 0


def _mapping_worker(rank, world, port, fail_at, result):
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        lib = _FakePeerLib(rank, fail_at)
        try:
            local, imported, ptrs = cs.map_exchange_buffers(lib, 4096, world, rank)
            result[rank] = ("mapped", local, imported, ptrs, lib.log)
        except RuntimeError as exc:
            result[rank] = ("raised", str(exc), lib.log)
        dist.barrier()  # still in step with the other ranks after either outcome
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fail_at", [None, (1, "alloc"), (2, "export"), (0, "import")])
def test_exchange_buffer_mapping_agrees_across_ranks(fail_at):
    """Every rank maps every peer's buffer, or, when one rank's allocation, export or import fails, every rank
    raises naming that rank and releases all it mapped and allocated (no rank is left waiting)."""
    import torch.multiprocessing as mp

    world = 3
    result = mp.Manager().dict()
    mp.spawn(_mapping_worker, args=(world, _free_port(), fail_at, result), nprocs=world, join=True)
    assert sorted(result.keys()) == list(range(world))
    for rank in range(world):
        outcome = result[rank]
        if fail_at is None:
            _, local, imported, ptrs, _ = outcome
            assert outcome[0] == "mapped" and local == 0x100000 * (rank + 1) and ptrs[rank] == local
            assert ptrs == [0x100000 * (r + 1) + (0 if r == rank else 0x1000) for r in range(world)]
            assert imported == [p for r, p in enumerate(ptrs) if r != rank]
            continue
        status, message, log = outcome
        assert status == "raised" and f"rank(s) [{fail_at[0]}]" in message
        opened = [p for step, p in log if step == "import"]
        allocated = [p for step, p in log if step == "alloc"]
        assert sorted(p for step, p in log if step == "close") == sorted(opened)
        assert [p for step, p in log if step == "free"] == allocated
        assert len(allocated) == (0 if fail_at == (rank, "alloc") else 1)
