"""Context-split decode kernels on the GPU.

Ranks are emulated on one device: each rank's packed (O, LSE) record comes
from ``mxfa_kvcache_attention_packed_launch`` over its own page range, the
records are stacked as an all-gather would leave them, and
``mxfa_lse_merge_launch`` merges them.  The result must match attention over
the whole context (oracle).  When two GPUs are visible, the same path also
runs with real NCCL ranks.
"""

from __future__ import annotations

import datetime
import socket

import numpy as np
import pytest

from helpers import assert_close_lse, assert_close_out, host, oracle_paged, out_tolerance
from mxflashattn_b200 import context_split as cs
from mxflashattn_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


def _case():
    return syn.paged_case(123, batch=4, q_heads=32, kv_heads=8, head_dim=128, dtype="bf16", page_size=16,
                          lengths=[16384, 3000, 17, 1], outlier_frac=0.01)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_emulated_ranks_merge_to_full_attention(world, cuda_device):
    import torch

    from mxflashattn_b200 import backend

    case = _case()
    tdt = syn.torch_dtype(case.dtype)
    q = torch.from_numpy(case.q).to(cuda_device, tdt)
    kc = torch.from_numpy(case.k_cache).to(cuda_device, tdt)
    vc = torch.from_numpy(case.v_cache).to(cuda_device, tdt)
    records = []
    for rank in range(world):
        ll, table = cs.local_view(case.cache_seqlens, case.block_table, world, rank, 16)
        records.append(backend.kvcache_attention_packed(q, kc, vc, torch.from_numpy(ll).to(cuda_device),
                                                        torch.from_numpy(table).to(cuda_device),
                                                        case.softmax_scale))
    gathered = torch.stack(records)
    out, lse = backend.lse_merge(gathered, 4 * 32, 128, tdt, lse=True)
    ref, ref_lse = oracle_paged(case)[:2]
    assert_close_out(host(out).reshape(ref.shape), ref, "bf16", f"context split world={world}")
    assert_close_lse(host(lse).reshape(4, 1, 32), ref_lse, f"context split world={world}")


def _nccl_worker(rank, world, port, result):
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        case = _case()
        tdt = syn.torch_dtype(case.dtype)
        dev = torch.device("cuda", rank)
        ll, table = cs.local_view(case.cache_seqlens, case.block_table, world, rank, 16)
        out = cs.context_parallel_decode(torch.from_numpy(case.q).to(dev, tdt),
                                         torch.from_numpy(case.k_cache).to(dev, tdt),
                                         torch.from_numpy(case.v_cache).to(dev, tdt),
                                         torch.from_numpy(ll).to(dev), torch.from_numpy(table).to(dev),
                                         case.softmax_scale)
        torch.cuda.synchronize()
        ref = oracle_paged(case)[0]
        excess = np.abs(host(out) - ref) - out_tolerance(ref, "bf16")
        result[rank] = float(np.max(excess))  # <= 0 when every element is within tolerance
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _fused_worker(rank, world, port, result, modes=(True,)):
    """Fused exchange vs the NCCL path and the oracle, over three calls (both buffer halves).

    ``modes`` cycles the exchange form per call: True merges inside the decode
    kernel (one launch), False in the separate merge kernel."""
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    fused = None
    try:
        from mxflashattn_b200 import _lib

        case = _case()
        tdt = syn.torch_dtype(case.dtype)
        dev = torch.device("cuda", rank)
        ll, table = cs.local_view(case.cache_seqlens, case.block_table, world, rank, 16)
        kc = torch.from_numpy(case.k_cache).to(dev, tdt)
        vc = torch.from_numpy(case.v_cache).to(dev, tdt)
        sl = torch.from_numpy(ll).to(dev)
        bt = torch.from_numpy(table).to(dev)
        fused = cs.FusedContextParallelDecode(4, 32, 8, 128, device=dev)
        worst = -1.0
        for step in range(4):
            fused.one_launch = modes[step % len(modes)]
            q_np = case.q if step == 0 else syn.round_dtype(np.random.default_rng(50 + step).standard_normal(
                case.q.shape).astype(np.float32), "bf16")
            q = torch.from_numpy(q_np).to(dev, tdt)
            out, lse = fused(q, kc, vc, sl, bt, case.softmax_scale, return_lse=True)
            nccl = cs.context_parallel_decode(q, kc, vc, sl, bt, case.softmax_scale)
            torch.cuda.synchronize()
            import dataclasses

            ref, ref_lse = oracle_paged(dataclasses.replace(case, q=q_np))[:2]
            worst = max(worst, float(np.max(np.abs(host(out) - ref) - out_tolerance(ref, "bf16"))))
            worst = max(worst, float(np.max(np.abs(host(out) - host(nccl)) - out_tolerance(ref, "bf16"))))
            lse_err = float(np.max(np.abs(host(lse).reshape(4, 1, 32) - ref_lse)))
            worst = max(worst, lse_err - 1e-3)
        result[rank] = worst  # <= 0 when every element is within tolerance
        result[f"flags{rank}"] = int(_lib.read_error_flags())
    finally:
        if fused is not None:
            fused.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("modes", [(True,), (False,), (True, False)], ids=["one_launch", "two_launches", "mixed"])
def test_two_gpu_fused_peer_exchange(cuda_device, modes):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two visible GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    manager = mp.Manager()
    result = manager.dict()
    mp.spawn(_fused_worker, args=(2, port, result, modes), nprocs=2, join=True)
    assert all(result[r] <= 0.0 for r in range(2)), dict(result)
    assert all(result[f"flags{r}"] == 0 for r in range(2)), dict(result)


@pytest.mark.parametrize("modes", [(True,), (False,), (True, False)], ids=["one_launch", "two_launches", "mixed"])
def test_single_rank_fused_exchange_matches_local_decode(cuda_device, modes):
    """world = 1: the exchange degenerates to the local record (no peer, no waiting on another device).

    Both exchange forms, and the two alternating on one buffer (their epoch
    and counters must hand over cleanly), against the oracle, LSE included."""
    import datetime as _dt
    import os

    import torch
    import torch.distributed as dist

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1,
                            timeout=_dt.timedelta(seconds=60))
    try:
        case = _case()
        tdt = syn.torch_dtype(case.dtype)
        q = torch.from_numpy(case.q).to(cuda_device, tdt)
        kc = torch.from_numpy(case.k_cache).to(cuda_device, tdt)
        vc = torch.from_numpy(case.v_cache).to(cuda_device, tdt)
        sl = torch.from_numpy(case.cache_seqlens.copy()).to(cuda_device)
        bt = torch.from_numpy(case.block_table).to(cuda_device)
        fused = cs.FusedContextParallelDecode(4, 32, 8, 128, device=cuda_device)
        try:
            from mxflashattn_b200 import _lib

            _lib.read_error_flags()  # clear what earlier tests left
            ref, ref_lse = oracle_paged(case)[:2]
            for step in range(5):
                fused.one_launch = modes[step % len(modes)]
                out, lse = fused(q, kc, vc, sl, bt, case.softmax_scale, return_lse=True)
                torch.cuda.synchronize()
                assert_close_out(host(out), ref, "bf16", f"single-rank fused exchange, call {step}")
                assert_close_lse(host(lse).reshape(ref_lse.shape), ref_lse, f"single-rank LSE, call {step}")
                # 32 units fit on the GPU at once: the one-call form merges inside the decode kernel
                assert fused.launches_per_call == (1 if fused.one_launch else 2)
            assert _lib.read_error_flags() == 0
        finally:
            fused.close()
    finally:
        dist.destroy_process_group()


def test_single_rank_exchange_with_more_units_than_resident_ctas(cuda_device):
    """1024 units (128 sequences x 8 KV heads) exceed what one GPU holds at once, so the one-call
    entry leaves the merge to its own kernel; the result still matches the oracle."""
    import datetime as _dt

    import torch
    import torch.distributed as dist

    from mxflashattn_b200 import _lib

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1,
                            timeout=_dt.timedelta(seconds=60))
    try:
        lengths = np.random.default_rng(7).integers(1, 300, size=128).tolist()
        case = syn.paged_case(321, batch=128, q_heads=32, kv_heads=8, head_dim=128, dtype="bf16", page_size=16,
                              lengths=lengths)
        tdt = syn.torch_dtype(case.dtype)
        args = [torch.from_numpy(a).to(cuda_device, tdt) for a in (case.q, case.k_cache, case.v_cache)]
        sl = torch.from_numpy(case.cache_seqlens.copy()).to(cuda_device)
        bt = torch.from_numpy(case.block_table).to(cuda_device)
        fused = cs.FusedContextParallelDecode(128, 32, 8, 128, device=cuda_device)
        try:
            _lib.read_error_flags()
            ref, ref_lse = oracle_paged(case)[:2]
            for step in range(3):
                out, lse = fused(*args, sl, bt, case.softmax_scale, return_lse=True)
                torch.cuda.synchronize()
                assert_close_out(host(out), ref, "bf16", f"128-sequence exchange, call {step}")
                assert_close_lse(host(lse).reshape(ref_lse.shape), ref_lse, f"128-sequence LSE, call {step}")
                assert fused.launches_per_call == 2  # the merge kernel ran
            assert _lib.read_error_flags() == 0
        finally:
            fused.close()
    finally:
        dist.destroy_process_group()


def test_two_gpu_nccl_context_split(cuda_device):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two visible GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    manager = mp.Manager()
    result = manager.dict()
    mp.spawn(_nccl_worker, args=(2, port, result), nprocs=2, join=True)
    assert all(result[r] <= 0.0 for r in range(2)), dict(result)


def test_exchange_wait_times_out_and_reports(cuda_device):
    """A merge whose peer never publishes gives up after its bounded wait and raises the timeout flag.

    The exchange buffer is sized for two ranks but only this process exists, so
    no record ever carries the step's tag: every warp waits ~1 s, then the
    kernel finishes, the context stays usable and the host reads the flag.
    """
    import ctypes
    import time

    import torch

    from mxflashattn_b200 import _lib

    lib = _lib.load()
    B, HQ, HKV, D = 1, 8, 2, 128
    nbytes = int(lib.mxfa_cp_buffer_bytes(2, B, HQ, HKV, D))
    buf = ctypes.c_void_p()
    _lib.check(lib.mxfa_peer_alloc(nbytes, ctypes.byref(buf)), "mxfa_peer_alloc")
    try:
        out = torch.empty((B * HQ, D), device=cuda_device, dtype=torch.bfloat16)
        _lib.read_error_flags()
        t0 = time.time()
        _lib.check(lib.mxfa_cp_merge_launch(buf, out.data_ptr(), None, 2, B, HQ, HKV, D, 1,
                                            torch.cuda.current_stream().cuda_stream), "mxfa_cp_merge_launch")
        torch.cuda.synchronize()
        waited = time.time() - t0
        assert _lib.read_error_flags() & 4  # MXFA_FLAG_WAIT_TIMEOUT
        assert 0.5 < waited < 30.0
        # the device still works
        x = torch.ones(4, device=cuda_device)
        assert float((x * 2).sum()) == 8.0
    finally:
        _lib.check(lib.mxfa_peer_free(buf), "mxfa_peer_free")


@pytest.mark.parametrize("world", [2, 4, 8])
def test_prefill_kv_head_shards_reassemble_the_full_result(world, cuda_device):
    """Emulated ranks on one device: each rank's KV-head share, concatenated over heads, equals the whole call."""
    import torch

    from mxflashattn_b200 import backend

    lens = [700, 129, 1]
    case = syn.varlen_case(310 + world, q_lens=lens, q_heads=32, kv_heads=8, head_dim=128, dtype="bf16",
                           causal=True)
    tdt = syn.torch_dtype(case.dtype)
    q, k, v = (torch.from_numpy(x).to(cuda_device, tdt) for x in (case.q, case.k, case.v))
    cu = torch.from_numpy(case.cu_q).to(cuda_device)
    full, full_lse = backend.flash_attn_varlen_func(q, k, v, cu, cu, max(lens), max(lens), True,
                                                    case.softmax_scale, return_lse=True)
    parts = [cs.prefill_local_heads(q, k, v, cu, cu, max(lens), max(lens), world_size=world, rank=r, causal=True,
                                    softmax_scale=case.softmax_scale, return_lse=True) for r in range(world)]
    torch.cuda.synchronize()
    assert torch.equal(torch.cat([o for o, _ in parts], dim=1), full)
    assert torch.equal(torch.cat([lse for _, lse in parts], dim=1), full_lse)
