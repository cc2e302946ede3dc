"""GPU parity of the fused append + attention launch.

``mxfa_kvcache_append_attention_launch`` writes the appended K/V rows from
inside the attention kernel (each CTA writes the rows of its own KV head and
position chunk, then reads them back through TMA or cp.async).  It must give
the same cache bytes as the separate ``mxfa_kv_append_launch`` and the same
output bits as the attention that follows it, for every page size, split
plan and dense cache, and report appends past the cache's capacity the way
the separate append does.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from helpers import assert_close_out, host, oracle_paged, to_device
from mxflashattn_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


def _two_launch(t, case, splits, chunk):
    from mxflashattn_b200 import backend

    backend.kv_append(t["k_cache"], t["v_cache"], t["k"], t["v"], t["cache_seqlens"], t["block_table"])
    return backend.kvcache_attention(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"], t["block_table"],
                                     case.softmax_scale, case.causal, append_len=t["k"].shape[1],
                                     return_lse=True, num_splits=splits, chunk_len=chunk)


def _fused(t, case, splits, chunk):
    from mxflashattn_b200 import backend

    return backend.kvcache_attention(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"], t["block_table"],
                                     case.softmax_scale, case.causal, append_len=t["k"].shape[1],
                                     return_lse=True, num_splits=splits, chunk_len=chunk, k_new=t["k"],
                                     v_new=t["v"])


@pytest.mark.parametrize("page_size", [1, 5, 16, 32, 48])
@pytest.mark.parametrize("q_len", [1, 2, 4])
@pytest.mark.parametrize("splits", [0, 1, 3, 7])
def test_fused_append_matches_two_launches_bitwise(page_size, q_len, splits, cuda_device):
    import torch

    from mxflashattn_b200 import _lib

    case = syn.paged_case(900 + page_size * 11 + q_len * 3 + splits, batch=4, q_heads=8, kv_heads=2,
                          head_dim=128, dtype="bf16", page_size=page_size, lengths=[0, 47, 130, 15],
                          q_len=q_len, append=q_len, causal=True, extra_table_cols=1)
    cap = page_size * case.block_table.shape[1]
    chunk = -(-cap // splits) if splits > 1 else 0
    t_sep = to_device(case, cuda_device)
    t_fus = to_device(case, cuda_device)
    out_s, lse_s = _two_launch(t_sep, case, splits, chunk)
    out_f, lse_f = _fused(t_fus, case, splits, chunk)
    torch.cuda.synchronize()
    assert _lib.read_error_flags() == 0
    np.testing.assert_array_equal(host(t_fus["k_cache"]), host(t_sep["k_cache"]))
    np.testing.assert_array_equal(host(t_fus["v_cache"]), host(t_sep["v_cache"]))
    assert torch.equal(out_f, out_s)
    assert torch.equal(lse_f, lse_s)
    ref, _, kc, vc, _ = oracle_paged(case)
    np.testing.assert_array_equal(host(t_fus["k_cache"]), kc)
    np.testing.assert_array_equal(host(t_fus["v_cache"]), vc)
    assert_close_out(host(out_f), ref, "bf16", f"fused ps{page_size} Sq{q_len} splits{splits}")


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
def test_fused_append_dense_cache(dt, cuda_device):
    import torch

    case = syn.paged_case(61, batch=3, q_heads=16, kv_heads=4, head_dim=64, dtype=dt, page_size=1,
                          lengths=[0, 33, 90], append=2, q_len=2, causal=True, dense=True, extra_table_cols=8)
    t_sep = to_device(case, cuda_device)
    t_fus = to_device(case, cuda_device)
    out_s, _ = _two_launch(t_sep, case, 0, 0)
    out_f, _ = _fused(t_fus, case, 0, 0)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(host(t_fus["k_cache"]), host(t_sep["k_cache"]))
    np.testing.assert_array_equal(host(t_fus["v_cache"]), host(t_sep["v_cache"]))
    assert torch.equal(out_f, out_s)


@pytest.mark.parametrize("splits", [0, 4])
def test_fused_append_past_capacity_is_flagged_and_skipped(splits, cuda_device):
    """A sequence already at capacity: the append is reported, nothing is written past the table."""
    import torch

    from mxflashattn_b200 import _lib

    page_size = 16
    case = syn.paged_case(73, batch=2, q_heads=8, kv_heads=2, head_dim=128, dtype="bf16", page_size=page_size,
                          lengths=[64, 10], append=1)
    t = to_device(case, cuda_device)
    t["block_table"] = t["block_table"][:, :4].contiguous()  # 64 slots: row 0 is full
    cap = page_size * 4
    chunk = -(-cap // splits) if splits > 1 else 0
    k_before = host(t["k_cache"]).copy()
    _lib.read_error_flags()
    _fused(t, case, splits, chunk)
    torch.cuda.synchronize()
    assert _lib.read_error_flags() & 2  # MXFA_FLAG_TABLE_TOO_NARROW
    k_after = host(t["k_cache"])
    # row 1's append landed at position 10 of its first page; nothing else changed
    phys = int(case.block_table[1, 0])
    np.testing.assert_array_equal(k_after[phys, 10], host(t["k"])[1, 0])
    k_after[phys, 10] = k_before[phys, 10]
    np.testing.assert_array_equal(k_after, k_before)


def test_fused_append_rejects_more_than_16_rows(cuda_device):
    import torch

    from mxflashattn_b200 import _lib

    lib = _lib.load()
    B, Sq, HQ, HKV, D, PS = 1, 3, 8, 1, 64, 16
    q = torch.zeros((B, Sq, HQ, D), device=cuda_device, dtype=torch.bfloat16)
    kc = torch.zeros((2, PS, HKV, D), device=cuda_device, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    bt = torch.zeros((B, 2), device=cuda_device, dtype=torch.int32)
    sl = torch.zeros((B,), device=cuda_device, dtype=torch.int32)
    kn = torch.zeros((B, Sq, HKV, D), device=cuda_device, dtype=torch.bfloat16)
    out = torch.empty_like(q)
    rc = lib.mxfa_kvcache_append_attention_launch(
        q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), sl.data_ptr(), out.data_ptr(), None, None, 0,
        None, kn.data_ptr(), kn.data_ptr(), B, Sq, HQ, HKV, D, PS, 2, 2, Sq, 1, 32, 1, 1, ctypes.c_float(0.125), None)
    assert rc == -1  # MXFA_ERR_UNSUPPORTED
    assert "16 query rows" in _lib.last_error()
