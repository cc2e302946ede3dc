"""GPU parity of the single-launch split decode (last-CTA merge).

``mxfa_kvcache_attention_counted_launch`` runs the split decode and the
combine in one kernel: the last split CTA of each (sequence, KV head, row
group) merges the partials.  It must give the same output and LSE bits as the
two-launch path (decode, then ``split_combine``), leave its counters at zero
after every launch, and replay correctly from a CUDA graph.
"""

from __future__ import annotations

import numpy as np
import pytest

from helpers import assert_close_lse, assert_close_out, host, oracle_paged, to_device
from mxflashattn_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


def _run(t, case, splits, chunk, single):
    from mxflashattn_b200 import backend

    return backend.kvcache_attention(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"], t["block_table"],
                                     case.softmax_scale, case.causal, return_lse=True, num_splits=splits,
                                     chunk_len=chunk, single_launch=single)


def _counters_zero(device):
    import torch

    from mxflashattn_b200 import backend

    torch.cuda.synchronize()
    for (dev, _), buf in backend._COUNTERS.items():
        if torch.device(dev) == torch.device(device):
            assert int(buf.abs().sum()) == 0


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("head_dim,gq,q_len", [(128, 4, 1), (128, 8, 1), (64, 2, 1), (128, 8, 2), (64, 8, 3)])
@pytest.mark.parametrize("splits", [2, 5, 16])
def test_single_launch_matches_two_launches_bitwise(dt, head_dim, gq, q_len, splits, cuda_device):
    import torch

    from mxflashattn_b200 import _lib

    case = syn.paged_case(1200 + head_dim + gq * 5 + q_len * 17 + splits, batch=5, q_heads=2 * gq, kv_heads=2,
                          head_dim=head_dim, dtype=dt, page_size=16, lengths=[3, 1, 300, 777, 64], q_len=q_len,
                          causal=q_len > 1, extra_table_cols=1)
    cap = 16 * case.block_table.shape[1]
    chunk = -(-cap // splits)
    t = to_device(case, cuda_device)
    out2, lse2 = _run(t, case, splits, chunk, single=False)
    for _ in range(2):  # the second launch checks the counters were left at zero
        out1, lse1 = _run(t, case, splits, chunk, single=True)
        torch.cuda.synchronize()
        assert torch.equal(out1, out2)
        assert torch.equal(lse1, lse2)
    assert _lib.read_error_flags() == 0
    _counters_zero(cuda_device)
    ref, ref_lse = oracle_paged(case)[:2]
    assert_close_out(host(out1), ref, dt, f"single-launch D{head_dim} gq{gq} Sq{q_len} np{splits}")
    assert_close_lse(host(lse1), ref_lse, f"single-launch lse np{splits}")


def test_single_launch_default_path_long_context(cuda_device):
    """Small batch, 16k context: the library plan splits; the default call is one launch."""
    import torch

    from mxflashattn_b200 import backend

    case = syn.paged_case(1300, batch=2, q_heads=32, kv_heads=8, head_dim=128, dtype="bf16", page_size=16,
                          lengths=[16384, 9000])
    t = to_device(case, cuda_device)
    cap = 16 * case.block_table.shape[1]
    splits, _ = backend.kvcache_plan(2, 1, 32, 8, 128, cap)
    assert splits > 1
    out = backend.kvcache_attention(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"], t["block_table"],
                                    case.softmax_scale, False)
    torch.cuda.synchronize()
    assert_close_out(host(out), oracle_paged(case)[0], "bf16", "16k single launch")
    _counters_zero(cuda_device)


def test_single_launch_replays_from_a_cuda_graph(cuda_device):
    import torch

    from mxflashattn_b200 import backend

    case = syn.paged_case(1301, batch=3, q_heads=16, kv_heads=4, head_dim=128, dtype="bf16", page_size=16,
                          lengths=[1000, 2, 513])
    t = to_device(case, cuda_device)
    cap = 16 * case.block_table.shape[1]
    out = torch.empty_like(t["q"])
    s = torch.cuda.Stream(cuda_device)
    s.wait_stream(torch.cuda.current_stream(cuda_device))
    with torch.cuda.stream(s):
        backend.kvcache_attention(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"], t["block_table"],
                                  case.softmax_scale, False, num_splits=4, chunk_len=-(-cap // 4), out=out)
    torch.cuda.current_stream(cuda_device).wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        backend.kvcache_attention(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"], t["block_table"],
                                  case.softmax_scale, False, num_splits=4, chunk_len=-(-cap // 4), out=out)
    ref = oracle_paged(case)[0]
    for step in range(3):
        out.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        assert_close_out(host(out), ref, "bf16", f"graph replay {step}")
    del g
    _counters_zero(cuda_device)


def test_counter_bytes_geometry():
    from mxflashattn_b200 import _lib

    lib = _lib.load()
    assert lib.mxfa_split_counter_bytes(128, 1, 32, 8) == 128 * 8 * 4       # 4 rows per KV head: one group
    assert lib.mxfa_split_counter_bytes(4, 3, 32, 4) == 4 * 4 * 2 * 4       # 24 rows: two groups of 16
    assert lib.mxfa_split_counter_bytes(0, 1, 32, 8) == 0
    assert np.int64(lib.mxfa_split_counter_bytes(2, 1, 30, 8)) == 0          # HQ not a multiple of HKV


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("splits", [63, 64, 65, 96])
def test_merge_forms_around_64_splits(dt, splits, cuda_device):
    """Up to 64 splits the merge loads every (m, d) pair in one round; past 64 it takes the loop form.

    Both sides of the boundary must give the same bits in one launch (merge
    inside the decode kernel) and in two (separate combine kernel), and match
    the oracle.
    """
    import torch

    from mxflashattn_b200 import _lib

    case = syn.paged_case(1400 + splits + (dt == "bf16"), batch=3, q_heads=16, kv_heads=4, head_dim=128, dtype=dt,
                          page_size=16, lengths=[3000, 1, 1500])
    cap = 16 * case.block_table.shape[1]
    chunk = -(-cap // splits)
    t = to_device(case, cuda_device)
    out2, lse2 = _run(t, case, splits, chunk, single=False)
    out1, lse1 = _run(t, case, splits, chunk, single=True)
    torch.cuda.synchronize()
    assert torch.equal(out1, out2)
    assert torch.equal(lse1, lse2)
    assert _lib.read_error_flags() == 0
    _counters_zero(cuda_device)
    ref, ref_lse = oracle_paged(case)[:2]
    assert_close_out(host(out1), ref, dt, f"{splits} splits")
    assert_close_lse(host(lse1), ref_lse, f"{splits} splits lse")
