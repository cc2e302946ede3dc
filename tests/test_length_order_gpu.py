"""Once-per-step length order: the order kernel and launches that take it.

The order only schedules the work (grid row y runs sequence order[y],
longest first), so a launch given it must produce the same bits as the one
that ranks the lengths in every CTA -- for every split plan, both 16-bit
dtypes, e4m3 caches, a stale order, and through the public API.
"""

from __future__ import annotations

import numpy as np
import pytest

from helpers import assert_close_out, host, oracle_paged
from mxflashattn_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


def _expected_order(lengths):
    """Longest first, ties by index (the kernel's packed key)."""
    return sorted(range(len(lengths)), key=lambda i: (-lengths[i], i))


@pytest.mark.parametrize("B", [2, 7, 128, 512])
def test_order_kernel_is_longest_first_with_ties_by_index(B, cuda_device):
    import torch

    from mxflashattn_b200 import kvcache_length_order

    rng = np.random.default_rng(B)
    lengths = rng.integers(0, 40, size=B).tolist()  # many ties
    order = kvcache_length_order(torch.tensor(lengths, dtype=torch.int32, device=cuda_device))
    assert order.dtype == torch.int32 and order.shape == (B,)
    assert host(order).tolist() == _expected_order(lengths)


def test_order_kernel_skips_batches_that_need_no_order(cuda_device):
    import torch

    from mxflashattn_b200 import kvcache_length_order

    assert kvcache_length_order(torch.tensor([5], dtype=torch.int32, device=cuda_device)) is None
    assert kvcache_length_order(torch.ones(513, dtype=torch.int64, device=cuda_device)) is None


def _device_case(case, device):
    import torch

    tdt = syn.torch_dtype(case.dtype)
    return (torch.from_numpy(case.q).to(device, tdt), torch.from_numpy(case.k_cache).to(device, tdt),
            torch.from_numpy(case.v_cache).to(device, tdt), torch.from_numpy(case.cache_seqlens.copy()).to(device),
            torch.from_numpy(case.block_table).to(device))


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("splits", [0, 1, 3])
def test_ordered_launch_is_bit_identical_to_ranking(dtype, splits, cuda_device):
    import torch

    from mxflashattn_b200 import _lib, backend

    lengths = syn.qwen3_4b_lengths(11, 48)
    case = syn.paged_case(900 + splits, batch=48, q_heads=32, kv_heads=8, head_dim=128, dtype=dtype, page_size=16,
                          lengths=lengths)
    q, kc, vc, sl, bt = _device_case(case, cuda_device)
    cap = 16 * bt.shape[1]
    kw = {} if splits == 0 else {"num_splits": splits, "chunk_len": -(-cap // splits)}
    _lib.read_error_flags()
    ref, ref_lse = backend.kvcache_attention(q, kc, vc, sl, bt, case.softmax_scale, False, return_lse=True, **kw)
    order = backend.kvcache_length_order(sl)
    out, lse = backend.kvcache_attention(q, kc, vc, sl, bt, case.softmax_scale, False, return_lse=True,
                                         length_order=order, **kw)
    # an order computed for other lengths of the same batch only schedules differently
    stale = backend.kvcache_length_order(torch.flip(sl, [0]).contiguous())
    out2 = backend.kvcache_attention(q, kc, vc, sl, bt, case.softmax_scale, False, length_order=stale, **kw)
    torch.cuda.synchronize()
    assert torch.equal(out, ref) and torch.equal(lse, ref_lse) and torch.equal(out2, ref)
    assert _lib.read_error_flags() == 0
    assert_close_out(host(out), oracle_paged(case)[0], dtype, "ordered launch vs oracle")


def test_ordered_launch_with_e4m3_caches(cuda_device):
    import torch

    from mxflashattn_b200 import _lib, backend

    lengths = syn.qwen3_4b_lengths(12, 32)
    case = syn.paged_case(950, batch=32, q_heads=32, kv_heads=8, head_dim=128, dtype="bf16", page_size=16,
                          lengths=lengths)
    q, kc, vc, sl, bt = _device_case(case, cuda_device)
    k8, v8 = kc.to(torch.float8_e4m3fn), vc.to(torch.float8_e4m3fn)
    _lib.read_error_flags()
    for splits in (0, 3):
        kw = {} if splits == 0 else {"num_splits": splits, "chunk_len": -(-16 * bt.shape[1] // splits)}
        ref = backend.kvcache_attention(q, k8, v8, sl, bt, case.softmax_scale, False, k_scale=0.5, v_scale=2.0, **kw)
        out = backend.kvcache_attention(q, k8, v8, sl, bt, case.softmax_scale, False, k_scale=0.5, v_scale=2.0,
                                        length_order=backend.kvcache_length_order(sl), **kw)
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
    assert _lib.read_error_flags() == 0


def test_order_entries_outside_the_batch_are_flagged_and_run_their_own_row(cuda_device):
    import torch

    from mxflashattn_b200 import _lib, backend

    case = syn.paged_case(960, batch=6, q_heads=8, kv_heads=2, head_dim=128, dtype="bf16", page_size=16,
                          lengths=[5, 300, 17, 64, 1, 128])
    q, kc, vc, sl, bt = _device_case(case, cuda_device)
    bad = torch.full((6,), 99, dtype=torch.int32, device=cuda_device)
    _lib.read_error_flags()
    out = backend.kvcache_attention(q, kc, vc, sl, bt, case.softmax_scale, False, length_order=bad)
    torch.cuda.synchronize()
    assert _lib.read_error_flags() & _lib.FLAG_BAD_ORDER
    assert_close_out(host(out), oracle_paged(case)[0], "bf16", "out-of-range order entries")


def test_public_api_takes_the_order(cuda_device):
    import torch

    from mxflashattn_b200 import flash_attn_with_kvcache, kvcache_length_order

    lengths = syn.qwen3_4b_lengths(13, 24)
    case = syn.paged_case(970, batch=24, q_heads=32, kv_heads=8, head_dim=128, dtype="bf16", page_size=16,
                          lengths=lengths)
    q, kc, vc, sl, bt = _device_case(case, cuda_device)
    ref = flash_attn_with_kvcache(q, kc, vc, cache_seqlens=sl, block_table=bt, softmax_scale=case.softmax_scale)
    out = flash_attn_with_kvcache(q, kc, vc, cache_seqlens=sl, block_table=bt, softmax_scale=case.softmax_scale,
                                  length_order=kvcache_length_order(sl))
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
