"""GPU parity of decode at the coverage matrix's largest cells.

The coverage matrix of the benchmark configs runs batches up to 256 with
contexts up to 8192 (Hk=4, GQ in {2,4,8}, D in {64,128}, fp16/bf16, KV with
1% x50 outliers); its largest cell, B=256 at 8192 tokens, holds 4.29 GB of
K/V.  Inputs are generated on the device; the whole batch must be finite,
and sampled sequences (always including the longest and the shortest) are
compared with the oracle, output and LSE, through the public API and through
the backend with an explicit split plan.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from helpers import assert_close_lse, assert_close_out, host
from mxflashattn_b200 import synthetic as syn

pytestmark = pytest.mark.gpu

PAGE = 16


def _outliers(t, seed):
    """Scale 1% of the cache entries by 50, on the device."""
    import torch

    gen = torch.Generator(device=t["k_cache"].device)
    gen.manual_seed(seed)
    for name in ("k_cache", "v_cache"):
        x = t[name]
        mask = torch.rand(x.shape, generator=gen, device=x.device) < 0.01
        x[mask] = x[mask] * 50


def _sampled_check(t, out, lse, lengths, picks, dt, what):
    import torch

    bt = t["block_table"]
    hkv, d = t["k_cache"].shape[2], t["k_cache"].shape[3]
    for b in picks:
        L = int(lengths[b])
        n = -(-L // PAGE)
        rows = bt[b, :n].long()
        kc = host(t["k_cache"][rows]).reshape(n * PAGE, hkv, d)[:L]
        vc = host(t["v_cache"][rows]).reshape(n * PAGE, hkv, d)[:L]
        ref, ref_lse = oracle.attention_single(host(t["q"][b]), kc, vc, return_lse=True)
        assert_close_out(host(out[b]), ref, dt, f"{what} sequence {b} (len {L})")
        if lse is not None:
            assert_close_lse(host(lse[b]).reshape(np.shape(ref_lse)), ref_lse, f"{what} lse {b}")
    torch.cuda.synchronize()


@pytest.mark.parametrize("batch,gq,d,dt", [(64, 8, 128, "bf16"), (64, 2, 64, "fp16"), (256, 4, 128, "fp16"),
                                           (256, 8, 64, "bf16")])
def test_large_batch_mixed_lengths(batch, gq, d, dt, cuda_device):
    import torch

    from mxflashattn_b200 import _lib, flash_attn_with_kvcache

    base = [1, 17, 1000, 4096, 8192]
    lengths = [base[i % len(base)] for i in range(batch)]
    t = syn.device_paged_decode(seed=batch + gq + d, lengths=lengths, q_heads=4 * gq, kv_heads=4, head_dim=d,
                                dtype=dt, page_size=PAGE, device=cuda_device)
    _outliers(t, batch * 7 + d)
    out = flash_attn_with_kvcache(t["q"], t["k_cache"], t["v_cache"], cache_seqlens=t["cache_seqlens"],
                                  block_table=t["block_table"])
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    assert _lib.read_error_flags() == 0
    # one sequence of each length, at the front and at the end of the batch
    picks = sorted({0, 1, 2, 3, 4, batch - 5, batch - 4, batch - 3, batch - 2, batch - 1})
    _sampled_check(t, out, None, lengths, picks, dt, f"B{batch} gq{gq} d{d}")


def test_largest_cell_b256_ctx8192(cuda_device):
    """B=256 x 8192 tokens, Hk=4, D=128 (4.29 GB of K/V): default plan and an explicit 4-way split."""
    import torch

    from mxflashattn_b200 import _lib, backend

    batch, gq, d, dt = 256, 8, 128, "bf16"
    lengths = [8192] * batch
    t = syn.device_paged_decode(seed=4290, lengths=lengths, q_heads=4 * gq, kv_heads=4, head_dim=d, dtype=dt,
                                page_size=PAGE, device=cuda_device)
    assert t["k_cache"].numel() * t["k_cache"].element_size() * 2 == batch * 8192 * 4 * d * 2 * 2
    _outliers(t, 4291)
    cap = PAGE * t["block_table"].shape[1]
    rng = np.random.default_rng(4292)
    picks = sorted(set(rng.choice(batch, size=4, replace=False).tolist()) | {0, batch - 1})
    for splits in (0, 4):
        out, lse = backend.kvcache_attention(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"],
                                             t["block_table"], d ** -0.5, False, return_lse=True,
                                             num_splits=splits, chunk_len=-(-cap // splits) if splits else 0)
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        assert _lib.read_error_flags() == 0
        _sampled_check(t, out, lse, lengths, picks, dt, f"largest cell splits={splits}")
