"""GPU parity of decode over e4m3 (FP8) KV caches.

The caches are quantised on the host with torch's float8_e4m3fn cast; the
oracle runs the reference algorithm on the dequantised values (stored x
scale), so the comparison isolates the kernel: widening e4m3 to f16 is exact,
and the remaining error is q's f16 rounding, P's f16 hi/lo split and the
output's own rounding -- the same bound as the 16-bit path.
"""

from __future__ import annotations

import dataclasses

import numpy as np
import pytest

from helpers import assert_close_lse, assert_close_out, host, oracle_paged
from mxflashattn_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


def _quantise(x: np.ndarray, scale: float):
    """(e4m3 CPU tensor of x / scale, its dequantised float32 values)."""
    import torch

    q8 = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32) / scale).to(torch.float8_e4m3fn)
    return q8, q8.to(torch.float32).numpy() * scale


def _fp8_case(case, k_scale, v_scale):
    kq, kd = _quantise(case.k_cache, k_scale)
    vq, vd = _quantise(case.v_cache, v_scale)
    kn = vn = None
    knd = vnd = None
    if case.k_new is not None:
        kn, knd = _quantise(case.k_new, k_scale)
        vn, vnd = _quantise(case.v_new, v_scale)
    deq = dataclasses.replace(case, k_cache=kd, v_cache=vd, k_new=knd, v_new=vnd)
    return (kq, vq, kn, vn), deq


def _dev(case, fp8, device, v_first=False):
    import torch

    kq, vq, kn, vn = fp8
    tdt = syn.torch_dtype(case.dtype)
    both = torch.empty((2,) + tuple(kq.shape), dtype=torch.float8_e4m3fn, device=device)
    k_c, v_c = (both[1], both[0]) if v_first else (both[0], both[1])
    k_c.copy_(kq.to(device))
    v_c.copy_(vq.to(device))
    return {
        "q": torch.from_numpy(case.q).to(device=device, dtype=tdt),
        "k_cache": k_c,
        "v_cache": v_c,
        "cache_seqlens": torch.from_numpy(case.cache_seqlens.copy()).to(device),
        "block_table": None if case.block_table is None else torch.from_numpy(case.block_table).to(device),
        "k": None if kn is None else kn.to(device),
        "v": None if vn is None else vn.to(device),
    }


@pytest.mark.parametrize("dt", ["bf16", "fp16"])
@pytest.mark.parametrize("gq,q_len", [(2, 1), (4, 1), (8, 1), (8, 2)])
@pytest.mark.parametrize("page_size", [16, 8])
def test_fp8_decode_matches_oracle(dt, gq, q_len, page_size, cuda_device):
    import torch

    from mxflashattn_b200 import _lib, backend

    case = syn.paged_case(1400 + gq * 3 + q_len * 7 + page_size, batch=4, q_heads=2 * gq, kv_heads=2,
                          head_dim=128, dtype=dt, page_size=page_size, lengths=[1, 33, 700, 129], q_len=q_len,
                          causal=q_len > 1)
    k_scale, v_scale = 0.25, 2.0
    fp8, deq = _fp8_case(case, k_scale, v_scale)
    t = _dev(case, fp8, cuda_device)
    ref, ref_lse = oracle_paged(deq)[:2]
    cap = page_size * case.block_table.shape[1]
    for splits in (0, 3):
        chunk = -(-cap // splits) if splits else 0
        out, lse = backend.kvcache_attention(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"],
                                             t["block_table"], case.softmax_scale, case.causal, return_lse=True,
                                             num_splits=splits, chunk_len=chunk, k_scale=k_scale, v_scale=v_scale)
        torch.cuda.synchronize()
        assert_close_out(host(out), ref, dt, f"fp8 gq{gq} Sq{q_len} ps{page_size} splits{splits}")
        assert_close_lse(host(lse), ref_lse, f"fp8 lse gq{gq} splits{splits}")
    assert _lib.read_error_flags() == 0


@pytest.mark.parametrize("v_first", [False, True])
def test_fp8_caches_in_either_address_order(v_first, cuda_device):
    import torch

    from mxflashattn_b200 import backend

    case = syn.paged_case(1450 + int(v_first), batch=3, q_heads=32, kv_heads=8, head_dim=128, dtype="bf16",
                          page_size=16, lengths=[300, 5, 1024])
    fp8, deq = _fp8_case(case, 1.0, 1.0)
    t = _dev(case, fp8, cuda_device, v_first=v_first)
    assert (t["v_cache"].data_ptr() < t["k_cache"].data_ptr()) == v_first
    out = backend.kvcache_attention(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"], t["block_table"],
                                    case.softmax_scale, False)
    torch.cuda.synchronize()
    assert_close_out(host(out), oracle_paged(deq)[0], "bf16", f"fp8 v_first={v_first}")


def test_fp8_public_api_with_append(cuda_device):
    """flash_attn_with_kvcache over e4m3 caches: e4m3 rows appended bit-exactly, lengths advanced."""
    import torch

    from mxflashattn_b200 import flash_attn_with_kvcache

    case = syn.paged_case(1460, batch=3, q_heads=16, kv_heads=4, head_dim=128, dtype="bf16", page_size=16,
                          lengths=[0, 100, 47], append=1, extra_table_cols=1)
    k_scale, v_scale = 0.5, 0.75
    fp8, deq = _fp8_case(case, k_scale, v_scale)
    t = _dev(case, fp8, cuda_device)
    out = flash_attn_with_kvcache(t["q"], t["k_cache"], t["v_cache"], k=t["k"], v=t["v"],
                                  cache_seqlens=t["cache_seqlens"], block_table=t["block_table"],
                                  softmax_scale=case.softmax_scale, k_scale=k_scale, v_scale=v_scale)
    torch.cuda.synchronize()
    ref, _, kc, vc, sl = oracle_paged(deq)
    assert_close_out(host(out), ref, "bf16", "fp8 api append")
    np.testing.assert_array_equal(t["k_cache"].to(torch.float32).cpu().numpy() * k_scale, kc)
    np.testing.assert_array_equal(t["v_cache"].to(torch.float32).cpu().numpy() * v_scale, vc)
    np.testing.assert_array_equal(t["cache_seqlens"].cpu().numpy(), sl)


def test_fp8_single_launch_equals_two_launches(cuda_device):
    import torch

    from mxflashattn_b200 import backend

    case = syn.paged_case(1470, batch=2, q_heads=32, kv_heads=8, head_dim=128, dtype="bf16", page_size=16,
                          lengths=[4000, 1500])
    fp8, _ = _fp8_case(case, 1.0, 1.0)
    t = _dev(case, fp8, cuda_device)
    outs = [backend.kvcache_attention(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"], t["block_table"],
                                      case.softmax_scale, False, num_splits=6, chunk_len=704, single_launch=s)
            for s in (False, True)]
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("splits", [0, 3])
def test_fp8_row_max_jumps_rescale(splits, cuda_device):
    """Keys scaled x12 at every 37th position: row maxima jump past the e4m3 path's 2^8 rescale threshold
    on many tiles after the first, so the accumulators are rescaled mid-sequence (and across splits)."""
    import torch

    from mxflashattn_b200 import backend

    case = syn.paged_case(1480 + splits, batch=3, q_heads=16, kv_heads=4, head_dim=128, dtype="bf16", page_size=16,
                          lengths=[900, 333, 1200])
    k_cache = case.k_cache.copy()
    for b, L in enumerate(case.cache_seqlens):
        for pos in range(5, int(L), 37):
            k_cache[case.block_table[b, pos // 16], pos % 16] *= 12.0
    case = dataclasses.replace(case, k_cache=k_cache)
    k_scale, v_scale = 0.25, 1.0  # boosted keys stay below e4m3's 448 after dividing by k_scale
    fp8, deq = _fp8_case(case, k_scale, v_scale)
    t = _dev(case, fp8, cuda_device)
    cap = 16 * case.block_table.shape[1]
    chunk = -(-cap // splits) if splits else 0
    out, lse = backend.kvcache_attention(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"], t["block_table"],
                                         case.softmax_scale, False, return_lse=True, num_splits=splits,
                                         chunk_len=chunk, k_scale=k_scale, v_scale=v_scale)
    torch.cuda.synchronize()
    ref, ref_lse = oracle_paged(deq)[:2]
    assert_close_out(host(out), ref, "bf16", f"fp8 rescale splits{splits}")
    assert_close_lse(host(lse), ref_lse, f"fp8 rescale lse splits{splits}")
