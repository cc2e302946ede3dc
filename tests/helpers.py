"""Test helpers: seeded cases -> device tensors, oracle calls, tolerances."""

from __future__ import annotations

import numpy as np

import oracle
from mxflashattn_b200 import synthetic as syn

# Output tolerances against the fp32 oracle: max-abs 2e-3 for
# fp16, 1e-2 for bf16; LSE within 1e-3.
OUT_ATOL = {"fp16": 2e-3, "bf16": 1e-2}
LSE_ATOL = 1e-3


def to_device(case, device):
    import torch

    tdt = syn.torch_dtype(case.dtype)
    t = {
        "q": torch.from_numpy(case.q).to(device=device, dtype=tdt),
        "k_cache": torch.from_numpy(case.k_cache).to(device=device, dtype=tdt),
        "v_cache": torch.from_numpy(case.v_cache).to(device=device, dtype=tdt),
        "cache_seqlens": torch.from_numpy(case.cache_seqlens.copy()).to(device),
        "block_table": None if case.block_table is None else torch.from_numpy(case.block_table).to(device),
        "k": None if case.k_new is None else torch.from_numpy(case.k_new).to(device=device, dtype=tdt),
        "v": None if case.v_new is None else torch.from_numpy(case.v_new).to(device=device, dtype=tdt),
    }
    return t


def oracle_paged(case, precision=np.float32):
    """(out, lse [B, Sq, HQ], k_cache_after, v_cache_after, seqlens_after) from the oracle."""
    kc, vc, sl = case.k_cache.copy(), case.v_cache.copy(), case.cache_seqlens.copy()
    out, lse = oracle.attention_kvcache(case.q, kc, vc, cache_seqlens=sl, block_table=case.block_table,
                                        k=case.k_new, v=case.v_new, softmax_scale=case.softmax_scale,
                                        causal=case.causal, precision=precision, return_lse=True)
    return out, lse.transpose(0, 2, 1), kc, vc, sl


def max_abs(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b))) if a.size else 0.0


def assert_close_out(actual, expected, dtype, what=""):
    err = max_abs(actual, expected)
    assert np.isfinite(np.asarray(actual, np.float64)).all(), f"{what}: non-finite output"
    assert err <= OUT_ATOL[dtype], f"{what}: max abs err {err:.3e} > {OUT_ATOL[dtype]:.0e} ({dtype})"


def assert_close_lse(actual, expected, what=""):
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    both_inf = np.isneginf(a) & np.isneginf(e)
    err = float(np.max(np.abs(np.where(both_inf, 0.0, a - e)))) if a.size else 0.0
    assert err <= LSE_ATOL, f"{what}: LSE max abs err {err:.3e} > {LSE_ATOL:.0e}"


def host(t) -> np.ndarray:
    return t.detach().float().cpu().numpy()
