"""Test helpers: seeded cases -> device tensors, oracle calls, tolerances."""

from __future__ import annotations

import numpy as np

import oracle
from mxflashattn_b200 import synthetic as syn

# Output tolerances against the fp32 oracle: max-abs 2e-3 for
# fp16, 1e-2 for bf16; LSE within 1e-3.  An output stored in bf16/fp16 cannot
# be closer to the fp32 value than half a storage ulp, so where |ref| is large
# (the x50-outlier cases) the bound is that half ulp instead:
#     |ours - ref| <= max(atol, half_ulp_rel * |ref|) + extra
# ``extra`` is used only by the prefill kernel, whose P@V product rounds P to
# the storage dtype once (as FlashAttention does): its error is at most
# u_P * sum(p |v|) / sum(p), computed by the oracle as attention over |V|.
OUT_ATOL = {"fp16": 2e-3, "bf16": 1e-2}
HALF_ULP_REL = {"fp16": 2.0 ** -11, "bf16": 2.0 ** -8}
P_ROUND_REL = {"fp16": 2.0 ** -11, "bf16": 2.0 ** -8}
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


def out_tolerance(expected, dtype, extra=0.0, ulps: float = 1.0):
    e = np.abs(np.asarray(expected, np.float64))
    return np.maximum(OUT_ATOL[dtype], ulps * HALF_ULP_REL[dtype] * e * 1.001 + 1e-6 * e) + extra


def assert_close_out(actual, expected, dtype, what="", extra=0.0, ulps: float = 1.0):
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    assert np.isfinite(a).all(), f"{what}: non-finite output"
    err = np.abs(a - e)
    tol = out_tolerance(e, dtype, extra, ulps)
    bad = err > tol
    if bad.any():
        i = np.unravel_index(np.argmax(err - tol), err.shape)
        raise AssertionError(f"{what}: {int(bad.sum())} elements out of tolerance; worst at {i}: "
                             f"|{a[i]:.6g} - {e[i]:.6g}| = {err[i]:.3e} > {np.broadcast_to(tol, err.shape)[i]:.3e} "
                             f"({dtype}); max abs err {err.max():.3e}")


def p_rounding_bound(dtype, abs_v_attention):
    """Prefill P-rounding error bound: u_P * (softmax-weighted mean of |V|)."""
    return P_ROUND_REL[dtype] * np.abs(np.asarray(abs_v_attention, np.float64)) * 1.01 + 1e-6


def assert_close_lse(actual, expected, what=""):
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    both_inf = np.isneginf(a) & np.isneginf(e)
    with np.errstate(invalid="ignore"):  # -inf - -inf is masked out just below
        diff = a - e
    err = float(np.max(np.abs(np.where(both_inf, 0.0, diff)))) if a.size else 0.0
    assert err <= LSE_ATOL, f"{what}: LSE max abs err {err:.3e} > {LSE_ATOL:.0e}"


def host(t) -> np.ndarray:
    return t.detach().float().cpu().numpy()
