"""Pin the numpy oracle against golden vectors produced by the reference itself.

The fixtures come from ``tests/golden/make_golden.py``, which ran the
reference's ``mxflashattn/reference.py`` (PyTorch, CPU) on the same seeded
inputs.  The oracle must reproduce the reference's float32 result, its
dtype-cast result, the harness LSE and the bit-exact append placement.
"""

from __future__ import annotations

import os

import numpy as np
import pytest

import cases as golden_cases
import oracle
from mxflashattn_b200 import synthetic as syn

PAGED = golden_cases.paged_cases()
VARLEN = golden_cases.varlen_cases()


def _run_paged(case, precision=np.float32):
    kc, vc, sl = case.k_cache.copy(), case.v_cache.copy(), case.cache_seqlens.copy()
    out, lse = oracle.attention_kvcache(
        case.q, kc, vc, cache_seqlens=sl, block_table=case.block_table, k=case.k_new, v=case.v_new,
        softmax_scale=case.softmax_scale, causal=case.causal, precision=precision, return_lse=True)
    return out, lse, kc, vc, sl


@pytest.mark.parametrize("name", sorted(PAGED))
def test_oracle_matches_reference_paged(name, golden):
    case = PAGED[name]
    assert golden[f"{name}.digest"].item() == golden_cases.digest(
        case.q, case.k_cache, case.v_cache, case.block_table, case.cache_seqlens, case.k_new, case.v_new)
    out, lse, kc, vc, sl = _run_paged(case)
    # float32 pipeline vs the reference's float32 pipeline: summation order only
    np.testing.assert_allclose(out, golden[f"{name}.out_f32"], rtol=1e-5, atol=2e-5)
    # final downcast: at most one storage ulp apart where float32 sums straddle a rounding boundary
    cast = syn.round_dtype(out, case.dtype)
    ref = golden[f"{name}.out"]
    ulp = 2.0 ** -7 if case.dtype == "bf16" else 2.0 ** -10
    assert np.all(np.abs(cast - ref) <= ulp * np.maximum(np.abs(ref), 1e-3) + 1e-6)
    # LSE is [B, HQ, Sq] from the oracle; goldens are [B, Sq, HQ]
    np.testing.assert_allclose(lse.transpose(0, 2, 1), golden[f"{name}.lse"], rtol=1e-5, atol=1e-5)
    if case.k_new is not None:
        assert golden_cases.digest(kc) == golden[f"{name}.k_cache_after_digest"].item()
        assert golden_cases.digest(vc) == golden[f"{name}.v_cache_after_digest"].item()
        np.testing.assert_array_equal(sl, golden[f"{name}.seqlens_after"])


@pytest.mark.parametrize("name", sorted(VARLEN))
def test_oracle_matches_reference_varlen(name, golden):
    case = VARLEN[name]
    assert golden[f"{name}.digest"].item() == golden_cases.digest(case.q, case.k, case.v, case.cu_q, case.cu_k)
    out, lse = oracle.attention_varlen(case.q, case.k, case.v, case.cu_q, case.cu_k,
                                       softmax_scale=case.softmax_scale, causal=case.causal, return_lse=True)
    np.testing.assert_allclose(out, golden[f"{name}.out_f32"], rtol=1e-5, atol=2e-5)
    np.testing.assert_allclose(lse.T, golden[f"{name}.lse"], rtol=1e-5, atol=1e-5)


def test_float64_cross_check_agrees_with_float32_oracle():
    case = PAGED["config1"]
    o32 = _run_paged(case, np.float32)[0]
    o64 = _run_paged(case, np.float64)[0]
    assert np.max(np.abs(o32 - o64)) < 1e-5


def test_split_partials_merge_to_the_full_softmax():
    rng = np.random.default_rng(3)
    keys = rng.standard_normal((203, 64))
    values = rng.standard_normal((203, 64))
    q = rng.standard_normal(64)
    scale = 0.125
    full, full_lse = oracle.attention_single(q[None, None], keys[:, None], values[:, None],
                                             softmax_scale=scale, precision=np.float64, return_lse=True)
    for num_splits, chunk in ((1, 203), (4, 51), (7, 32), (9, 64)):
        o, m, d = oracle.split_partials(q, keys, values, scale, num_splits, chunk)
        out, lse = oracle.merge_partials(o, m, d)
        np.testing.assert_allclose(out, full[0, 0], rtol=1e-10, atol=1e-12)
        assert abs(lse - full_lse[0, 0]) < 1e-10


def test_empty_split_merge_is_zero():
    o = np.zeros((3, 8))
    m = np.full(3, -np.inf)
    d = np.zeros(3)
    out, lse = oracle.merge_partials(o, m, d)
    assert np.all(out == 0) and lse == -np.inf


CHUNKED = golden_cases.chunked_cases()


@pytest.fixture(scope="module")
def chunked_golden():
    with np.load(os.path.join(os.path.dirname(golden_cases.__file__), "chunked.npz")) as z:
        return {k: z[k] for k in z.files}


@pytest.mark.parametrize("name", sorted(CHUNKED))
def test_chunked_oracle_matches_the_reference_prototype(name, chunked_golden):
    """The chunked online-softmax restatement against the reference's own prefill_chunked_reference outputs."""
    case = CHUNKED[name]
    assert chunked_golden[f"{name}.digest"].item() == golden_cases.digest(case.q, case.k, case.v)
    kw = dict(chunk_size=case.chunk_size, softmax_scale=case.softmax_scale, causal=case.causal)
    out = oracle.attention_chunked(case.q, case.k, case.v, **kw)
    np.testing.assert_allclose(out, chunked_golden[f"{name}.out_f32"], rtol=1e-5, atol=2e-5)
    cast = syn.round_dtype(out, case.dtype)
    ref = chunked_golden[f"{name}.out"]
    ulp = 2.0 ** -7 if case.dtype == "bf16" else 2.0 ** -10
    assert np.all(np.abs(cast - ref) <= ulp * np.maximum(np.abs(ref), 1e-3) + 1e-6)
    if f"{name}.fallback_f32" in chunked_golden:
        fb = oracle.attention_chunked_fallback(case.q, case.k, case.v, **kw)
        np.testing.assert_allclose(fb, chunked_golden[f"{name}.fallback_f32"], rtol=1e-5, atol=2e-5)


def test_chunked_fallback_takes_the_direct_oracle_for_one_chunk():
    """One chunk covering every key runs attention_batched itself (prefill.py:98-99)."""
    case = CHUNKED["chunked_one_chunk_c256"]
    fb = oracle.attention_chunked_fallback(case.q, case.k, case.v, chunk_size=case.k.shape[1],
                                           softmax_scale=case.softmax_scale, causal=case.causal)
    direct = oracle.attention_batched(case.q, case.k, case.v, softmax_scale=case.softmax_scale, causal=case.causal)
    assert np.array_equal(fb, direct)


@pytest.mark.parametrize("chunk_size", [0, -4, 2.5])
def test_chunked_oracle_rejects_invalid_chunk_sizes(chunk_size):
    """A chunk size that is not a positive integer is refused (prefill.py:28-29)."""
    case = CHUNKED["chunked_causal_bf16_c7"]
    with pytest.raises(ValueError, match="chunk_size must be a positive integer"):
        oracle.attention_chunked(case.q, case.k, case.v, chunk_size=chunk_size)
