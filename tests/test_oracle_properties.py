"""Size-independent identities of the oracle's split-KV algebra (CPU, hypothesis).

The decode kernel's split plan, its single-launch merge and the
context-parallel exchange all rest on one identity: attention over a key set
is the LSE merge of attention over any partition of it, in any order and in
any grouping.  These properties pin that identity on the oracle
(split_partials / merge_partials, after m1_kernel.cpp:846-888, and
attention_single, after reference.py:8-40) for random lengths, split plans,
rank partitions and merge orders, so the GPU parity tests can lean on it at
sizes the oracle cannot reach.
"""

from __future__ import annotations

import math

import numpy as np
from hypothesis import given, settings
from hypothesis import strategies as st

import oracle

LOG2E = oracle.attention.LOG2E
SETTINGS = settings(max_examples=40, deadline=None)


def _row_case(seed: int, length: int, dim: int):
    rng = np.random.default_rng(seed)
    keys = rng.standard_normal((length, dim))
    values = rng.standard_normal((length, dim))
    q = rng.standard_normal(dim) * 2.0  # sharper rows than N(0,1) scores alone give
    return q, keys, values


def _full(q, keys, values, scale):
    out, lse = oracle.attention_single(q[None, None], keys[:, None], values[:, None], softmax_scale=scale,
                                       precision=np.float64, return_lse=True)
    return out[0, 0], float(lse[0, 0])


def _record(out, lse):
    """(O, LSE) as a partial: o = O, m = lse * log2 e, d = 1 (empty: m = -inf, d = 0)."""
    if not math.isfinite(lse):
        return np.zeros_like(out), -np.inf, 0.0
    return out, lse * LOG2E, 1.0


@SETTINGS
@given(seed=st.integers(0, 2**31 - 1), length=st.integers(1, 700), chunk=st.integers(1, 256),
       extra=st.integers(0, 3), dim=st.sampled_from([16, 64]))
def test_any_split_plan_merges_to_the_full_softmax(seed, length, chunk, extra, dim):
    """NP chunks of chunk_len covering the sequence (plus empty trailing chunks) merge to the full row."""
    q, keys, values = _row_case(seed, length, dim)
    scale = 1.0 / math.sqrt(dim)
    num_splits = -(-length // chunk) + extra
    o, m, d = oracle.split_partials(q, keys, values, scale, num_splits, chunk)
    out, lse = oracle.merge_partials(o, m, d)
    full, full_lse = _full(q, keys, values, scale)
    np.testing.assert_allclose(out, full, rtol=1e-10, atol=1e-12)
    assert abs(lse - full_lse) < 1e-10


@SETTINGS
@given(seed=st.integers(0, 2**31 - 1), length=st.integers(1, 500), chunk=st.integers(1, 64),
       perm_seed=st.integers(0, 2**31 - 1))
def test_merge_ignores_the_order_of_the_partials(seed, length, chunk, perm_seed):
    q, keys, values = _row_case(seed, length, 32)
    num_splits = -(-length // chunk)
    o, m, d = oracle.split_partials(q, keys, values, 0.2, num_splits, chunk)
    perm = np.random.default_rng(perm_seed).permutation(num_splits)
    a_out, a_lse = oracle.merge_partials(o, m, d)
    b_out, b_lse = oracle.merge_partials(o[perm], m[perm], d[perm])
    np.testing.assert_allclose(a_out, b_out, rtol=1e-12, atol=1e-14)
    assert abs(a_lse - b_lse) < 1e-12


@SETTINGS
@given(seed=st.integers(0, 2**31 - 1), length=st.integers(1, 600), chunk=st.integers(1, 128),
       groups=st.integers(1, 6))
def test_merging_in_two_levels_equals_one_merge(seed, length, chunk, groups):
    """Splits merged per group into (O, LSE) records, then the records merged, equal one flat merge."""
    q, keys, values = _row_case(seed, length, 32)
    num_splits = -(-length // chunk)
    o, m, d = oracle.split_partials(q, keys, values, 0.15, num_splits, chunk)
    flat_out, flat_lse = oracle.merge_partials(o, m, d)
    bounds = np.linspace(0, num_splits, groups + 1).astype(int)
    recs = [_record(*oracle.merge_partials(o[a:b], m[a:b], d[a:b])) if b > a else (np.zeros(32), -np.inf, 0.0)
            for a, b in zip(bounds, bounds[1:])]
    out, lse = oracle.merge_partials(np.stack([r[0] for r in recs]), np.array([r[1] for r in recs]),
                                     np.array([r[2] for r in recs]))
    np.testing.assert_allclose(out, flat_out, rtol=1e-10, atol=1e-12)
    assert abs(lse - flat_lse) < 1e-10


@SETTINGS
@given(seed=st.integers(0, 2**31 - 1), pages=st.integers(1, 40), page_size=st.sampled_from([1, 16, 32]),
       world=st.integers(1, 8), tail=st.integers(0, 15))
def test_context_ranges_per_rank_merge_to_the_full_attention(seed, pages, page_size, world, tail):
    """Each rank attends over its page-aligned range of the context (ranks past the end hold none); the
    ranks' (O, LSE) records, merged in rank order, equal attention over the whole context."""
    length = max(1, pages * page_size - min(tail, page_size - 1))
    q, keys, values = _row_case(seed, length, 64)
    scale = 0.125
    per_rank = -(-pages // world) * page_size
    recs = []
    for rank in range(world):
        lo, hi = rank * per_rank, min((rank + 1) * per_rank, length)
        if hi <= lo:
            recs.append((np.zeros(64), -np.inf, 0.0))
            continue
        recs.append(_record(*_full(q, keys[lo:hi], values[lo:hi], scale)))
    out, lse = oracle.merge_partials(np.stack([r[0] for r in recs]), np.array([r[1] for r in recs]),
                                     np.array([r[2] for r in recs]))
    full, full_lse = _full(q, keys, values, scale)
    np.testing.assert_allclose(out, full, rtol=1e-10, atol=1e-12)
    assert abs(lse - full_lse) < 1e-10


@SETTINGS
@given(seed=st.integers(0, 2**31 - 1), q_len=st.integers(1, 24), extra_keys=st.integers(0, 40))
def test_causal_rows_see_the_bottom_right_aligned_prefix(seed, q_len, extra_keys):
    """Causal row i over k_len keys equals non-causal attention over keys [0, i + k_len - q_len]."""
    rng = np.random.default_rng(seed)
    k_len = q_len + extra_keys
    q = rng.standard_normal((q_len, 1, 32))
    k = rng.standard_normal((k_len, 1, 32))
    v = rng.standard_normal((k_len, 1, 32))
    causal = oracle.attention_single(q, k, v, softmax_scale=0.3, causal=True, precision=np.float64)
    for i in range(q_len):
        hi = i + k_len - q_len + 1
        row = oracle.attention_single(q[i:i + 1], k[:hi], v[:hi], softmax_scale=0.3, precision=np.float64)
        np.testing.assert_allclose(causal[i], row[0], rtol=1e-12, atol=1e-13)


@SETTINGS
@given(seed=st.integers(0, 2**31 - 1), q_len=st.integers(1, 40), extra_keys=st.integers(-3, 60),
       chunk=st.integers(1, 80), gq=st.sampled_from([1, 2, 4]), causal=st.booleans())
def test_chunked_online_softmax_equals_the_direct_oracle(seed, q_len, extra_keys, chunk, gq, causal):
    """The chunked prototype's restatement (prefill.py:11-81) against attention_batched, as the reference's own
    prefill tests check it: any chunk size, GQA, causal rows with and without visible keys."""
    rng = np.random.default_rng(seed)
    k_len = max(1, q_len + extra_keys)
    q = rng.standard_normal((2, q_len, 2 * gq, 32)).astype(np.float32)
    k = (rng.standard_normal((2, k_len, 2, 32)) * 1.5).astype(np.float32)
    v = rng.standard_normal((2, k_len, 2, 32)).astype(np.float32)
    chunked = oracle.attention_chunked(q, k, v, chunk_size=chunk, softmax_scale=0.2, causal=causal)
    direct = oracle.attention_batched(q, k, v, softmax_scale=0.2, causal=causal)
    np.testing.assert_allclose(chunked, direct, rtol=2e-5, atol=2e-5)


def test_long_context_chunked_error_summary_is_stable():
    """Causal self-attention over 128, 512 and 4096 tokens, chunk 64: the chunked oracle against the direct one
    through the error report, at the bounds of the reference's long-context test (test_long_context_accuracy.py:
    max 1e-4, p99 1e-5) plus a 4096-token case."""
    import torch

    from mxflashattn_b200.accuracy import summarize_error

    for kv_len in (128, 512, 4096):
        rng = np.random.default_rng(20261016 + kv_len)
        q = rng.standard_normal((1, kv_len, 2, 64)).astype(np.float32)
        k = rng.standard_normal((1, kv_len, 1, 64)).astype(np.float32)
        v = rng.standard_normal((1, kv_len, 1, 64)).astype(np.float32)
        chunked = oracle.attention_chunked(q, k, v, chunk_size=64, causal=True)
        direct = oracle.attention_batched(q, k, v, causal=True)
        summary = summarize_error(torch.from_numpy(chunked), torch.from_numpy(direct))
        assert summary.finite
        assert summary.max_abs < 1e-4 and summary.p99_abs < 1e-5, (kv_len, summary)
