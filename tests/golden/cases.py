"""Seeded golden-vector cases shared by ``make_golden.py`` and the tests.

Every case is rebuilt from its seed by ``mxflashattn_b200.synthetic``; the
committed ``.npz`` fixtures hold only the reference's outputs (plus a digest
of the inputs so a generator drift is caught instead of silently compared).
"""

from __future__ import annotations

import hashlib

import numpy as np

from mxflashattn_b200 import synthetic as syn


def digest(*arrays) -> str:
    h = hashlib.sha1()
    for a in arrays:
        if a is None:
            h.update(b"none")
            continue
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def paged_cases():
    """name -> PagedCase for ``flash_attn_with_kvcache`` goldens."""
    cases = {"config1": syn.config1_case(0)}
    cases["append_paged_bf16"] = syn.paged_case(
        11, batch=3, q_heads=8, kv_heads=2, head_dim=64, dtype="bf16", page_size=16,
        lengths=[5, 16, 31], append=1)
    cases["append_paged_fp16_ps4"] = syn.paged_case(
        12, batch=2, q_heads=4, kv_heads=1, head_dim=128, dtype="fp16", page_size=4,
        lengths=[2, 7], append=1, num_pages=9)
    cases["append_dense_q2_causal"] = syn.paged_case(
        13, batch=2, q_heads=4, kv_heads=2, head_dim=64, dtype="bf16", page_size=1,
        lengths=[3, 9], q_len=2, append=2, causal=True, dense=True, extra_table_cols=3)
    cases["ps2_table_order"] = syn.paged_case(
        14, batch=2, q_heads=2, kv_heads=1, head_dim=64, dtype="fp16", page_size=2,
        lengths=[3, 6], num_pages=10)
    cases["q3_paged_causal"] = syn.paged_case(
        15, batch=2, q_heads=8, kv_heads=2, head_dim=128, dtype="bf16", page_size=16,
        lengths=[40, 1], q_len=3, append=3, causal=True)
    seed = 100
    for gq in (2, 4, 8):
        for d in (64, 128):
            for dt in ("fp16", "bf16"):
                cases[f"cov_gq{gq}_d{d}_{dt}"] = syn.paged_case(
                    seed, batch=3, q_heads=4 * gq, kv_heads=4, head_dim=d, dtype=dt, page_size=16,
                    lengths=[1, 17, 100], outlier_frac=0.01)
                seed += 1
    return cases


def varlen_cases():
    """name -> VarlenCase for ``flash_attn_varlen_func`` goldens."""
    return {
        "varlen_causal_bf16": syn.varlen_case(
            200, q_lens=[37, 64, 5], q_heads=4, kv_heads=2, head_dim=64, dtype="bf16", causal=True),
        "varlen_noncausal_fp16_k_longer": syn.varlen_case(
            201, q_lens=[3, 20], k_lens=[9, 33], q_heads=8, kv_heads=2, head_dim=128, dtype="fp16",
            causal=False),
        "varlen_causal_q_longer_than_k": syn.varlen_case(
            202, q_lens=[6, 4], k_lens=[2, 4], q_heads=2, kv_heads=1, head_dim=64, dtype="bf16",
            causal=True),
        "varlen_causal_d128_gq4": syn.varlen_case(
            203, q_lens=[70, 1, 33], q_heads=8, kv_heads=2, head_dim=128, dtype="bf16", causal=True,
            outlier_frac=0.01),
        "varlen_zero_scale": syn.varlen_case(
            204, q_lens=[2, 5], k_lens=[5, 3], q_heads=4, kv_heads=2, head_dim=64, dtype="fp16",
            causal=False, softmax_scale=0.0),
    }


class ChunkedCase:
    """Dense [B, S, H, D] inputs of a chunked-prefill golden and the chunk size it runs with."""

    def __init__(self, base, batch: int, chunk_size: int):
        self.q = base.q.reshape(batch, -1, *base.q.shape[1:])
        self.k = base.k.reshape(batch, -1, *base.k.shape[1:])
        self.v = base.v.reshape(batch, -1, *base.v.shape[1:])
        self.dtype, self.softmax_scale, self.causal = base.dtype, base.softmax_scale, base.causal
        self.chunk_size = chunk_size


def chunked_cases():
    """name -> ChunkedCase for the chunked online-softmax prototype (``prefill.py``) goldens."""
    return {
        "chunked_causal_bf16_c7": ChunkedCase(syn.varlen_case(
            300, q_lens=[33, 33], q_heads=4, kv_heads=2, head_dim=64, dtype="bf16", causal=True), 2, 7),
        "chunked_noncausal_fp16_k_longer_c64": ChunkedCase(syn.varlen_case(
            301, q_lens=[5, 5], k_lens=[130, 130], q_heads=8, kv_heads=2, head_dim=128, dtype="fp16",
            causal=False), 2, 64),
        "chunked_causal_q_longer_than_k_c1": ChunkedCase(syn.varlen_case(
            302, q_lens=[6], k_lens=[4], q_heads=2, kv_heads=1, head_dim=64, dtype="bf16", causal=True), 1, 1),
        "chunked_causal_outliers_c16": ChunkedCase(syn.varlen_case(
            303, q_lens=[48], q_heads=4, kv_heads=2, head_dim=128, dtype="bf16", causal=True,
            outlier_frac=0.01), 1, 16),
        "chunked_one_chunk_c256": ChunkedCase(syn.varlen_case(
            304, q_lens=[40, 40, 40], q_heads=4, kv_heads=4, head_dim=64, dtype="fp16", causal=True), 3, 256),
        "chunked_zero_scale_c3": ChunkedCase(syn.varlen_case(
            305, q_lens=[4, 4], k_lens=[9, 9], q_heads=4, kv_heads=2, head_dim=64, dtype="fp16", causal=False,
            softmax_scale=0.0), 2, 3),
    }
