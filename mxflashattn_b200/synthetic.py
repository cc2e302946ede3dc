"""Seeded synthetic inputs with the shapes of the benchmark configurations.

The reference measures on synthetic tensors only (no dataset); these
generators reproduce its configurations (paged decode, coverage matrix,
long-context, varlen prefill) deterministically from a seed so that tests,
golden-vector generation and the benchmark all see identical inputs.

Small cases are produced in numpy (values rounded onto the bf16/fp16 grid so
that converting them to a torch tensor of that dtype is lossless).  Large
benchmark workloads are produced directly on the device with a seeded torch
generator (``device_paged_decode``), never through host memory.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

DTYPES = ("bf16", "fp16")


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), as float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    bits = x.view(np.uint32).astype(np.uint64)
    lsb = (bits >> np.uint64(16)) & np.uint64(1)
    rounded = ((bits + np.uint64(0x7FFF) + lsb) >> np.uint64(16)) << np.uint64(16)
    out = (rounded & np.uint64(0xFFFFFFFF)).astype(np.uint32).view(np.float32)
    return np.where(np.isnan(x), x, out).astype(np.float32)


def round_dtype(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round to the storage grid of ``dtype`` ('bf16', 'fp16' or 'fp32')."""
    if dtype == "bf16":
        return round_bf16(x)
    if dtype == "fp16":
        return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)
    if dtype == "fp32":
        return np.asarray(x, np.float32)
    raise ValueError(f"unknown dtype {dtype!r}")


def torch_dtype(dtype: str):
    import torch

    return {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[dtype]


def _normal(rng: np.random.Generator, shape, outlier_frac: float = 0.0, outlier_scale: float = 50.0):
    x = rng.standard_normal(shape, dtype=np.float32)
    if outlier_frac > 0:
        mask = rng.random(shape) < outlier_frac
        x = np.where(mask, x * np.float32(outlier_scale), x)
    return x


@dataclass
class PagedCase:
    """One ``flash_attn_with_kvcache`` call on a paged (or dense) cache."""

    q: np.ndarray                 # [B, Sq, HQ, D]
    k_cache: np.ndarray           # paged [P, PS, HKV, D] or dense [B, S, HKV, D]
    v_cache: np.ndarray
    cache_seqlens: np.ndarray     # int32 [B]
    block_table: np.ndarray | None  # int32 [B, BTW] or None (dense cache)
    dtype: str
    softmax_scale: float
    k_new: np.ndarray | None = None  # [B, Sk, HKV, D]
    v_new: np.ndarray | None = None
    causal: bool = False
    meta: dict = field(default_factory=dict)

    @property
    def total_lengths(self) -> np.ndarray:
        extra = 0 if self.k_new is None else self.k_new.shape[1]
        return self.cache_seqlens.astype(np.int64) + extra


def paged_case(
    seed: int,
    *,
    batch: int,
    q_heads: int,
    kv_heads: int,
    head_dim: int,
    dtype: str,
    page_size: int,
    lengths,
    num_pages: int | None = None,
    q_len: int = 1,
    append: int = 0,
    outlier_frac: float = 0.0,
    poison: float | None = None,
    softmax_scale: float | None = None,
    causal: bool = False,
    dense: bool = False,
    extra_table_cols: int = 0,
) -> PagedCase:
    """Seeded paged-decode case.

    ``lengths`` are the cached lengths before the call; ``append`` new tokens
    per sequence are added by the call.  The block table is a random
    permutation of the physical pages (as in the benchmark configuration).
    ``poison`` fills every cache slot that no sequence covers with that value
    (e.g. NaN) so tests can prove padding never leaks into a result.
    """
    rng = np.random.default_rng(seed)
    lengths = np.asarray(lengths, dtype=np.int64)
    assert lengths.shape == (batch,)
    totals = lengths + append
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(head_dim)
    q = round_dtype(_normal(rng, (batch, q_len, q_heads, head_dim)), dtype)
    if dense:
        cap = max(int(totals.max()), 1) + extra_table_cols
        shape = (batch, cap, kv_heads, head_dim)
        block_table = None
    else:
        width = max(int(max((t + page_size - 1) // page_size for t in totals)), 1) + extra_table_cols
        needed = batch * width
        num_pages = max(num_pages or needed, needed)
        perm = rng.permutation(num_pages).astype(np.int32)
        block_table = perm[:needed].reshape(batch, width).copy()
        shape = (num_pages, page_size, kv_heads, head_dim)
    k_cache = round_dtype(_normal(rng, shape, outlier_frac), dtype)
    v_cache = round_dtype(_normal(rng, shape, outlier_frac), dtype)
    k_new = v_new = None
    if append:
        k_new = round_dtype(_normal(rng, (batch, append, kv_heads, head_dim), outlier_frac), dtype)
        v_new = round_dtype(_normal(rng, (batch, append, kv_heads, head_dim), outlier_frac), dtype)
    if poison is not None:
        used = np.zeros(shape[:2], dtype=bool)
        for b in range(batch):
            # slots that hold cached tokens before the call stay valid; slots
            # the append will write are poisoned too (the append overwrites them)
            for pos in range(int(lengths[b])):
                if dense:
                    used[b, pos] = True
                else:
                    used[block_table[b, pos // page_size], pos % page_size] = True
        k_cache[~used] = poison
        v_cache[~used] = poison
    return PagedCase(
        q=q,
        k_cache=k_cache,
        v_cache=v_cache,
        cache_seqlens=lengths.astype(np.int32),
        block_table=block_table,
        dtype=dtype,
        softmax_scale=scale,
        k_new=k_new,
        v_new=v_new,
        causal=causal,
        meta={"seed": seed, "page_size": page_size, "outlier_frac": outlier_frac},
    )


# ---------------------------------------------------------------- configurations

def config1_case(seed: int = 0) -> PagedCase:
    """Benchmark config 1: B=4, Hq=8, Hk=2, D=128, bf16, page 16, ctx U[1,512], 160 pages."""
    rng = np.random.default_rng(seed)
    lengths = rng.integers(1, 513, size=4)
    return paged_case(seed + 1, batch=4, q_heads=8, kv_heads=2, head_dim=128, dtype="bf16",
                      page_size=16, lengths=lengths, num_pages=160)


def qwen3_4b_lengths(seed: int, batch: int = 128) -> np.ndarray:
    """Config 2 context lengths: prompt U[128,1024] plus U[1,256] generated tokens."""
    rng = np.random.default_rng(seed)
    return rng.integers(128, 1025, size=batch) + rng.integers(1, 257, size=batch)


def qwen3_8b_lengths(seed: int, batch: int = 16) -> np.ndarray:
    """Config 3 context lengths: U[256,1280]."""
    rng = np.random.default_rng(seed)
    return rng.integers(256, 1281, size=batch)


@dataclass
class VarlenCase:
    q: np.ndarray      # [Tq, HQ, D]
    k: np.ndarray      # [Tk, HKV, D]
    v: np.ndarray
    cu_q: np.ndarray   # int32 [B+1]
    cu_k: np.ndarray
    dtype: str
    softmax_scale: float
    causal: bool


def varlen_case(seed: int, *, q_lens, k_lens=None, q_heads: int, kv_heads: int, head_dim: int,
                dtype: str, causal: bool = True, softmax_scale: float | None = None,
                outlier_frac: float = 0.0) -> VarlenCase:
    rng = np.random.default_rng(seed)
    k_lens = q_lens if k_lens is None else k_lens
    cu_q = np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int32)
    cu_k = np.concatenate([[0], np.cumsum(k_lens)]).astype(np.int32)
    q = round_dtype(_normal(rng, (int(cu_q[-1]), q_heads, head_dim)), dtype)
    k = round_dtype(_normal(rng, (int(cu_k[-1]), kv_heads, head_dim), outlier_frac), dtype)
    v = round_dtype(_normal(rng, (int(cu_k[-1]), kv_heads, head_dim), outlier_frac), dtype)
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(head_dim)
    return VarlenCase(q, k, v, cu_q, cu_k, dtype, scale, causal)


# ------------------------------------------------------- device-side (benchmark)

def device_paged_decode(
    *,
    seed: int,
    lengths,
    q_heads: int,
    kv_heads: int,
    head_dim: int,
    dtype: str,
    page_size: int,
    device,
    spare_pages: int = 0,
):
    """Large paged-decode inputs generated on the device (no host round trip).

    Returns a dict of device tensors: q [B,1,HQ,D], k_cache/v_cache
    [P,PS,HKV,D], block_table int32 [B,BTW] (random permutation of the
    pages), cache_seqlens int32 [B].
    """
    import torch

    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    lengths = [int(x) for x in lengths]
    batch = len(lengths)
    width = max((L + spare_pages * page_size + page_size - 1) // page_size for L in lengths)
    # allocate exactly the pages the sequences occupy (plus spares), like a paged
    # serving cache, and scatter them over a random permutation
    need = [(L + spare_pages * page_size + page_size - 1) // page_size for L in lengths]
    pages = max(sum(need), 1)
    tdt = torch_dtype(dtype)
    k_cache = torch.randn((pages, page_size, kv_heads, head_dim), generator=gen, device=device, dtype=tdt)
    v_cache = torch.randn((pages, page_size, kv_heads, head_dim), generator=gen, device=device, dtype=tdt)
    perm = torch.randperm(pages, generator=gen, device=device).to(torch.int32).cpu().numpy()
    table = np.zeros((batch, width), dtype=np.int32)
    offset = 0
    for b, n in enumerate(need):
        table[b, :n] = perm[offset:offset + n]
        offset += n
    block_table = torch.from_numpy(table).to(device)
    q = torch.randn((batch, 1, q_heads, head_dim), generator=gen, device=device, dtype=tdt)
    seqlens = torch.tensor(lengths, dtype=torch.int32, device=device)
    return {"q": q, "k_cache": k_cache, "v_cache": v_cache, "block_table": block_table,
            "cache_seqlens": seqlens}


def kv_bytes(lengths, kv_heads: int, head_dim: int, elem_bytes: int = 2) -> int:
    """Algorithmic K+V bytes one decode step reads: sum_b len_b * Hk * D * 2 (K,V) * elem."""
    return int(sum(int(x) for x in lengths)) * kv_heads * head_dim * 2 * elem_bytes
