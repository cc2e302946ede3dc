"""The workload grid on which the dispatch policy's decisions are recorded and compared.

Shared by ``make_policy_decisions.py`` (which runs the reference's policy)
and the policy test.  The grid straddles every threshold of both phases
under four configurations; ``invalid_shapes`` are rejected on construction.
"""

from __future__ import annotations

import itertools

CONFIGS = (
    {},
    {"enabled": True},
    {"enabled": True, "calibrated": True},
    {"enabled": True, "calibrated": True, "prefill_batch_min": 2, "prefill_kv_len_min": 100,
     "decode_batch_min": 5, "decode_kv_len_min": 64},
)
PHASES = ("prefill", "decode")
BATCHES = (1, 2, 3, 4, 5, 15, 16, 64)
KV_LENS = (1, 63, 64, 99, 100, 255, 256, 511, 512, 4096)
HEAD_DIMS = (32, 64, 96, 128)
GQA = (1, 2, 3, 4, 8, 16)


def grid():
    """(config index, phase, batch, query_len, kv_len, head_dim, gqa) in a fixed order."""
    for c, phase, b, kv, d, g in itertools.product(range(len(CONFIGS)), PHASES, BATCHES, KV_LENS, HEAD_DIMS, GQA):
        yield c, phase, b, 1 if phase == "decode" else 17, kv, d, g


def invalid_shapes():
    return {
        "phase": ("train", 1, 1, 1, 64, 1),
        "zero_batch": ("decode", 0, 1, 1, 64, 1),
        "zero_query": ("prefill", 1, 0, 1, 64, 1),
        "negative_kv": ("decode", 1, 1, -5, 64, 1),
        "zero_head_dim": ("decode", 1, 1, 1, 0, 1),
        "zero_gqa": ("decode", 1, 1, 1, 64, 0),
    }
