"""The allocation-free KV-cache attention entry point, checked on the GPU.

``mxfa_kvcache_attention_noalloc_launch`` serves callers that cannot
allocate device memory when they run attention -- an engine that reserved
all of the GPU's memory for its own pools up front, a host written in
another language that reaches the library through a bare C FFI and has no
device allocator, or a latency-critical loop that must not risk the device
synchronisation a cudaMalloc can trigger.  Instead of a caller workspace it
keeps the split partials in one fixed buffer built into the library.

This test calls it through the C ABI twice in a row, on two different
inputs so that partials left in the shared buffer by the first call cannot
leak into the second.  Both entry points run the same decode and combine
kernels on the same inputs, so each result must equal the regular entry
point's (caller-provided workspace) bit for bit; each is also checked
against the CPU oracle within the decode tolerance the other tests use.
One case passes num_splits = chunk_len = 0 so the library plans the split
itself through this entry.  A request larger than the built-in buffer must
be refused with a clear error instead of being launched.  The file name
sorts last so that a run stopping at the first failure has already run
every other test.
"""

from __future__ import annotations

import ctypes
import re

import pytest

from helpers import assert_close_lse, assert_close_out, host, oracle_paged, to_device
from mxflashattn_b200 import _lib, synthetic as syn

pytestmark = pytest.mark.gpu


def _scratch_limit() -> int:
    import os

    header = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "mxfa_b200.h")
    m = re.search(r"#define MXFA_NOALLOC_SCRATCH_BYTES \((\d+)u << (\d+)\)", open(header).read())
    return int(m.group(1)) << int(m.group(2))


def _plan(lib, B, Sq, HQ, HKV, D, max_len):
    ns, cl = ctypes.c_int(0), ctypes.c_int(0)
    _lib.check(lib.mxfa_kvcache_plan(B, Sq, HQ, HKV, D, max_len, ctypes.byref(ns), ctypes.byref(cl)), "plan")
    return ns.value, cl.value


def _launch(case, t, splits, chunk, *, noalloc):
    import torch

    lib = _lib.load()
    B, Sq, HQ, D = case.q.shape
    HKV = case.k_cache.shape[2]
    PS = case.k_cache.shape[1]
    BTW = case.block_table.shape[1]
    out = torch.empty_like(t["q"])
    lse = torch.empty((B, Sq, HQ), device=t["q"].device, dtype=torch.float32)
    stream = torch.cuda.current_stream().cuda_stream
    common = (B, Sq, HQ, HKV, D, PS, BTW, case.k_cache.shape[0], 0, splits, chunk, 0, int(case.dtype == "bf16"),
              case.softmax_scale, stream)
    ptrs = (t["q"].data_ptr(), t["k_cache"].data_ptr(), t["v_cache"].data_ptr(), t["block_table"].data_ptr(),
            t["cache_seqlens"].data_ptr(), out.data_ptr(), lse.data_ptr())
    if noalloc:
        rc = lib.mxfa_kvcache_attention_noalloc_launch(*ptrs, *common)
    else:
        if splits <= 0 or chunk <= 0:  # the plan the library makes for the same call
            splits, chunk = _plan(lib, B, Sq, HQ, HKV, D, PS * BTW)
            common = common[:9] + (splits, chunk) + common[11:]
        ws_bytes = max(lib.mxfa_split_workspace_bytes(B * Sq * HQ, D, splits), 16)
        ws = torch.empty((ws_bytes // 4,), device=t["q"].device, dtype=torch.float32)
        rc = lib.mxfa_kvcache_attention_launch(*ptrs, ws.data_ptr(), ws_bytes, *common)
    _lib.check(rc, "noalloc test launch")
    torch.cuda.synchronize()
    return out, lse


CASES = [
    # (seed, batch, q_heads, kv_heads, head_dim, dtype, lengths, splits); splits 0 = library plan
    (4001, 3, 32, 8, 128, "bf16", [3000, 777, 1], 6),
    (4002, 2, 16, 4, 64, "fp16", [45, 2500], 9),
    (4003, 2, 32, 8, 128, "bf16", [5000, 1200], 0),
]


def test_noalloc_entry_matches_workspace_entry_on_two_calls_in_a_row(cuda_device):
    import torch

    lib = _lib.load()
    for seed, batch, hq, hkv, d, dt, lengths, splits in CASES:
        case = syn.paged_case(seed, batch=batch, q_heads=hq, kv_heads=hkv, head_dim=d, dtype=dt, page_size=16,
                              lengths=lengths, outlier_frac=0.01)
        t = to_device(case, cuda_device)
        cap = 16 * case.block_table.shape[1]
        chunk = -(-cap // splits) if splits > 0 else 0
        if splits == 0:  # the plan must split, or this case would not touch the built-in buffer
            assert _plan(lib, batch, 1, hq, hkv, d, cap)[0] > 1
        ref_out, ref_lse = _launch(case, t, splits, chunk, noalloc=False)
        out, lse = _launch(case, t, splits, chunk, noalloc=True)
        assert torch.equal(out, ref_out), f"noalloc seed {seed}: output differs from the workspace entry"
        assert torch.equal(lse, ref_lse), f"noalloc seed {seed}: LSE differs from the workspace entry"
        o_ref, lse_ref, _, _, _ = oracle_paged(case)
        assert_close_out(host(out), o_ref, dt, f"noalloc seed {seed} vs oracle")
        assert_close_lse(host(lse), lse_ref, f"noalloc seed {seed} vs oracle")
    assert _lib.read_error_flags() == 0


def test_noalloc_entry_refuses_requests_beyond_its_buffer(cuda_device):
    lib = _lib.load()
    limit = _scratch_limit()
    rows, d = 64 * 32, 128
    splits = limit // (rows * (d + 2) * 4) + 1  # one split more than fits
    assert lib.mxfa_split_workspace_bytes(rows, d, splits) > limit
    dummy = ctypes.c_void_p(16)  # never dereferenced: the size check refuses before any launch
    rc = lib.mxfa_kvcache_attention_noalloc_launch(dummy, dummy, dummy, dummy, dummy, dummy, None, 64, 1, 32, 8, d,
                                                   16, 4096, 100000, 0, splits, 16, 0, 1, 0.1, None)
    assert rc == _lib.MXFA_ERR_UNSUPPORTED
    assert "built-in buffer" in _lib.last_error()
    # a bad argument is reported as itself, not as a buffer refusal
    rc = lib.mxfa_kvcache_attention_noalloc_launch(dummy, dummy, dummy, dummy, dummy, dummy, None, 64, 1, 32, 8, 96,
                                                   16, 4096, 100000, 0, splits, 16, 0, 1, 0.1, None)
    assert rc == _lib.MXFA_ERR_UNSUPPORTED and "head dim" in _lib.last_error()
