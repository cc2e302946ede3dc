"""Drop-in for the reference's M1 split-decode module (``mxmmain``).

``paged_decode_split`` keeps the signature, checks and error behaviour of
the pybind function it replaces (csrc_native/m1_binding.cpp:78-115): it
allocates ``out`` and the fp32 split workspaces, launches the split-KV
decode plus combine on the given stream through
``mxfa_paged_decode_split_launch`` and raises ``RuntimeError`` on a
non-zero status.  ``split_plan`` is the vLLM hook's NP / c_len heuristic
(integrations/vllm/vllm_plugin.py:271-276) re-derived for B200's SM count.
"""

from __future__ import annotations

import os
import re

import torch

from . import _lib


def softmax_variant_from_env() -> int:
    """``um`` as the reference binding reads it per call (m1_binding.cpp:100-105): 2 unless ``MXFA_M1_UM``
    parses, the way C ``atoi`` does (leading blanks, sign, digits; 0 when there are none), to 0 or 1."""
    env = os.getenv("MXFA_M1_UM")
    if env is None:
        return 2
    m = re.match(r"[ \t\n\v\f\r]*([+-]?\d+)", env)
    val = int(m.group(1)) if m else 0
    return val if val in (0, 1) else 2


def paged_decode_split(q, k, v, bt, sl, scale, stream, np, c_len):
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise RuntimeError("tensors must be on device")
    # Stricter than the reference binding, which checks q/k/v only: a block
    # table, lengths or cache on another device would reach the kernel as a
    # foreign pointer, so they are rejected with the same message instead.
    if any(t.device != q.device for t in (k, v, bt, sl)):
        raise RuntimeError("tensors must be on device")
    ok = (q.dtype in (torch.float16, torch.bfloat16) and q.dtype == k.dtype == v.dtype and q.is_contiguous()
          and k.is_contiguous() and v.is_contiguous() and bt.is_contiguous() and sl.is_contiguous()
          and sl.dtype == torch.int32 and bt.dtype == torch.int32)
    if not ok:
        raise RuntimeError("dtype/layout check failed")
    if q.dim() != 4 or q.shape[1] != 1:
        raise RuntimeError("q must be [B, 1, HQ, D]")
    B, _, HQ, D = q.shape
    HKV, PS = k.shape[2], k.shape[1]
    BTW = bt.shape[1]
    ows = torch.empty((B, HQ, np, D), device=q.device, dtype=torch.float32)
    mdws = torch.empty((B, HQ, np, 2), device=q.device, dtype=torch.float32)
    out = torch.empty((B, 1, HQ, D), device=q.device, dtype=q.dtype)
    um = softmax_variant_from_env()
    with torch.cuda.device(q.device):
        rc = _lib.load().mxfa_paged_decode_split_launch(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), bt.data_ptr(), sl.data_ptr(), out.data_ptr(), ows.data_ptr(),
            mdws.data_ptr(), float(scale), B, HQ, HKV, D, PS, BTW, int(q.dtype == torch.bfloat16), int(np),
            int(c_len), um, int(stream) if stream else None)
    if rc != 0:
        raise RuntimeError(f"split kernel unsupported config: D={D} GQ={HQ // max(HKV, 1)} "
                           f"({_lib.last_error()})")
    return out


def split_plan(batch: int, kv_heads: int, max_len: int, q_heads: int | None = None, head_dim: int = 128):
    """(np, c_len) for a decode batch, sized to this GPU by the library's planner."""
    from .backend import kvcache_plan

    return kvcache_plan(batch, 1, q_heads or kv_heads, kv_heads, head_dim, max_len)
