"""vLLM hook on the GPU: the decoder adapter and the native decode fast path vs the oracle."""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import pytest

from helpers import assert_close_out, host, oracle_paged
from mxflashattn_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


@dataclass
class Metadata:
    num_actual_tokens: int
    max_query_len: int
    query_start_loc: object
    max_seq_len: int
    seq_lens: object
    block_table: object
    slot_mapping: object
    use_cascade: bool = False
    scheduler_metadata: object = None
    causal: bool = True


def _vllm_case(device, dtype="bf16"):
    import torch

    case = syn.paged_case(2024, batch=5, q_heads=32, kv_heads=8, head_dim=128, dtype=dtype, page_size=16,
                          lengths=[1, 17, 300, 1024, 64])
    tdt = syn.torch_dtype(dtype)
    kv = torch.stack([torch.from_numpy(case.k_cache), torch.from_numpy(case.v_cache)]).to(device, tdt)
    query = torch.from_numpy(case.q[:, 0]).to(device, tdt)  # [tokens, heads, dim]
    md = Metadata(num_actual_tokens=5, max_query_len=1, query_start_loc=torch.arange(6, device=device),
                  max_seq_len=1024, seq_lens=torch.from_numpy(case.cache_seqlens).to(device),
                  block_table=torch.from_numpy(case.block_table).to(device),
                  slot_mapping=torch.zeros(5, dtype=torch.int64, device=device))
    return case, kv, query, md


@pytest.mark.parametrize("strict", [False, True])
def test_decode_forward_matches_oracle(strict, monkeypatch, cuda_device):
    from mxflashattn_b200.integrations.vllm import decoder_adapter

    monkeypatch.setattr(decoder_adapter, "STRICT_LAYOUT", strict)
    case, kv, query, md = _vllm_case(cuda_device)
    out, layout = decoder_adapter.decode_forward(query, kv, md, softmax_scale=case.softmax_scale)
    assert out.shape == (5, 32 * 128)
    ref = oracle_paged(case)[0].reshape(5, -1)
    assert_close_out(host(out), ref, "bf16", "decode_forward")
    if strict:
        assert layout.seq_lens == tuple(int(x) for x in case.cache_seqlens)


@pytest.mark.parametrize("m1", ["0", "1"])
def test_native_decode_fast_path_matches_oracle(m1, monkeypatch, cuda_device):
    pytest.importorskip("vllm")
    import torch

    from mxflashattn_b200.integrations.vllm import vllm_plugin

    monkeypatch.setenv("MXFA_NATIVE_DECODE", "1")
    monkeypatch.setenv("MXFA_M1_DECODE", m1)
    events = []
    monkeypatch.setattr(vllm_plugin, "_record_worker_event", lambda e: events.append(e))
    case, kv, query, md = _vllm_case(cuda_device, "fp16")
    out = torch.empty_like(query)
    result = vllm_plugin._mx_kvcache_compat(query.unsqueeze(1), k_cache=kv[0], v_cache=kv[1],
                                            block_table=md.block_table, cache_seqlens=md.seq_lens,
                                            softmax_scale=case.softmax_scale, out=out)
    assert result is out
    assert events and events[0]["path"] == ("m1_split_decode" if m1 == "1" else "native_decode")
    ref = oracle_paged(case)[0][:, 0]
    assert_close_out(host(out), ref, "fp16", f"native decode m1={m1}")
