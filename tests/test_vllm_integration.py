"""vLLM hook on the CPU: decoder adapter contract, version pin, plugin fallbacks.

Mirrors the reference's tests/test_decoder_adapter.py, test_vllm_bridge.py,
test_vllm_official_split_fallback.py and test_vllm_compat.py.  The CUDA
backend is replaced by fakes here; the -m gpu tests run the real kernels.
"""

from __future__ import annotations

from dataclasses import dataclass

import pytest
import torch

from mxflashattn_b200.integrations.vllm import decoder_adapter
from mxflashattn_b200.integrations.vllm.compat import classify_vllm
from mxflashattn_b200.integrations.vllm.config import VLLM_TARGET_VERSION, validate_vllm_version
from mxflashattn_b200.integrations.vllm.decoder_adapter import DecoderAdapterBlocked, decode_forward, inspect_layout


@dataclass
class Metadata:
    num_actual_tokens: int
    max_query_len: int
    query_start_loc: torch.Tensor
    max_seq_len: int
    seq_lens: torch.Tensor
    block_table: torch.Tensor
    slot_mapping: torch.Tensor
    use_cascade: bool = False
    scheduler_metadata: torch.Tensor | None = None
    causal: bool = True


def make_case(query_lens=(1, 1)):
    q = torch.randn(sum(query_lens), 4, 64, dtype=torch.float16)
    cache = torch.randn(2, 4, 16, 2, 64, dtype=torch.float16)
    starts = [0]
    for length in query_lens:
        starts.append(starts[-1] + length)
    md = Metadata(num_actual_tokens=sum(query_lens), max_query_len=max(query_lens),
                  query_start_loc=torch.tensor(starts), max_seq_len=17, seq_lens=torch.tensor([17, 16]),
                  block_table=torch.tensor([[0, 1], [2, 3]]), slot_mapping=torch.tensor([0, 1]))
    return q, cache, md


@pytest.fixture
def fake_flash(monkeypatch):
    seen = {}

    def fake(q, key_cache, value_cache, **kwargs):
        seen.update(kwargs, q=q, key_cache=key_cache, value_cache=value_cache)
        return torch.zeros_like(q)

    monkeypatch.setattr(decoder_adapter, "flash_attn_with_kvcache", fake)
    return seen


def test_decode_adapter_calls_the_paged_api_with_vllm_layout(fake_flash):
    q, cache, md = make_case()
    out, layout = decode_forward(q, cache, md, softmax_scale=64 ** -0.5)
    assert out.shape == (2, 4 * 64)
    assert layout.query_lens == (1, 1) and layout.kv_cache_shape == (2, 4, 16, 2, 64)
    assert fake_flash["q"].shape == (2, 1, 4, 64)
    assert fake_flash["key_cache"].shape == (4, 16, 2, 64)
    assert fake_flash["cache_seqlens"].dtype == torch.int32 and fake_flash["block_table"].dtype == torch.int32
    assert fake_flash["softmax_scale"] == 64 ** -0.5


def test_prefill_is_blocked_instead_of_delegated():
    q, cache, md = make_case((2, 1))
    with pytest.raises(DecoderAdapterBlocked, match="single_token_decode"):
        decode_forward(q, cache, md, softmax_scale=64 ** -0.5)


def test_layout_rejects_wrong_cache_rank():
    q, _, md = make_case()
    with pytest.raises(DecoderAdapterBlocked, match="kv_cache_shape"):
        inspect_layout(q, torch.empty(2, 4, 16, 64), md)


def test_cascade_is_blocked(fake_flash):
    q, cache, md = make_case()
    md.use_cascade = True
    with pytest.raises(DecoderAdapterBlocked, match="cascade"):
        decode_forward(q, cache, md, softmax_scale=0.125)


def test_transparent_path_flattens_capture_seq_lens(monkeypatch, fake_flash):
    monkeypatch.setenv("MXFLASHATTN_TRANSPARENT", "1")
    q, cache, md = make_case()
    md.seq_lens = md.seq_lens.reshape(1, -1)
    out, layout = decode_forward(q, cache, md, softmax_scale=64 ** -0.5)
    assert out.shape == (2, 4 * 64) and layout is None
    assert fake_flash["cache_seqlens"].shape == (2,)
    assert fake_flash["block_table"].shape == (2, 2)


def test_graph_path_uses_the_decode_subset(monkeypatch, fake_flash):
    monkeypatch.setenv("MXFLASHATTN_GRAPH_DECODE", "1")
    q, cache, md = make_case()
    md.num_decode_tokens, md.num_decodes = 2, 2
    md.decode_seq_lens = torch.tensor([5, 9])
    md.decode_block_table = torch.tensor([[3, 0], [1, 2]])
    out, _ = decode_forward(q, cache, md, softmax_scale=0.125)
    assert out.shape == (2, 256)
    assert fake_flash["cache_seqlens"].tolist() == [5, 9]
    assert fake_flash["block_table"].tolist() == [[3, 0], [1, 2]]


def test_vllm_target_version_is_pinned():
    validate_vllm_version(VLLM_TARGET_VERSION)
    with pytest.raises(RuntimeError, match="targets vLLM"):
        validate_vllm_version("0.29.0")


def test_vllm_compat_classification():
    assert classify_vllm("0.17.0").supported
    assert classify_vllm("0.30.0").status == "probe_required"
    assert classify_vllm(None).status == "not_installed"
    assert classify_vllm("future-build").status == "unknown"
    assert classify_vllm("0.40.0").status == "unsupported"


@pytest.fixture(scope="module")
def plugin():
    pytest.importorskip("vllm")
    from mxflashattn_b200.integrations.vllm import vllm_plugin

    return vllm_plugin


def test_m1_split_plan_is_the_reference_heuristic(plugin):
    # np doubles until B*HKV*np >= 2048 or np == 64; c_len = ceil(max_len / np)
    assert plugin._m1_split_plan(128, 8, 1280) == (2, 640)
    assert plugin._m1_split_plan(1, 8, 16384) == (64, 256)
    assert plugin._m1_split_plan(16, 8, 1280) == (16, 80)


@pytest.mark.parametrize("head_dim,q_heads,kv_heads", [(256, 16, 4), (128, 24, 8)])
def test_official_kvcache_compat_falls_back_for_unsupported_shapes(monkeypatch, plugin, head_dim, q_heads,
                                                                   kv_heads):
    calls = []
    expected = object()
    args = (torch.empty(1, 1, q_heads, head_dim),)
    kwargs = {"k_cache": torch.empty(1, 16, kv_heads, head_dim), "v_cache": torch.empty(1, 16, kv_heads, head_dim),
              "block_table": torch.zeros(1, 1, dtype=torch.int32), "cache_seqlens": torch.ones(1, dtype=torch.int32)}
    monkeypatch.setenv("MXFA_NATIVE_DECODE", "1")
    monkeypatch.setattr(plugin, "_try_native_decode", lambda *a, **k: None)
    monkeypatch.setattr(plugin, "_official_kvcache", lambda *a, **k: calls.append((a, k)) or expected)
    monkeypatch.setattr(plugin, "flash_attn_with_kvcache",
                        lambda *a, **k: pytest.fail("unsupported shape must not enter the MX API"))
    assert plugin._mx_kvcache_compat(*args, **kwargs) is expected
    assert calls == [(args, kwargs)]


def test_native_decode_declines_cpu_and_float32(monkeypatch, plugin):
    monkeypatch.setenv("MXFA_NATIVE_DECODE", "1")
    q = torch.empty(1, 1, 4, 64)
    kw = {"k_cache": torch.empty(1, 16, 2, 64), "v_cache": torch.empty(1, 16, 2, 64),
          "block_table": torch.zeros(1, 1, dtype=torch.int32), "cache_seqlens": torch.ones(1, dtype=torch.int32)}
    assert plugin._try_native_decode((q,), kw) is None


def test_official_split_retries_vendor_after_invalid_argument(monkeypatch, plugin):
    calls, events = [], []
    expected = object()

    def fake_forward(*args, **kwargs):
        calls.append(1)
        if len(calls) == 1:
            raise RuntimeError("CUDA error: invalid argument")
        return expected

    monkeypatch.setattr(plugin.FlashAttentionImpl, "forward", fake_forward)
    monkeypatch.setattr(plugin, "_record_worker_event", lambda event: events.append(event))
    impl = object.__new__(plugin.MXFlashAttnImpl)
    result = plugin._forward_official_split_with_mx(impl, None, None, None, None, None, None, None, None, None)
    assert result is expected and len(calls) == 2
    assert events == [{"path": "vendor_direct", "operation": "official_split_invalid_argument_fallback",
                       "fallback": "true", "fallback_reason": "official_split_invalid_argument"}]


def test_registration_points_flash_attn_at_the_plugin(plugin, monkeypatch):
    from mxflashattn_b200.integrations.vllm import backend as vbackend

    recorded = {}
    import vllm.v1.attention.backends.registry as registry

    monkeypatch.setattr(registry, "register_backend", lambda enum, class_path: recorded.update(enum=enum,
                                                                                                path=class_path))
    info = vbackend.register_vllm_v1_backend()
    assert info["registered"] == "true"
    assert recorded["path"] == "mxflashattn_b200.integrations.vllm.vllm_plugin.MXFlashAttnBackend"
    assert plugin.MXFlashAttnBackend.get_impl_cls() is plugin.MXFlashAttnImpl


# ------------------------------------------------ end-to-end script helpers

def test_smoke_generate_model_dir_and_prompts(tmp_path):
    import json as _json

    from mxflashattn_b200.integrations.vllm import smoke_generate as sg

    path = sg.write_model_dir("qwen3-4b", tmp_path)
    cfg = _json.loads((path / "config.json").read_text())
    assert cfg["num_attention_heads"] == 32 and cfg["num_key_value_heads"] == 8 and cfg["head_dim"] == 128
    assert cfg["num_hidden_layers"] == 36 and cfg["architectures"] == ["Qwen3ForCausalLM"]
    with pytest.raises(ValueError, match="unknown architecture"):
        sg.write_model_dir("qwen3-1b", tmp_path)
    a = sg.make_prompts(5, 10, 20, seed=3)
    assert a == sg.make_prompts(5, 10, 20, seed=3)
    assert all(10 <= len(p) <= 20 for p in a) and len(a) == 5


def test_smoke_generate_compare_and_event_counts(tmp_path):
    from mxflashattn_b200.integrations.vllm import smoke_generate as sg

    base = {"outputs": [{"token_ids": [1, 2, 3, 4], "logprobs": [-1.0, -2.0, -3.0, -4.0]},
                        {"token_ids": [5, 6], "logprobs": [-0.5, -0.25]}], "decode_tok_per_s": 10.0}
    cand = {"outputs": [{"token_ids": [1, 2, 9, 4], "logprobs": [-1.0, -2.001, -3.5, -4.0]},
                        {"token_ids": [5, 6], "logprobs": [-0.5, -0.25]}], "decode_tok_per_s": 12.0}
    summary = sg.compare_runs(base, cand)
    assert summary["token_agreement"] == 5 / 6
    assert summary["first_divergence_min"] == 2
    assert abs(summary["max_logprob_gap_before_divergence"] - 0.001) < 1e-9
    log = tmp_path / "events.jsonl"
    log.write_text('{"path": "cuda_sm100"}\n{"path": "cuda_sm100"}\n{"path": "vendor_prefill_or_blocked"}\n')
    assert sg.count_events(log) == {"cuda_sm100": 2, "vendor_prefill_or_blocked": 1}
    assert sg.count_events(tmp_path / "missing.jsonl") == {}


def test_length_order_is_computed_once_per_step_metadata(monkeypatch):
    """Every layer of a step gets the metadata object the first layer saw: one order kernel per step."""
    from types import SimpleNamespace

    made = []

    def fake_order(seqlens):
        made.append(seqlens)
        return SimpleNamespace(shape=seqlens.shape, device=seqlens.device)

    monkeypatch.setattr(decoder_adapter, "kvcache_length_order", fake_order)
    seq = SimpleNamespace(is_cuda=True, shape=(2,), device="cuda:0")
    md = SimpleNamespace()
    first = decoder_adapter._step_length_order(md, seq)
    assert decoder_adapter._step_length_order(md, seq) is first and len(made) == 1
    # another batch size on the same object: recomputed
    decoder_adapter._step_length_order(md, SimpleNamespace(is_cuda=True, shape=(3,), device="cuda:0"))
    assert len(made) == 2
    # host tensors: no order
    assert decoder_adapter._step_length_order(SimpleNamespace(), torch.tensor([1, 2])) is None
