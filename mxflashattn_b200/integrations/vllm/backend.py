"""vLLM registration, dense bridge and dispatch evidence (integrations/vllm/backend.py:1-158).

``register_vllm_v1_backend`` points vLLM's FLASH_ATTN backend at this
package's plugin class; ``attention_forward`` adapts vLLM's dense
``[tokens, heads, dim]`` tensors to ``flash_attn_func``; ``_record_event``
keeps the reference's per-call JSONL evidence trail
(``MXFLASHATTN_DISPATCH_LOG``, sampled by ``MXFLASHATTN_DISPATCH_SAMPLE``)
so existing tooling that counts ``m1_split_decode`` events still works.
"""

from __future__ import annotations

import json
import os

import torch

from mxflashattn_b200 import flash_attn_func

DISPATCH_EVENTS: list[dict[str, str]] = []
_JSON_CACHE: dict[tuple[tuple[str, str], ...], str] = {}
_SAMPLE_EVERY = int(os.getenv("MXFLASHATTN_DISPATCH_SAMPLE", "0") or 0)
_event_count = 0
PLUGIN_CLASS_PATH = "mxflashattn_b200.integrations.vllm.vllm_plugin.MXFlashAttnBackend"


def get_dispatch_events() -> list[dict[str, str]]:
    return list(DISPATCH_EVENTS)


def clear_dispatch_events(truncate_log: bool = True) -> None:
    """Drop buffered events; ``truncate_log=False`` keeps the on-disk trail."""
    DISPATCH_EVENTS.clear()
    if not truncate_log:
        return
    path = os.getenv("MXFLASHATTN_DISPATCH_LOG")
    if path:
        try:
            open(path, "w", encoding="utf-8").close()
        except OSError:
            pass


def _event_log_path() -> str | None:
    path = os.getenv("MXFLASHATTN_DISPATCH_LOG")
    if not path:
        plugin_log = os.getenv("MXFLASHATTN_PLUGIN_IMPORT_LOG")
        if plugin_log:
            path = plugin_log.removesuffix(".plugin.log") + ".dispatch.jsonl"
    return path


def _record_event(event: dict[str, str]) -> None:
    DISPATCH_EVENTS.append(event)
    path = _event_log_path()
    if not path:
        return
    if _SAMPLE_EVERY > 0:
        global _event_count
        _event_count += 1
        if _event_count % _SAMPLE_EVERY != 1:
            return
    key = tuple(sorted(event.items()))
    rendered = _JSON_CACHE.get(key)
    if rendered is None:
        rendered = _JSON_CACHE[key] = json.dumps(event, sort_keys=True) + "\n"
    try:
        with open(path, "a", encoding="utf-8") as stream:
            stream.write(rendered)
    except OSError:
        pass


def attention_forward(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, *, causal: bool,
                      scale: float) -> torch.Tensor:
    """Dense vLLM [tokens, heads, dim] tensors through ``flash_attn_func``."""
    if query.ndim != 3 or key.ndim != 3 or value.shape != key.shape:
        raise ValueError("vLLM Q/K/V must use [tokens, heads, head_dim] layout")
    out = flash_attn_func(query.unsqueeze(0), key.unsqueeze(0), value.unsqueeze(0), causal=causal,
                          softmax_scale=scale)
    return out.squeeze(0)


def register_vllm_v1_backend() -> dict[str, str]:
    """Point vLLM's FLASH_ATTN backend at the B200 plugin class (importable in spawned workers)."""
    try:
        from vllm.v1.attention.backends.registry import AttentionBackendEnum, register_backend
    except Exception as exc:  # depends on the installed vLLM
        return {"registered": "false", "reason": f"vllm_v1_api_unavailable: {type(exc).__name__}: {exc}"}
    register_backend(AttentionBackendEnum.FLASH_ATTN, class_path=PLUGIN_CLASS_PATH)
    return {
        "registered": "true",
        "backend_name": "MXFLASHATTN_B200",
        "backend_path": PLUGIN_CLASS_PATH,
        "decoder_path": "cuda_sm100",
        "encoder_path": "mxflashattn_b200_public_api",
    }
