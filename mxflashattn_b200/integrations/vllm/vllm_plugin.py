"""vLLM v1 attention backend classes routing decode to the B200 kernels.

Mirrors the reference hook (integrations/vllm/vllm_plugin.py:199-511):

* ``MXFlashAttnImpl.forward`` sends one-token decode batches through
  ``decode_forward`` (paged ``flash_attn_with_kvcache`` on the CUDA
  backend) and everything else (prefill, mixed batches) back to vLLM's own
  FlashAttention implementation; it records a dispatch event per call.
* ``MXFLASHATTN_GRAPH_OFFICIAL_SPLIT=1`` keeps vLLM's forward and swaps the
  kernel functions it calls (``_mx_kvcache_compat`` / ``_mx_varlen_compat``)
  for the duration of the call, retrying once with the untouched functions
  if the swapped call fails with "invalid argument".
* ``_try_native_decode`` is the fast path behind ``MXFA_NATIVE_DECODE=1``:
  with ``MXFA_M1_DECODE=1`` it calls ``mxflashattn_b200.m1.paged_decode_split``
  (the drop-in for the reference's ``mxmmain.paged_decode_split``) with the
  reference's NP / c_len heuristic, otherwise the B200 split plan; it returns
  None whenever the call falls outside the supported contract.

The classes live at module scope because vLLM resolves the backend by import
path inside spawned workers.
"""

from __future__ import annotations

import json
import os

from vllm.v1.attention.backend import AttentionType
from vllm.v1.attention.backends.flash_attn import FlashAttentionBackend, FlashAttentionImpl

from mxflashattn_b200 import flash_attn_func, flash_attn_varlen_func, flash_attn_with_kvcache
from mxflashattn_b200.dispatch import BACKEND_LABEL, get_last_dispatch_info
from mxflashattn_b200.integrations.vllm.backend import _record_event
from mxflashattn_b200.integrations.vllm.decoder_adapter import DecoderAdapterBlocked, decode_forward

_worker_event_count = 0
_plugin_log = os.getenv("MXFLASHATTN_PLUGIN_IMPORT_LOG")
_shadow_calls = 0


def _record_worker_event(event: dict) -> None:
    """Worker-side JSONL evidence (sampled by MXFLASHATTN_DISPATCH_SAMPLE)."""
    global _worker_event_count
    _worker_event_count += 1
    sample = int(os.getenv("MXFLASHATTN_DISPATCH_SAMPLE", "0") or 0)
    if sample > 1 and _worker_event_count % sample != 1:
        return
    path = os.getenv("MXFLASHATTN_DISPATCH_LOG")
    if not path and _plugin_log:
        path = _plugin_log.removesuffix(".plugin.log") + ".dispatch.jsonl"
    if not path:
        return
    try:
        with open(path, "a", encoding="utf-8") as stream:
            stream.write(json.dumps(event, sort_keys=True) + "\n")
    except OSError:
        pass


if _plugin_log:
    with open(_plugin_log, "a", encoding="utf-8") as _s:
        _s.write(f"plugin_imported pid={os.getpid()} impl_module={FlashAttentionImpl.__module__}\n")

_official_varlen = None
_official_kvcache = None


def _mx_varlen_compat(*args, **kwargs):
    """vLLM's varlen call during the official split: paged calls stay with vLLM."""
    if "block_table" in kwargs:  # the public varlen API has no paged block table
        return _official_varlen(*args, **kwargs)
    out = kwargs.pop("out", None)
    seqused_k = kwargs.pop("seqused_k", None)
    if seqused_k is not None and "cu_seqlens_k" not in kwargs:
        import torch

        lengths = seqused_k.to(dtype=torch.int32)
        kwargs["cu_seqlens_k"] = torch.cat((torch.zeros(1, dtype=torch.int32, device=lengths.device),
                                            lengths.cumsum(0).to(torch.int32)))
    for unused in ("s_aux", "return_attn_probs", "scheduler_metadata", "fa_version", "q_descale", "k_descale",
                   "v_descale", "num_splits"):
        kwargs.pop(unused, None)
    result = flash_attn_varlen_func(*args, **kwargs)
    if isinstance(result, tuple):
        result = result[0]
    if out is not None:
        out.copy_(result)
        return out
    return result


def _m1_split_plan(batch: int, kv_heads: int, max_len: int) -> tuple[int, int]:
    """The reference hook's NP / c_len heuristic (vllm_plugin.py:271-276)."""
    np_ = 1
    base = batch * kv_heads
    while np_ < 64 and base * np_ < 2048:
        np_ *= 2
    return np_, (max_len + np_ - 1) // np_


def _try_native_decode(args, kwargs):
    """Single-token paged decode straight to the B200 kernels, or None if out of contract."""
    if os.getenv("MXFA_NATIVE_DECODE", "0") != "1":
        return None
    import torch

    try:
        q = args[0] if args else kwargs.get("q")
        if q is None or q.dim() not in (3, 4):
            return None
        bt = kwargs.get("block_table")
        sl = kwargs.get("cache_seqlens")
        if bt is None or sl is None or sl.shape[0] != q.shape[0]:
            return None
        if kwargs.get("alibi_slopes") is not None:
            return None
        ws = kwargs.get("window_size")
        if ws is not None:
            vals = ws if isinstance(ws, (tuple, list)) else (ws,)
            if any(int(v) > 0 for v in vals):
                return None
        k_cache = kwargs.get("k_cache", args[1] if len(args) > 1 else None)
        v_cache = kwargs.get("v_cache", args[2] if len(args) > 2 else None)
        if k_cache is None or v_cache is None:
            return None
        if q.dtype not in (torch.float16, torch.bfloat16) or k_cache.dtype != q.dtype:
            return None
        B, HQ, D = q.shape[0], q.shape[-2], q.shape[-1]
        if q.dim() == 4 and q.shape[-3] != 1:
            return None
        scale = kwargs.get("softmax_scale") or D ** -0.5
        q4 = q.reshape(B, 1, HQ, D)
        if not q4.is_contiguous():
            q4 = q4.contiguous()
        bt32, sl32 = bt.to(torch.int32), sl.to(torch.int32)
        if os.getenv("MXFA_M1_DECODE", "0") == "1":
            from mxflashattn_b200 import m1

            np_, c_len = _m1_split_plan(B, int(k_cache.shape[2]), int(bt.shape[1]) * int(k_cache.shape[1]))
            out = m1.paged_decode_split(q4, k_cache, v_cache, bt32.contiguous(), sl32.contiguous(), scale,
                                        torch.cuda.current_stream().cuda_stream, np_, c_len)
            event = {"path": "m1_split_decode", "operation": "paged_decode_split", "fallback": "false", "np": np_}
        else:
            from mxflashattn_b200 import backend

            out = backend.kvcache_attention(q4, k_cache, v_cache, sl32, bt32, scale, False)
            event = {"path": "native_decode", "operation": "paged_decode", "fallback": "false"}
        provided = kwargs.get("out")
        if provided is not None:
            provided.copy_(out.reshape_as(provided))
            result = provided
        else:
            result = out.reshape(q.shape)
        _record_worker_event(event)
        return result
    except Exception as exc:  # the native path must never take the model down
        _record_worker_event({"path": "native_decode", "fallback": "true", "fallback_reason": repr(exc)})
        return None


def _mx_kvcache_compat(*args, **kwargs):
    """vLLM's kvcache call during the official split: native decode, else the original function."""
    for unused in ("s_aux", "return_softmax_lse", "scheduler_metadata", "fa_version", "q_descale", "k_descale",
                   "v_descale"):
        kwargs.pop(unused, None)
    native = _try_native_decode(args, kwargs)
    if native is not None:
        return native
    if _official_kvcache is not None:  # unsupported shapes return to the original implementation
        return _official_kvcache(*args, **kwargs)
    return flash_attn_with_kvcache(*args, **kwargs)


def _forward_official_split_with_mx(self, layer, query, key, value, kv_cache, metadata, output, output_scale,
                                    output_block_scale):
    """vLLM's own forward with its kernel functions swapped for this call (retry once on invalid argument)."""
    global _official_varlen, _official_kvcache
    glb = FlashAttentionImpl.forward.__globals__
    old_var = glb.get("flash_attn_varlen_func")
    old_kv = glb.get("flash_attn_with_kvcache")
    _official_varlen, _official_kvcache = old_var, old_kv
    glb["flash_attn_varlen_func"] = _mx_varlen_compat
    glb["flash_attn_with_kvcache"] = _mx_kvcache_compat
    event = {"path": "vendor_direct", "operation": "official_split_mx", "fallback": "false"}
    try:
        try:
            result = super(MXFlashAttnImpl, self).forward(layer, query, key, value, kv_cache, metadata, output,
                                                           output_scale, output_block_scale)
        except Exception as exc:
            if "invalid argument" not in str(exc).lower():
                raise
            glb["flash_attn_varlen_func"] = old_var
            glb["flash_attn_with_kvcache"] = old_kv
            result = super(MXFlashAttnImpl, self).forward(layer, query, key, value, kv_cache, metadata, output,
                                                           output_scale, output_block_scale)
            event = {"path": "vendor_direct", "operation": "official_split_invalid_argument_fallback",
                     "fallback": "true", "fallback_reason": "official_split_invalid_argument"}
    finally:
        glb["flash_attn_varlen_func"] = old_var
        glb["flash_attn_with_kvcache"] = old_kv
        _official_varlen = None
        _official_kvcache = None
    _record_worker_event(event)
    return result


class MXFlashAttnImpl(FlashAttentionImpl):
    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output=None, output_scale=None,
                output_block_scale=None):
        if attn_metadata is None:  # profiling run
            if output is None:
                raise ValueError("vLLM must provide an output buffer for profiling")
            return output.fill_(0)
        if os.getenv("MXFLASHATTN_SPLIT_PURE", "0") == "1":
            return super().forward(layer, query, key, value, kv_cache, attn_metadata, output, output_scale,
                                   output_block_scale)
        if os.getenv("MXFLASHATTN_GRAPH_OFFICIAL_SPLIT", "0") == "1":
            return _forward_official_split_with_mx(self, layer, query, key, value, kv_cache, attn_metadata,
                                                   output, output_scale, output_block_scale)
        if self.attn_type in (AttentionType.ENCODER_ONLY, AttentionType.ENCODER):
            if output is None:
                raise ValueError("vLLM must provide an output buffer")
            n = attn_metadata.num_actual_tokens
            result = flash_attn_func(query[:n].unsqueeze(0), key[:n].unsqueeze(0), value[:n].unsqueeze(0),
                                     causal=False, softmax_scale=self.scale).reshape(-1, self.num_heads * self.head_size)
            _record_event({"path": "mxflashattn_encoder", "operation": "flash_attn_func", "fallback": "false"})
            output[: result.shape[0]].copy_(result)
            return output
        try:
            result, _ = decode_forward(query, kv_cache, attn_metadata, softmax_scale=self.scale,
                                       causal=bool(attn_metadata.causal))
        except DecoderAdapterBlocked as exc:
            event = {"path": "vendor_prefill_or_blocked", "reason": str(exc)}
            _record_event(event)
            _record_worker_event(event)
            if "single_token_decode" in str(exc):
                return super().forward(layer, query, key, value, kv_cache, attn_metadata, output, output_scale,
                                       output_block_scale)
            raise
        info = get_last_dispatch_info()
        if info is None:
            raise RuntimeError("MXFlashAttn decoder returned without dispatch evidence")
        if info.backend == BACKEND_LABEL:
            event = {"path": BACKEND_LABEL, "operation": info.operation, "fallback": "false"}
        else:
            event = {"path": info.backend, "operation": info.operation, "fallback": "true",
                     "fallback_reason": info.fallback_reason or "unspecified"}
        _record_event(event)
        _record_worker_event(event)
        if output is None:
            raise ValueError("vLLM must provide an output buffer")
        _shadow_check(self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale,
                      output_block_scale, result)
        target = output[: result.shape[0]]
        if target.numel() != result.numel():
            raise RuntimeError(f"MXFlashAttn decoder output size mismatch: target={tuple(target.shape)} "
                               f"result={tuple(result.shape)}")
        target.copy_(result.reshape_as(target))
        return output


def _shadow_check(impl, layer, query, key, value, kv_cache, attn_metadata, output, output_scale,
                  output_block_scale, result) -> None:
    """Every MXFLASHATTN_SHADOW_CHECK_EVERY-th decode call, also run vLLM's own
    attention on the same live inputs and record the largest difference.

    A debug aid for end-to-end parity (no reference counterpart): it syncs the
    device and doubles the checked call's attention cost, so it is off unless
    the variable is set.  Re-running vLLM's forward re-writes the same cache
    rows, which leaves the cache unchanged.
    """
    global _shadow_calls
    every = int(os.getenv("MXFLASHATTN_SHADOW_CHECK_EVERY", "0") or 0)
    if every <= 0:
        return
    _shadow_calls += 1
    if _shadow_calls % every != 1 and every != 1:
        return
    import torch

    ref = torch.zeros_like(output)
    FlashAttentionImpl.forward(impl, layer, query, key, value, kv_cache, attn_metadata, ref, output_scale,
                               output_block_scale)
    n = result.shape[0]
    mine = result.reshape(n, -1).float()
    theirs = ref[:n].reshape(n, -1).float()
    event = {
        "path": "shadow_check",
        "tokens": int(n),
        "max_abs_diff": float((mine - theirs).abs().max()),
        "max_abs_ref": float(theirs.abs().max()),
    }
    exact = _fp32_decode_reference(query, kv_cache, attn_metadata, impl.scale, n)
    if exact is not None:
        # scale-free: the call's largest error in units of one bf16 ulp of the
        # call's largest exact output (per-element ulps blow up where a row's
        # weighted sum nearly cancels, for any kernel that rounds P)
        event["max_ulps_kernel_vs_fp32"] = _max_ulps(mine, exact)
        event["max_ulps_vllm_vs_fp32"] = _max_ulps(theirs, exact)
        event["max_abs_fp32"] = float(exact.abs().max())
    _record_worker_event(event)


def _fp32_decode_reference(query, kv_cache, attn_metadata, scale, n):
    """fp32 attention of the n live decode queries over their cached keys
    (gathered through the block table), the math of mxflashattn/reference.py
    in torch: softmax(q k^T * scale) v per sequence, GQA heads sharing a KV
    head.  None when the metadata is not one query token per sequence."""
    import torch

    seq_lens = attn_metadata.seq_lens.reshape(-1)
    if seq_lens.numel() != n or int(getattr(attn_metadata, "max_query_len", 1)) != 1:
        return None
    key_cache, value_cache = kv_cache.unbind(0)
    page, hkv, d = key_cache.shape[1], key_cache.shape[2], key_cache.shape[3]
    hq = query.shape[1]
    out = torch.empty((n, hq, d), device=query.device, dtype=torch.float32)
    lens = seq_lens.tolist()
    table = attn_metadata.block_table
    for b, length in enumerate(lens):
        pages = table[b, : (int(length) + page - 1) // page].long()
        k = key_cache[pages].reshape(-1, hkv, d)[: int(length)].float()
        v = value_cache[pages].reshape(-1, hkv, d)[: int(length)].float()
        q = query[b].float().reshape(hkv, hq // hkv, d)
        s = torch.einsum("hgd,thd->hgt", q, k) * scale
        out[b] = torch.einsum("hgt,thd->hgd", torch.softmax(s, dim=-1), v).reshape(hq, d)
    return out.reshape(n, -1)


def _max_ulps(actual, exact) -> float:
    """max |actual - exact| / ulp_bf16(max |exact|): the error in bf16 ulps of the largest output."""
    import math

    top = float(exact.abs().max())
    if top <= 0.0:
        return 0.0
    ulp = 2.0 ** (math.floor(math.log2(top)) - 7)
    return float((actual - exact).abs().max()) / ulp


class MXFlashAttnBackend(FlashAttentionBackend):
    @staticmethod
    def get_name() -> str:
        # vLLM layers index the backend enum by this name; the registry path points here
        return "FLASH_ATTN"

    @staticmethod
    def get_impl_cls():
        return MXFlashAttnImpl
