"""MXFlashAttn hot path on B200 (sm_100a): FlashAttention-compatible API.

Drop-in for the reference package ``mxflashattn`` on its hot path -- the
split-KV paged decode behind ``flash_attn_with_kvcache`` and the causal
dense / varlen forward behind ``flash_attn_func`` / ``flash_attn_varlen_func``
-- with one CUDA backend (``libmxfa_b200.so``) under the same API, dispatch
record, validation and policy objects.
"""

from .accuracy import ErrorSummary, summarize_error
from .api import flash_attn_func, flash_attn_varlen_func, flash_attn_with_kvcache, kvcache_length_order
from .dispatch import BACKEND_LABEL, BackendUnavailableError, DispatchInfo, get_last_dispatch_info
from .policy import AdaptiveDispatchPolicy, DispatchDecision, DispatchPolicyConfig, WorkloadShape

__all__ = [
    "BACKEND_LABEL",
    "BackendUnavailableError",
    "DispatchInfo",
    "flash_attn_func",
    "flash_attn_varlen_func",
    "flash_attn_with_kvcache",
    "get_last_dispatch_info",
    "kvcache_length_order",
    "AdaptiveDispatchPolicy",
    "DispatchDecision",
    "DispatchPolicyConfig",
    "ErrorSummary",
    "WorkloadShape",
    "summarize_error",
]

__version__ = "0.1.0"
