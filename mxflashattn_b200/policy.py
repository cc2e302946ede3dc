"""Tensor-free candidate dispatch policy (mxflashattn/policy.py:1-111).

Kept with the reference's semantics: disabled by default, refuses to pick a
candidate until its thresholds are marked calibrated, and then selects the
prefill or split-KV decode candidate by shape.  It reads no tensors and
queries no device.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Literal

Phase = Literal["prefill", "decode"]
Backend = Literal["vendor", "m1_prefill_chunked", "m1_split_kv"]

_DECODE_GQA = (2, 4, 8)
_DECODE_HEAD_DIMS = (64, 128)


@dataclass(frozen=True)
class WorkloadShape:
    """Shape metadata of one attention call (no tensors, no device queries)."""

    phase: Phase
    batch_size: int
    query_len: int
    kv_len: int
    head_dim: int
    gqa_ratio: int

    def __post_init__(self) -> None:
        if self.phase not in ("prefill", "decode"):
            raise ValueError("phase must be 'prefill' or 'decode'")
        if min(self.batch_size, self.query_len, self.kv_len) <= 0:
            raise ValueError("batch_size, query_len, and kv_len must be positive")
        if min(self.head_dim, self.gqa_ratio) <= 0:
            raise ValueError("head_dim and gqa_ratio must be positive")


@dataclass(frozen=True)
class DispatchPolicyConfig:
    """Candidate thresholds; disabled and uncalibrated unless set explicitly."""

    enabled: bool = False
    calibrated: bool = False
    prefill_batch_min: int = 4
    prefill_kv_len_min: int = 512
    decode_batch_min: int = 16
    decode_kv_len_min: int = 256


@dataclass(frozen=True)
class DispatchDecision:
    backend: Backend
    reason: str
    eligible: bool
    policy_enabled: bool
    thresholds_calibrated: bool


class AdaptiveDispatchPolicy:
    """Safe candidate policy; the default configuration always answers 'vendor'."""

    def __init__(self, config: DispatchPolicyConfig | None = None) -> None:
        self.config = config or DispatchPolicyConfig()

    def _decision(self, backend: Backend, reason: str, eligible: bool) -> DispatchDecision:
        return DispatchDecision(backend=backend, reason=reason, eligible=eligible,
                                policy_enabled=self.config.enabled,
                                thresholds_calibrated=self.config.calibrated)

    def select(self, shape: WorkloadShape) -> DispatchDecision:
        cfg = self.config
        if not cfg.enabled:
            return self._decision("vendor", "policy_disabled", False)
        if not cfg.calibrated:
            return self._decision("vendor", "thresholds_not_calibrated", False)
        if shape.phase == "prefill":
            ok = shape.batch_size >= cfg.prefill_batch_min and shape.kv_len >= cfg.prefill_kv_len_min
            return self._decision("m1_prefill_chunked" if ok else "vendor",
                                  "prefill_threshold_match" if ok else "prefill_below_threshold", ok)
        ok = (shape.batch_size >= cfg.decode_batch_min and shape.kv_len >= cfg.decode_kv_len_min
              and shape.gqa_ratio in _DECODE_GQA and shape.head_dim in _DECODE_HEAD_DIMS)
        return self._decision("m1_split_kv" if ok else "vendor",
                              "decode_threshold_match" if ok else "decode_shape_or_threshold_miss", ok)
