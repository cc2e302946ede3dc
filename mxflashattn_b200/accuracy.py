"""Error summary used by parity reports (mxflashattn/accuracy.py:23-51)."""

from __future__ import annotations

from dataclasses import asdict, dataclass
from typing import Any

import torch


@dataclass(frozen=True)
class ErrorSummary:
    sample_count: int
    finite: bool
    max_abs: float
    mean_abs: float
    p95_abs: float
    p99_abs: float
    max_relative: float

    def as_dict(self) -> dict[str, Any]:
        return asdict(self)


def summarize_error(actual: torch.Tensor, expected: torch.Tensor) -> ErrorSummary:
    """Distribution of |actual - expected|; non-finite errors report as +inf, never raise."""
    if not isinstance(actual, torch.Tensor) or not isinstance(expected, torch.Tensor):
        raise TypeError("actual and expected must be torch.Tensor values")
    if actual.shape != expected.shape:
        raise ValueError("actual and expected must have identical shapes")
    if actual.numel() == 0:
        raise ValueError("cannot summarize an empty tensor")
    a = actual.detach().float().reshape(-1)
    e = expected.detach().float().reshape(-1)
    finite = bool(torch.isfinite(a).all() and torch.isfinite(e).all())
    inf = float("inf")
    err = torch.nan_to_num((a - e).abs(), nan=inf, posinf=inf, neginf=inf)
    rel = torch.nan_to_num((a - e).abs() / e.abs().clamp_min(1e-6), nan=inf, posinf=inf, neginf=inf)
    return ErrorSummary(
        sample_count=err.numel(),
        finite=finite,
        max_abs=float(err.max()),
        mean_abs=float(err.mean()),
        p95_abs=float(torch.quantile(err, 0.95)),
        p99_abs=float(torch.quantile(err, 0.99)),
        max_relative=float(rel.max()),
    )
