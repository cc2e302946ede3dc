"""Policy and accuracy objects keep the reference's behaviour (tests/test_policy.py, test_accuracy.py)."""

from __future__ import annotations

import pytest
import torch

from mxflashattn_b200.accuracy import summarize_error
from mxflashattn_b200.policy import AdaptiveDispatchPolicy, DispatchPolicyConfig, WorkloadShape


def shape(**overrides):
    values = {"phase": "prefill", "batch_size": 8, "query_len": 512, "kv_len": 1024, "head_dim": 128, "gqa_ratio": 4}
    values.update(overrides)
    return WorkloadShape(**values)


def test_policy_is_safe_by_default():
    d = AdaptiveDispatchPolicy().select(shape())
    assert (d.backend, d.reason, d.eligible) == ("vendor", "policy_disabled", False)


def test_enabled_policy_waits_for_calibration():
    d = AdaptiveDispatchPolicy(DispatchPolicyConfig(enabled=True)).select(shape())
    assert (d.backend, d.reason, d.thresholds_calibrated) == ("vendor", "thresholds_not_calibrated", False)


def test_calibrated_prefill_and_decode_candidates():
    p = AdaptiveDispatchPolicy(DispatchPolicyConfig(enabled=True, calibrated=True))
    assert p.select(shape()).backend == "m1_prefill_chunked"
    assert p.select(shape(batch_size=1)).backend == "vendor"
    assert p.select(shape(kv_len=128)).backend == "vendor"
    assert p.select(shape(phase="decode", batch_size=32, query_len=1, kv_len=1024)).backend == "m1_split_kv"
    assert p.select(shape(phase="decode", gqa_ratio=7)).backend == "vendor"
    assert p.select(shape(phase="decode", head_dim=256)).backend == "vendor"


@pytest.mark.parametrize("kwargs", [{"phase": "other"}, {"batch_size": 0}, {"query_len": 0}, {"kv_len": 0},
                                    {"head_dim": 0}, {"gqa_ratio": -1}])
def test_workload_shape_rejects_invalid_metadata(kwargs):
    with pytest.raises(ValueError):
        shape(**kwargs)


def test_error_summary_statistics():
    s = summarize_error(torch.tensor([1.0, 2.1, 3.5, 10.0]), torch.tensor([1.0, 2.0, 4.0, 8.0]))
    assert s.sample_count == 4 and s.finite
    assert s.max_abs == pytest.approx(2.0)
    assert s.mean_abs == pytest.approx(0.65)
    assert s.p99_abs >= s.p95_abs >= s.mean_abs
    assert s.max_relative == pytest.approx(0.25)
    assert s.as_dict()["max_abs"] == s.max_abs


def test_error_summary_nonfinite_and_invalid():
    s = summarize_error(torch.tensor([float("nan")]), torch.tensor([1.0]))
    assert not s.finite and s.max_abs == float("inf")
    with pytest.raises(ValueError, match="empty"):
        summarize_error(torch.empty(0), torch.empty(0))
    with pytest.raises(ValueError, match="identical shapes"):
        summarize_error(torch.zeros(2), torch.zeros(3))


def _recorded_policy():
    import json
    import os

    with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "policy_decisions.json")) as f:
        return json.load(f)


def test_policy_decisions_on_the_threshold_grid_are_the_references():
    """Every grid point straddling the thresholds (tests/golden/policy_grid.py) gets the decision the reference's
    policy made there (tests/golden/policy_decisions.json, recorded by running it)."""
    import policy_grid

    recorded = _recorded_policy()
    table = [tuple(row) for row in recorded["decisions"]]
    points = list(policy_grid.grid())
    assert len(points) == len(recorded["index"])
    mismatches = []
    for (c, phase, b, q, kv, d, g), code in zip(points, recorded["index"]):
        dec = AdaptiveDispatchPolicy(DispatchPolicyConfig(**policy_grid.CONFIGS[c])).select(
            WorkloadShape(phase, b, q, kv, d, g))
        got = (dec.backend, dec.reason, dec.eligible, dec.policy_enabled, dec.thresholds_calibrated)
        if got != table[ord(code) - ord("a")]:
            mismatches.append(((c, phase, b, q, kv, d, g), got))
    assert mismatches == []


def test_invalid_workload_shapes_raise_what_the_reference_raises():
    import policy_grid

    for name, fields in policy_grid.invalid_shapes().items():
        with pytest.raises(Exception) as info:
            WorkloadShape(*fields)
        assert [type(info.value).__name__, str(info.value)] == _recorded_policy()["invalid"][name], name


@pytest.mark.parametrize("case", ["bf16_rounding", "small_noise", "zeros_expected", "one_nan", "one_inf", "fp16_pair",
                                  "shape_mismatch", "empty", "not_a_tensor"])
def test_error_reports_are_the_references(case):
    """summarize_error's report, or its exception, on seeded inputs (tests/golden/accuracy_summaries.json,
    recorded by running the reference's summarize_error)."""
    import json
    import os

    import make_accuracy_summaries as gen

    with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "accuracy_summaries.json")) as f:
        expected = json.load(f)[case]
    ours = gen.report(summarize_error, case)
    assert ours.keys() == expected.keys()
    for key, value in expected.items():
        if isinstance(value, float):
            assert ours[key] == pytest.approx(value, rel=1e-6, abs=1e-12), key
        else:
            assert ours[key] == value, key
