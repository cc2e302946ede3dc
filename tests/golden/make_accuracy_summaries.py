"""Record the reference's ``summarize_error`` reports on seeded inputs, made by running it.

Usage (in a container where the reference checkout is present):

    python tests/golden/make_accuracy_summaries.py [--reference-root PATH]

It imports ``mxflashattn/accuracy.py`` of the MXFlashAttn checkout and writes
``tests/golden/accuracy_summaries.json``: for each case of ``CASES`` (built by
``build``, shared with the test) the report's ``as_dict()``, or the exception
type and message.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def build(name: str):
    """(actual, expected) of one case; seeded CPU tensors."""
    g = torch.Generator().manual_seed(sum(map(ord, name)))
    expected = torch.randn(4, 33, 8, generator=g)
    noise = torch.randn(4, 33, 8, generator=g) * 1e-3
    if name == "bf16_rounding":
        return expected.bfloat16(), expected
    if name == "small_noise":
        return expected + noise, expected
    if name == "zeros_expected":
        return noise, torch.zeros_like(noise)
    if name == "one_nan":
        actual = expected + noise
        actual[1, 2, 3] = float("nan")
        return actual, expected
    if name == "one_inf":
        actual = expected + noise
        actual[0, 0, 0] = float("inf")
        return actual, expected
    if name == "fp16_pair":
        return (expected + noise).half(), expected.half()
    if name == "shape_mismatch":
        return expected, expected[:3]
    if name == "empty":
        return expected[:0], expected[:0]
    if name == "not_a_tensor":
        return expected.tolist(), expected
    raise KeyError(name)


CASES = ("bf16_rounding", "small_noise", "zeros_expected", "one_nan", "one_inf", "fp16_pair", "shape_mismatch",
         "empty", "not_a_tensor")


def report(summarize, name):
    actual, expected = build(name)
    try:
        out = summarize(actual, expected).as_dict()
    except Exception as exc:  # the record is the point
        return {"error": [type(exc).__name__, str(exc)]}
    return {k: (repr(v) if isinstance(v, float) and not math.isfinite(v) else v) for k, v in out.items()}


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference-root", default=os.environ.get("MXFA_REFERENCE_ROOT"),
                        help="checkout of the reference project (or set MXFA_REFERENCE_ROOT)")
    parser.add_argument("--out", default=os.path.join(HERE, "accuracy_summaries.json"))
    args = parser.parse_args()
    if not args.reference_root:
        parser.error("--reference-root (or MXFA_REFERENCE_ROOT) is required")
    sys.path.insert(0, args.reference_root)
    from mxflashattn.accuracy import summarize_error  # the reference's report

    with open(args.out, "w") as f:
        json.dump({name: report(summarize_error, name) for name in CASES}, f, indent=1)
        f.write("\n")
    print(f"wrote {args.out}")


if __name__ == "__main__":
    main()
