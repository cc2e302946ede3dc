"""Record the reference's dispatch-policy decisions on ``policy_grid.py``, made by running it.

Usage (in a container where the reference checkout is present):

    python tests/golden/make_policy_decisions.py [--reference-root PATH]

It imports ``mxflashattn/policy.py`` of the MXFlashAttn checkout, evaluates
``AdaptiveDispatchPolicy(DispatchPolicyConfig(**config)).select(WorkloadShape(...))``
at every grid point and writes ``tests/golden/policy_decisions.json``: the
distinct decisions (backend, reason, eligible, policy_enabled,
thresholds_calibrated), one index into them per grid point in grid order,
and the exception type and message of each invalid shape.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import policy_grid  # noqa: E402


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference-root", default=os.environ.get("MXFA_REFERENCE_ROOT"),
                        help="checkout of the reference project (or set MXFA_REFERENCE_ROOT)")
    parser.add_argument("--out", default=os.path.join(HERE, "policy_decisions.json"))
    args = parser.parse_args()
    if not args.reference_root:
        parser.error("--reference-root (or MXFA_REFERENCE_ROOT) is required")
    sys.path.insert(0, args.reference_root)
    from mxflashattn import policy  # the reference's policy

    table, index = [], []
    for c, phase, b, q, kv, d, g in policy_grid.grid():
        decision = policy.AdaptiveDispatchPolicy(policy.DispatchPolicyConfig(**policy_grid.CONFIGS[c])).select(
            policy.WorkloadShape(phase, b, q, kv, d, g))
        row = [decision.backend, decision.reason, decision.eligible, decision.policy_enabled,
               decision.thresholds_calibrated]
        if row not in table:
            table.append(row)
        index.append(table.index(row))
    invalid = {}
    for name, fields in policy_grid.invalid_shapes().items():
        try:
            policy.WorkloadShape(*fields)
            invalid[name] = ["none", ""]
        except Exception as exc:  # the record is the point
            invalid[name] = [type(exc).__name__, str(exc)]
    with open(args.out, "w") as f:
        json.dump({"decisions": table, "index": "".join(chr(ord("a") + i) for i in index), "invalid": invalid},
                  f, indent=1)
        f.write("\n")
    print(f"wrote {args.out}: {len(index)} grid points, {len(table)} distinct decisions")


if __name__ == "__main__":
    main()
