"""Record what the reference's public API raises on the invalid calls of ``api_error_cases.py``.

Usage (in a container where the reference checkout is present):

    python tests/golden/make_api_errors.py [--reference-root PATH]

It imports the reference package, makes each call (strict cases with
``MXFLASHATTN_STRICT_VALIDATION=1``) and writes the exception type name and
message per case to ``tests/golden/api_errors.json``.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import api_error_cases  # noqa: E402


def outcome(fn, args, kwargs):
    try:
        fn(*args, **kwargs)
    except Exception as exc:  # the record is the point
        return [type(exc).__name__, str(exc)]
    return ["none", ""]


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference-root", default=os.environ.get("MXFA_REFERENCE_ROOT"),
                        help="checkout of the reference project (or set MXFA_REFERENCE_ROOT)")
    parser.add_argument("--out", default=os.path.join(HERE, "api_errors.json"))
    args = parser.parse_args()
    if not args.reference_root:
        parser.error("--reference-root (or MXFA_REFERENCE_ROOT) is required")
    sys.path.insert(0, args.reference_root)
    import mxflashattn  # the reference's public API

    os.environ.pop("MXFLASHATTN_ALLOW_FALLBACK", None)
    record = {}
    for name, (fn_name, build, strict) in api_error_cases.cases().items():
        os.environ["MXFLASHATTN_STRICT_VALIDATION"] = "1" if strict else "0"
        call_args, call_kwargs = build()
        record[name] = outcome(getattr(mxflashattn, fn_name), call_args, call_kwargs)
    os.environ.pop("MXFLASHATTN_STRICT_VALIDATION", None)
    with open(args.out, "w") as f:
        json.dump(record, f, indent=1, sort_keys=True)
        f.write("\n")
    print(f"wrote {args.out}: {len(record)} cases")


if __name__ == "__main__":
    main()
