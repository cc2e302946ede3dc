"""Record the reference's public API signatures, read from the reference itself.

Usage (in a container where the reference checkout is present):

    python tests/golden/make_api_signatures.py [--reference-root PATH]

It imports the MXFlashAttn checkout's package and writes to
``tests/golden/api_signatures.json``, for ``flash_attn_func``,
``flash_attn_varlen_func`` and ``flash_attn_with_kvcache``, each parameter's
name, kind and default (as ``repr``) in order, and, for the records and
policy objects the package exports (``DispatchInfo``, ``ErrorSummary``,
``DispatchPolicyConfig``, ``WorkloadShape``, ``DispatchDecision``), each
field's name and default in order.
"""

from __future__ import annotations

import argparse
import dataclasses
import inspect
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
FUNCTIONS = ("flash_attn_func", "flash_attn_varlen_func", "flash_attn_with_kvcache")
RECORDS = ("DispatchInfo", "ErrorSummary", "DispatchPolicyConfig", "WorkloadShape", "DispatchDecision")


def describe(fn) -> list[list[str]]:
    return [[name, p.kind.name, repr(p.default)] for name, p in inspect.signature(fn).parameters.items()]


def fields(cls) -> list[list[str | None]]:
    return [[f.name, None if f.default is dataclasses.MISSING else repr(f.default)] for f in dataclasses.fields(cls)]


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference-root", default=os.environ.get("MXFA_REFERENCE_ROOT"),
                        help="checkout of the reference project (or set MXFA_REFERENCE_ROOT)")
    parser.add_argument("--out", default=os.path.join(HERE, "api_signatures.json"))
    args = parser.parse_args()
    if not args.reference_root:
        parser.error("--reference-root (or MXFA_REFERENCE_ROOT) is required")
    sys.path.insert(0, args.reference_root)
    import mxflashattn  # the reference's public package
    from mxflashattn import api

    record = {name: describe(getattr(api, name)) for name in FUNCTIONS}
    record["records"] = {name: fields(getattr(mxflashattn, name)) for name in RECORDS}
    with open(args.out, "w") as f:
        json.dump(record, f, indent=1)
        f.write("\n")
    print(f"wrote {args.out}")


if __name__ == "__main__":
    main()
