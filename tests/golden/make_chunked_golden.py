"""Golden vectors of the reference's chunked online-softmax prototype, made by running it.

Usage (in a container where the reference checkout is present):

    python tests/golden/make_chunked_golden.py [--reference-root PATH]

It imports ``mxflashattn/prefill.py`` of the MXFlashAttn checkout and runs
``prefill_chunked_reference`` and ``prefill_chunked_reference_fallback`` with
PyTorch on the CPU over ``cases.chunked_cases()``, writing
``tests/golden/chunked.npz``.  For each case it stores

* ``<name>.out``          -- the prototype's output in the case dtype (as float32),
* ``<name>.out_f32``      -- the prototype on float32 copies of the same inputs,
* ``<name>.fallback_f32`` -- the fallback switch on float32 copies, for the
  cases where one chunk covers every key (it takes the direct oracle there;
  otherwise it runs the prototype itself),
* ``<name>.digest``       -- sha1 of the regenerated inputs.

Only the numbers the reference computes go into the fixture.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, HERE)

import cases as golden_cases  # noqa: E402


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference-root", default=os.environ.get("MXFA_REFERENCE_ROOT"),
                        help="checkout of the reference project (or set MXFA_REFERENCE_ROOT)")
    parser.add_argument("--out", default=os.path.join(HERE, "chunked.npz"))
    args = parser.parse_args()
    if not args.reference_root:
        parser.error("--reference-root (or MXFA_REFERENCE_ROOT) is required")
    sys.path.insert(0, args.reference_root)
    import torch
    from mxflashattn import prefill as ref  # the reference's own prototype

    store: dict[str, np.ndarray] = {}
    for name, case in golden_cases.chunked_cases().items():
        tdt = {"bf16": torch.bfloat16, "fp16": torch.float16}[case.dtype]
        store[f"{name}.digest"] = np.array(golden_cases.digest(case.q, case.k, case.v))
        kw = dict(chunk_size=case.chunk_size, softmax_scale=case.softmax_scale, causal=case.causal)
        runs = [("out", tdt, ref.prefill_chunked_reference),
                ("out_f32", torch.float32, ref.prefill_chunked_reference)]
        if case.chunk_size >= case.k.shape[1]:
            runs.append(("fallback_f32", torch.float32, ref.prefill_chunked_reference_fallback))
        for suffix, dt, fn in runs:
            q, k, v = (torch.from_numpy(a).to(dt) for a in (case.q, case.k, case.v))
            store[f"{name}.{suffix}"] = fn(q, k, v, **kw).float().numpy()
    np.savez_compressed(args.out, **store)
    print(f"wrote {args.out}: {len(store)} arrays")


if __name__ == "__main__":
    main()
