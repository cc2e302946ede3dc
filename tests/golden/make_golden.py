"""Generate golden vectors by running the reference implementation itself.

Usage (in a container where the reference checkout is present):

    python tests/golden/make_golden.py [--reference-root PATH]

It imports the reference's own oracle module (``mxflashattn/reference.py`` of
the MXFlashAttn checkout), runs it with PyTorch on the CPU over the seeded
cases of ``tests/golden/cases.py`` and writes ``tests/golden/golden.npz``.
For each case it stores

* ``<name>.out``      -- the reference output in the case dtype (as float32),
* ``<name>.out_f32``  -- the reference run on float32 copies of the same
  inputs (no final downcast), the tighter anchor for the numpy oracle,
* ``<name>.lse``      -- harness log-sum-exp (the reference returns none; it
  is computed here in float64 from the same scaled scores),
* for appends: sha1 digests of the caches (as float32) and ``cache_seqlens``
  after the call -- the bit-exact append anchor,
* ``<name>.digest``   -- sha1 of the regenerated inputs.

The reference tree is read-only input here; nothing from it is copied into
the fixtures except the numbers it computes.
"""

from __future__ import annotations

import argparse
import math
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, HERE)

import cases as golden_cases  # noqa: E402


def _lse_paged(case, torch):
    """float64 natural-log LSE of the scaled scores, per (b, q-row, head)."""
    q = torch.from_numpy(case.q).double()
    B, Sq, HQ, D = case.q.shape
    HKV = case.k_cache.shape[2]
    G = HQ // HKV
    out = np.zeros((B, Sq, HQ), np.float64)
    kc = case.k_cache.copy()
    lengths = case.cache_seqlens.astype(np.int64)
    app = 0 if case.k_new is None else case.k_new.shape[1]
    for b in range(B):
        total = int(lengths[b]) + app
        if case.block_table is None:
            keys = kc[b, :total].copy()
            if app:
                keys[int(lengths[b]):total] = case.k_new[b]
        else:
            ps = kc.shape[1]
            row = case.block_table[b]
            keys = np.concatenate([kc[row[p]] for p in range((total + ps - 1) // ps)], 0)[:total].copy()
            if app:
                keys[int(lengths[b]):total] = case.k_new[b]
        k = torch.from_numpy(keys).double()                       # [L, HKV, D]
        for h in range(HQ):
            s = (q[b, :, h, :] @ k[:, h // G, :].T) * case.softmax_scale   # [Sq, L]
            if case.causal:
                qpos = torch.arange(Sq) + (total - Sq)
                s = s.masked_fill(torch.arange(total)[None, :] > qpos[:, None], float("-inf"))
            out[b, :, h] = torch.logsumexp(s, dim=-1).numpy()
    return out


def _lse_varlen(case, torch):
    HQ = case.q.shape[1]
    HKV = case.k.shape[1]
    G = HQ // HKV
    out = np.zeros((case.q.shape[0], HQ), np.float64)
    for i in range(len(case.cu_q) - 1):
        qs, qe, ks, ke = (int(case.cu_q[i]), int(case.cu_q[i + 1]), int(case.cu_k[i]), int(case.cu_k[i + 1]))
        q = torch.from_numpy(case.q[qs:qe]).double()
        k = torch.from_numpy(case.k[ks:ke]).double()
        for h in range(HQ):
            s = (q[:, h] @ k[:, h // G].T) * case.softmax_scale
            if case.causal:
                qpos = torch.arange(qe - qs) + ((ke - ks) - (qe - qs))
                s = s.masked_fill(torch.arange(ke - ks)[None, :] > qpos[:, None], float("-inf"))
            out[qs:qe, h] = torch.logsumexp(s, dim=-1).numpy()
    return out


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference-root", default=os.environ.get("MXFA_REFERENCE_ROOT"),
                        help="checkout of the reference project (or set MXFA_REFERENCE_ROOT)")
    parser.add_argument("--out", default=os.path.join(HERE, "golden.npz"))
    args = parser.parse_args()
    if not args.reference_root:
        parser.error("--reference-root (or MXFA_REFERENCE_ROOT) is required")
    sys.path.insert(0, args.reference_root)
    import torch
    from mxflashattn import reference as ref  # the reference's own oracle

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    store: dict[str, np.ndarray] = {}

    for name, case in golden_cases.paged_cases().items():
        tdt = {"bf16": torch.bfloat16, "fp16": torch.float16}[case.dtype]
        store[f"{name}.digest"] = np.array(golden_cases.digest(
            case.q, case.k_cache, case.v_cache, case.block_table, case.cache_seqlens, case.k_new, case.v_new))
        for suffix, dt in (("out", tdt), ("out_f32", torch.float32)):
            q = torch.from_numpy(case.q).to(dt)
            kc = torch.from_numpy(case.k_cache).to(dt)
            vc = torch.from_numpy(case.v_cache).to(dt)
            kn = None if case.k_new is None else torch.from_numpy(case.k_new).to(dt)
            vn = None if case.v_new is None else torch.from_numpy(case.v_new).to(dt)
            sl = torch.from_numpy(case.cache_seqlens.copy())
            bt = None if case.block_table is None else torch.from_numpy(case.block_table)
            out = ref.attention_kvcache(q, kc, vc, cache_seqlens=sl, block_table=bt, k=kn, v=vn,
                                        softmax_scale=case.softmax_scale, causal=case.causal)
            store[f"{name}.{suffix}"] = out.float().numpy()
            if suffix == "out" and kn is not None:
                store[f"{name}.k_cache_after_digest"] = np.array(golden_cases.digest(kc.float().numpy()))
                store[f"{name}.v_cache_after_digest"] = np.array(golden_cases.digest(vc.float().numpy()))
                store[f"{name}.seqlens_after"] = sl.numpy().astype(np.int32)
        store[f"{name}.lse"] = _lse_paged(case, torch).astype(np.float32)

    for name, case in golden_cases.varlen_cases().items():
        tdt = {"bf16": torch.bfloat16, "fp16": torch.float16}[case.dtype]
        store[f"{name}.digest"] = np.array(golden_cases.digest(case.q, case.k, case.v, case.cu_q, case.cu_k))
        for suffix, dt in (("out", tdt), ("out_f32", torch.float32)):
            out = ref.attention_varlen(
                torch.from_numpy(case.q).to(dt), torch.from_numpy(case.k).to(dt),
                torch.from_numpy(case.v).to(dt), [int(x) for x in case.cu_q], [int(x) for x in case.cu_k],
                softmax_scale=case.softmax_scale, causal=case.causal)
            store[f"{name}.{suffix}"] = out.float().numpy()
        store[f"{name}.lse"] = _lse_varlen(case, torch).astype(np.float32)

    np.savez_compressed(args.out, **store)
    total = sum(v.nbytes for v in store.values())
    print(f"wrote {args.out}: {len(store)} arrays, {total / 1e6:.2f} MB uncompressed")
    assert math.isfinite(total)


if __name__ == "__main__":
    main()
