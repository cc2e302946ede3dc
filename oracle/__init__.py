"""CPU correctness oracle for the MXFlashAttn hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in ``mxflashattn_b200`` imports this
package; only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg
of ``bench.py`` (and its ``--impl reference`` arm) may use it, and there only
as the checker or the timed CPU baseline, never as a product path.

The oracle restates, in numpy float32 (plus a float64 cross-check), the
algorithm of the reference's PyTorch oracle ``mxflashattn/reference.py``:

* ``attention_single``   -> reference.py:8-40
* ``attention_batched``  -> reference.py:43-57
* ``attention_varlen``   -> reference.py:60-85
* ``attention_kvcache``  -> reference.py:88-139 (paged/dense append + gather)
* ``attention_chunked``, ``attention_chunked_fallback`` -> the chunked
  online-softmax prototype ``mxflashattn/prefill.py:11-108`` (a second
  oracle for the online softmax; pinned by ``tests/golden/chunked.npz``,
  which ``tests/golden/make_chunked_golden.py`` produced by running it)

The reference returns no log-sum-exp; ``lse`` here is the harness addition
the split-KV merge needs (natural-log logsumexp of the scaled scores, the
same scores the reference softmax normalises).

Parity pin: ``tests/test_oracle_golden.py`` checks this oracle against the
golden vectors in ``tests/golden/`` that ``tests/golden/make_golden.py``
produced by importing and running the reference implementation itself.
"""

from .attention import (
    attention_batched,
    attention_chunked,
    attention_chunked_fallback,
    attention_kvcache,
    attention_single,
    attention_varlen,
    gather_paged_kv,
    split_partials,
    merge_partials,
)

__all__ = [
    "attention_single",
    "attention_batched",
    "attention_chunked",
    "attention_chunked_fallback",
    "attention_varlen",
    "attention_kvcache",
    "gather_paged_kv",
    "split_partials",
    "merge_partials",
]
