"""End-to-end vLLM generation through the B200 decode hook (integrations/vllm/smoke_generate.py).

Plays the role of the reference's smoke script: one run with vLLM's own
FLASH_ATTN backend (``--baseline-only``) and one with the MXFlashAttn class
registered in its place (``--candidate``), each writing a JSON record, and
``--compare`` to set the two side by side.

Differences from the reference, all forced by this environment (no network,
a vLLM newer than the reference's pin):

* The model is built from an architecture config written locally
  (``qwen3-4b`` / ``qwen3-8b`` or a directory holding a config.json) and
  initialised with ``load_format="dummy"`` (seeded random weights).
* Prompts are seeded random token ids (``skip_tokenizer_init``), so no
  tokenizer is needed; generation is greedy with ``ignore_eos`` so every
  request decodes exactly ``--max-tokens`` tokens.
* The engine runs in this process (``VLLM_ENABLE_V1_MULTIPROCESSING=0``) so
  the backend registration made here is the one the model runner sees.
* The vLLM version pin (0.17.0) is reported, not enforced.

The candidate record counts the dispatch events the hook wrote for every
decode call (path ``cuda_sm100``) and the calls it handed back to vLLM
(prefill and mixed batches).
"""

from __future__ import annotations

import argparse
import json
import os
import tempfile
import time
from pathlib import Path

# Architecture hyper-parameters of the published Qwen3 dense models (the
# shapes BASELINE configs 2 and 3 are quoted on).  Weights are random.
ARCHITECTURES = {
    "qwen3-4b": dict(hidden_size=2560, intermediate_size=9728, num_hidden_layers=36, num_attention_heads=32,
                     num_key_value_heads=8, head_dim=128, tie_word_embeddings=True),
    "qwen3-8b": dict(hidden_size=4096, intermediate_size=12288, num_hidden_layers=36, num_attention_heads=32,
                     num_key_value_heads=8, head_dim=128, tie_word_embeddings=False),
}
_COMMON = dict(architectures=["Qwen3ForCausalLM"], model_type="qwen3", vocab_size=151936, hidden_act="silu",
               max_position_embeddings=40960, rms_norm_eps=1e-6, rope_theta=1000000.0, attention_bias=False,
               attention_dropout=0.0, torch_dtype="bfloat16", bos_token_id=151643, eos_token_id=151645,
               use_sliding_window=False, initializer_range=0.02)


def write_model_dir(name: str, root: str | os.PathLike) -> Path:
    """A directory holding the config.json of one of ARCHITECTURES."""
    if name not in ARCHITECTURES:
        raise ValueError(f"unknown architecture {name!r}; choose from {sorted(ARCHITECTURES)}")
    path = Path(root) / name
    path.mkdir(parents=True, exist_ok=True)
    config = dict(_COMMON, **ARCHITECTURES[name])
    (path / "config.json").write_text(json.dumps(config, indent=2), encoding="utf-8")
    (path / "generation_config.json").write_text(
        json.dumps({"bos_token_id": config["bos_token_id"], "eos_token_id": config["eos_token_id"]}),
        encoding="utf-8")
    return path


def make_prompts(batch: int, min_len: int, max_len: int, seed: int, vocab: int = 151936) -> list[list[int]]:
    """Seeded random token-id prompts with lengths U[min_len, max_len]."""
    import numpy as np

    rng = np.random.default_rng(seed)
    lengths = rng.integers(min_len, max_len + 1, size=batch)
    return [rng.integers(0, vocab, size=int(n)).tolist() for n in lengths]


def count_events(path: Path | None) -> dict[str, int]:
    """Dispatch-event counts by path from the hook's JSONL trail."""
    counts: dict[str, int] = {}
    if path is None or not path.exists():
        return counts
    for line in path.read_text(encoding="utf-8").splitlines():
        if line.strip():
            key = json.loads(line).get("path", "unknown")
            counts[key] = counts.get(key, 0) + 1
    return counts


def shadow_summary(path: Path | None) -> dict | None:
    """Largest kernel-vs-vLLM difference over the recorded shadow checks."""
    if path is None or not path.exists():
        return None
    checks = [json.loads(line) for line in path.read_text(encoding="utf-8").splitlines() if line.strip()]
    checks = [c for c in checks if c.get("path") == "shadow_check"]
    if not checks:
        return None
    summary = {
        "checks": len(checks),
        "max_abs_diff": max(c["max_abs_diff"] for c in checks),
        "max_abs_ref": max(c["max_abs_ref"] for c in checks),
        "worst_relative": max(c["max_abs_diff"] / max(c["max_abs_ref"], 1e-30) for c in checks),
    }
    exact = [c for c in checks if "max_ulps_kernel_vs_fp32" in c]
    if exact:
        summary["fp32_checks"] = len(exact)
        summary["max_ulps_kernel_vs_fp32"] = max(c["max_ulps_kernel_vs_fp32"] for c in exact)
        summary["max_ulps_vllm_vs_fp32"] = max(c["max_ulps_vllm_vs_fp32"] for c in exact)
        summary["max_abs_fp32"] = max(c["max_abs_fp32"] for c in exact)
    return summary


def compare_runs(baseline: dict, candidate: dict) -> dict:
    """Greedy-token agreement of two records with the same prompts.

    With random weights the logits sit close together, so two numerically
    different but correct attention kernels can pick different argmaxes; the
    log-probabilities of the chosen tokens, taken while the sequences still
    agree, show how close the runs are.
    """
    b_runs, c_runs = baseline["outputs"], candidate["outputs"]
    if len(b_runs) != len(c_runs):
        raise ValueError("records hold different numbers of requests")
    first_diff, same, total, lp_gap = [], 0, 0, 0.0
    for b, c in zip(b_runs, c_runs):
        bt, ct = b["token_ids"], c["token_ids"]
        n = min(len(bt), len(ct))
        k = next((i for i in range(n) if bt[i] != ct[i]), n)
        first_diff.append(k)
        same += sum(1 for i in range(n) if bt[i] == ct[i])
        total += n
        for i in range(k):
            if b.get("logprobs") and c.get("logprobs"):
                lp_gap = max(lp_gap, abs(b["logprobs"][i] - c["logprobs"][i]))
    return {
        "requests": len(b_runs),
        "token_agreement": same / total if total else None,
        "first_divergence_median": sorted(first_diff)[len(first_diff) // 2] if first_diff else None,
        "first_divergence_min": min(first_diff) if first_diff else None,
        "max_logprob_gap_before_divergence": lp_gap,
        "baseline_tok_per_s": baseline.get("decode_tok_per_s"),
        "candidate_tok_per_s": candidate.get("decode_tok_per_s"),
    }


def run(args) -> dict:
    os.environ.setdefault("VLLM_ENABLE_V1_MULTIPROCESSING", "0")
    import torch

    registration = None
    dispatch_log = None
    if args.candidate:
        dispatch_log = args.output.with_suffix(".dispatch.jsonl").resolve()
        if dispatch_log.exists():
            dispatch_log.unlink()
        os.environ["MXFLASHATTN_DISPATCH_LOG"] = str(dispatch_log)
        # one line per N calls: per-call file appends would tax the timed run
        os.environ.setdefault("MXFLASHATTN_DISPATCH_SAMPLE", str(args.event_sample))
        if args.shadow_every > 0:
            os.environ["MXFLASHATTN_SHADOW_CHECK_EVERY"] = str(args.shadow_every)
        from mxflashattn_b200.integrations.vllm import backend as hook

        registration = hook.register_vllm_v1_backend()
        if registration.get("registered") != "true":
            raise SystemExit(f"MXFlashAttn backend registration failed: {registration}")
    from vllm import LLM, SamplingParams
    from vllm.inputs import TokensPrompt

    model = args.model
    if model in ARCHITECTURES:
        model = str(write_model_dir(model, tempfile.mkdtemp(prefix="mxfa_vllm_")))
    engine = LLM(model=model, load_format="dummy", skip_tokenizer_init=True, enforce_eager=args.eager,
                 max_model_len=args.max_model_len, gpu_memory_utilization=args.gpu_memory_utilization,
                 seed=args.seed, dtype=args.dtype, attention_backend="FLASH_ATTN")
    prompts = make_prompts(args.batch, args.prompt_min, args.prompt_max, args.seed)
    params = SamplingParams(temperature=0.0, max_tokens=args.max_tokens, ignore_eos=True, detokenize=False,
                            logprobs=0)
    engine.generate([TokensPrompt(prompt_token_ids=prompts[0][:16])],
                    SamplingParams(temperature=0.0, max_tokens=4, ignore_eos=True, detokenize=False),
                    use_tqdm=False)  # warm-up
    if dispatch_log is not None and dispatch_log.exists():
        dispatch_log.unlink()
    torch.cuda.synchronize()
    start = time.perf_counter()
    results = engine.generate([TokensPrompt(prompt_token_ids=p) for p in prompts], params, use_tqdm=False)
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - start
    outputs = []
    for r in results:
        comp = r.outputs[0]
        lps = None
        if comp.logprobs:
            lps = [float(step[tok].logprob) for step, tok in zip(comp.logprobs, comp.token_ids)]
        outputs.append({"prompt_len": len(r.prompt_token_ids), "token_ids": list(comp.token_ids), "logprobs": lps})
    generated = sum(len(o["token_ids"]) for o in outputs)
    events = count_events(dispatch_log)
    shadow = shadow_summary(dispatch_log)
    import vllm

    record = {
        "schema_version": 1,
        "kind": "vllm_mxflashattn_candidate" if args.candidate else "vllm_baseline_only",
        "model": args.model,
        "vllm": vllm.__version__,
        "vllm_pin": "0.17.0 (reference); not enforced",
        "torch": torch.__version__,
        "device": torch.cuda.get_device_name(),
        "batch": args.batch,
        "dtype": args.dtype,
        "prompt_lengths": [args.prompt_min, args.prompt_max],
        "max_tokens": args.max_tokens,
        "eager": args.eager,
        "registration": registration,
        "elapsed_s": elapsed,
        "generated_tokens": generated,
        "decode_tok_per_s": generated / elapsed if elapsed > 0 else None,
        "dispatch_event_counts": events,
        "shadow_checks": shadow,
        "dispatch_event_sample": int(os.environ.get("MXFLASHATTN_DISPATCH_SAMPLE", "0") or 0) if args.candidate else None,
        "outputs": outputs,
    }
    if args.candidate:
        decode_calls = events.get("cuda_sm100", 0)
        record["candidate_dispatch_verified"] = decode_calls > 0
        record["status"] = "candidate_dispatch_verified" if decode_calls > 0 else "candidate_not_verified"
    else:
        record["status"] = "baseline_only"
    return record


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--model", default="qwen3-4b", help="qwen3-4b, qwen3-8b, or a directory with config.json")
    parser.add_argument("--batch", type=int, default=64)
    parser.add_argument("--prompt-min", type=int, default=128)
    parser.add_argument("--prompt-max", type=int, default=1024)
    parser.add_argument("--max-tokens", type=int, default=256)
    parser.add_argument("--max-model-len", type=int, default=2048)
    parser.add_argument("--gpu-memory-utilization", type=float, default=0.5)
    parser.add_argument("--seed", type=int, default=0)
    parser.add_argument("--dtype", choices=("bfloat16", "float16"), default="bfloat16")
    parser.add_argument("--graphs", dest="eager", action="store_false", help="let vLLM compile and capture graphs")
    parser.add_argument("--output", type=Path, default=Path("vllm-run.json"))
    parser.add_argument("--event-sample", type=int, default=64, help="record one dispatch event per N calls")
    parser.add_argument("--shadow-every", type=int, default=0,
                        help="candidate: compare every N-th decode call with vLLM's own attention (syncs)")
    group = parser.add_mutually_exclusive_group(required=True)
    group.add_argument("--baseline-only", action="store_true")
    group.add_argument("--candidate", action="store_true")
    group.add_argument("--compare", nargs=2, type=Path, metavar=("BASELINE", "CANDIDATE"))
    args = parser.parse_args()
    if args.compare:
        base, cand = (json.loads(p.read_text(encoding="utf-8")) for p in args.compare)
        summary = compare_runs(base, cand)
        args.output.write_text(json.dumps(summary, indent=2), encoding="utf-8")
        print(json.dumps(summary))
        return
    record = run(args)
    args.output.parent.mkdir(parents=True, exist_ok=True)
    args.output.write_text(json.dumps(record), encoding="utf-8")
    print(json.dumps({k: v for k, v in record.items() if k != "outputs"}))


if __name__ == "__main__":
    main()
