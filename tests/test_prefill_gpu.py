"""GPU parity of the dense / varlen attention forward against the oracle."""

from __future__ import annotations

import numpy as np
import pytest

import cases as golden_cases
import oracle
from helpers import assert_close_lse, assert_close_out, host, p_rounding_bound
from mxflashattn_b200 import synthetic as syn

pytestmark = pytest.mark.gpu

VARLEN_GOLDEN = golden_cases.varlen_cases()


def _dev(case, device):
    import torch

    tdt = syn.torch_dtype(case.dtype)
    return (torch.from_numpy(case.q).to(device, tdt), torch.from_numpy(case.k).to(device, tdt),
            torch.from_numpy(case.v).to(device, tdt), torch.from_numpy(case.cu_q).to(device),
            torch.from_numpy(case.cu_k).to(device))


@pytest.mark.parametrize("name", sorted(VARLEN_GOLDEN))
def test_varlen_matches_reference_goldens(name, golden, cuda_device):
    from mxflashattn_b200 import flash_attn_varlen_func, get_last_dispatch_info

    case = VARLEN_GOLDEN[name]
    q, k, v, cu_q, cu_k = _dev(case, cuda_device)
    out = flash_attn_varlen_func(q, k, v, cu_q, cu_k, int(np.diff(case.cu_q).max()), int(np.diff(case.cu_k).max()),
                                 softmax_scale=case.softmax_scale, causal=case.causal)
    assert get_last_dispatch_info().backend == "cuda_sm100"
    abs_v = oracle.attention_varlen(case.q, case.k, np.abs(case.v), case.cu_q, case.cu_k,
                                    softmax_scale=case.softmax_scale, causal=case.causal)
    assert_close_out(host(out), golden[f"{name}.out_f32"], case.dtype, name,
                     extra=p_rounding_bound(case.dtype, abs_v))


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("d", [64, 128])
def test_varlen_normal_inputs_within_north_star_bound_without_allowance(dt, d, cuda_device):
    """Config 5's value distribution (q, k, v ~ N(0,1)) over several key tiles, every row and head against the
    fp32 oracle at the plain north-star bound: max-abs 2e-3 (fp16) / 1e-2 (bf16), no P-rounding allowance."""
    from mxflashattn_b200 import flash_attn_varlen_func

    case = syn.varlen_case(70 + d, q_lens=[300, 77, 1000], q_heads=8, kv_heads=2, head_dim=d, dtype=dt,
                           causal=True)
    q, k, v, cu_q, cu_k = _dev(case, cuda_device)
    out = flash_attn_varlen_func(q, k, v, cu_q, cu_k, 1000, 1000, causal=True)
    ref = oracle.attention_varlen(case.q, case.k, case.v, case.cu_q, case.cu_k, softmax_scale=case.softmax_scale,
                                  causal=True)
    assert_close_out(host(out), ref, dt, f"N(0,1) {dt} d{d} (strict)")


@pytest.mark.parametrize("name", sorted(VARLEN_GOLDEN))
def test_exact_p_varlen_goldens_within_north_star_bound_without_allowance(name, golden, cuda_device):
    """With P kept at ~16 bits (exact_p), every golden, outlier cases included, meets the north-star bound as
    stated: max-abs 2e-3 (fp16) / 1e-2 (bf16) against the reference's fp32 output, no P-rounding allowance."""
    from mxflashattn_b200 import backend

    case = VARLEN_GOLDEN[name]
    q, k, v, cu_q, cu_k = _dev(case, cuda_device)
    out = backend.flash_attn_varlen_func(q, k, v, cu_q, cu_k, int(np.diff(case.cu_q).max()),
                                         int(np.diff(case.cu_k).max()), case.causal, case.softmax_scale,
                                         exact_p=True)
    assert_close_out(host(out), golden[f"{name}.out_f32"], case.dtype, name + " (exact P, strict)")


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("d", [64, 128])
def test_exact_p_outliers_within_north_star_bound_without_allowance(dt, d, cuda_device):
    """The coverage matrix's value distribution (1% of K/V entries x50) over several key tiles, every row and head,
    output and LSE, at the plain north-star bound with exact_p."""
    from mxflashattn_b200 import backend

    case = syn.varlen_case(70 + d, q_lens=[300, 77, 1000], q_heads=8, kv_heads=2, head_dim=d, dtype=dt,
                           causal=True, outlier_frac=0.01)
    q, k, v, cu_q, cu_k = _dev(case, cuda_device)
    out, lse = backend.flash_attn_varlen_func(q, k, v, cu_q, cu_k, 1000, 1000, True, case.softmax_scale,
                                              return_lse=True, exact_p=True)
    ref, ref_lse = oracle.attention_varlen(case.q, case.k, case.v, case.cu_q, case.cu_k,
                                           softmax_scale=case.softmax_scale, causal=True, return_lse=True)
    assert_close_out(host(out), ref, dt, f"outliers {dt} d{d} (exact P, strict)")
    assert_close_lse(host(lse), np.asarray(ref_lse).T, f"outliers {dt} d{d} (exact P) LSE")  # oracle LSE is [H, T]


@pytest.mark.parametrize("name", ["varlen_causal_bf16", "varlen_causal_d128_gq4"])
def test_varlen_lse(name, golden, cuda_device):
    from mxflashattn_b200 import backend

    case = VARLEN_GOLDEN[name]
    q, k, v, cu_q, cu_k = _dev(case, cuda_device)
    _, lse = backend.flash_attn_varlen_func(q, k, v, cu_q, cu_k, int(np.diff(case.cu_q).max()),
                                            int(np.diff(case.cu_k).max()), case.causal, case.softmax_scale,
                                            return_lse=True)
    assert_close_lse(host(lse), golden[f"{name}.lse"], name)


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("causal", [True, False])
def test_dense_batched_forward(dt, d, causal, cuda_device):
    import torch

    from mxflashattn_b200 import flash_attn_func

    rng = np.random.default_rng(d + causal)
    q = syn.round_dtype(rng.standard_normal((2, 77, 8, d), dtype=np.float32), dt)
    k = syn.round_dtype(rng.standard_normal((2, 130, 2, d), dtype=np.float32), dt)
    v = syn.round_dtype(rng.standard_normal((2, 130, 2, d), dtype=np.float32), dt)
    tdt = syn.torch_dtype(dt)
    out = flash_attn_func(torch.from_numpy(q).to(cuda_device, tdt), torch.from_numpy(k).to(cuda_device, tdt),
                          torch.from_numpy(v).to(cuda_device, tdt), causal=causal)
    ref = oracle.attention_batched(q, k, v, causal=causal)
    assert_close_out(host(out), ref, dt, f"dense d{d} causal={causal}")


def test_causal_query_longer_than_key_gives_zero_rows(cuda_device):
    """reference test_api.py:52-62 on the device: rows with no visible key are exactly 0."""
    import torch

    from mxflashattn_b200 import flash_attn_func

    torch.manual_seed(0)
    q = torch.randn(1, 3, 2, 64, device=cuda_device, dtype=torch.float16)
    k = torch.randn(1, 1, 1, 64, device=cuda_device, dtype=torch.float16)
    v = torch.randn_like(k)
    out = flash_attn_func(q, k, v, causal=True)
    assert torch.isfinite(out).all()
    assert torch.equal(out[:, :2], torch.zeros_like(out[:, :2]))
    torch.testing.assert_close(out[:, 2:], v.expand(-1, -1, 2, -1), rtol=0, atol=1e-3)


def test_zero_scale_is_uniform_average(cuda_device):
    import torch

    from mxflashattn_b200 import flash_attn_func

    torch.manual_seed(1)
    q = torch.randn(1, 4, 4, 64, device=cuda_device, dtype=torch.bfloat16)
    k = torch.randn(1, 6, 2, 64, device=cuda_device, dtype=torch.bfloat16)
    v = torch.randn_like(k)
    out = flash_attn_func(q, k, v, softmax_scale=0.0)
    expect = v.float().mean(dim=1, keepdim=True).repeat_interleave(2, dim=2).expand(-1, 4, -1, -1)
    torch.testing.assert_close(out.float(), expect, rtol=0, atol=1e-2)


def test_prefill_config_varlen_sampled_rows(cuda_device):
    """Config 5 prefill ({15000, 1024, 512, 37}, Hq=32, Hk=8, D=128, causal): rows sampled vs oracle."""
    import torch

    from mxflashattn_b200 import flash_attn_varlen_func

    lens = [15000, 1024, 512, 37]
    case = syn.varlen_case(55, q_lens=lens, q_heads=32, kv_heads=8, head_dim=128, dtype="bf16", causal=True)
    q, k, v, cu_q, cu_k = _dev(case, cuda_device)
    out = flash_attn_varlen_func(q, k, v, cu_q, cu_k, max(lens), max(lens), causal=True)
    torch.cuda.synchronize()
    out_h = host(out)
    assert np.isfinite(out_h).all()
    rng = np.random.default_rng(3)
    for s, L in enumerate(lens):
        start = int(case.cu_q[s])
        rows = np.unique(np.concatenate([[0, L - 1], rng.integers(0, L, size=6)]))
        for h in (0, 13, 31):
            kh = h // 4
            keys = case.k[start:start + L, kh]
            vals = case.v[start:start + L, kh]
            for r in rows:
                sc = (keys[: r + 1] @ case.q[start + r, h]) * case.softmax_scale
                p = np.exp(sc - sc.max())
                ref = (p / p.sum()) @ vals[: r + 1]
                err = float(np.max(np.abs(out_h[start + r, h] - ref)))
                assert err <= 1e-2, f"seq {s} row {r} head {h}: {err:.3e}"


@pytest.mark.parametrize("causal", [True, False])
def test_no_reads_past_the_packed_tensors(causal, cuda_device):
    """q/k/v are prefixes of NaN-filled buffers: a read past their last row would poison the output."""
    import torch

    from mxflashattn_b200 import flash_attn_varlen_func

    case = syn.varlen_case(61, q_lens=[37, 130, 3], q_heads=8, kv_heads=2, head_dim=128, dtype="bf16",
                           causal=causal)
    tdt = syn.torch_dtype(case.dtype)

    def poisoned(x):
        big = torch.full((x.shape[0] + 256,) + x.shape[1:], float("nan"), device=cuda_device, dtype=tdt)
        big[: x.shape[0]] = torch.from_numpy(x).to(cuda_device, tdt)
        return big[: x.shape[0]]

    q, k, v = poisoned(case.q), poisoned(case.k), poisoned(case.v)
    cu = torch.from_numpy(case.cu_q).to(cuda_device)
    out = flash_attn_varlen_func(q, k, v, cu, cu, 130, 130, causal=causal)
    ref = oracle.attention_varlen(case.q, case.k, case.v, case.cu_q, case.cu_k, causal=causal)
    assert_close_out(host(out), ref, "bf16", f"poisoned tail causal={causal}",
                     extra=p_rounding_bound("bf16", oracle.attention_varlen(
                         case.q, case.k, np.abs(case.v), case.cu_q, case.cu_k, causal=causal)))


def _rescale_case(seed, lens, dt, boost_every=197, boost=12.0):
    """Varlen q/k/v ~ N(0,1) whose keys at every ``boost_every``-th position are scaled by ``boost``.

    Those keys' scores sit far above everything before them, so row maxima
    jump past the lazy-rescale threshold deep into each sequence, after both
    softmax groups' first tiles: the accumulators are rescaled in tensor
    memory mid-sequence.  A stride of 197 puts the boosted keys in key tiles
    1, 3, 4, 6 and 7 of 128, so both softmax groups (odd and even tiles) see
    jumps after their first tile.
    """
    rng = np.random.default_rng(seed)
    total = sum(lens)
    q = syn.round_dtype(rng.standard_normal((total, 8, 128), dtype=np.float32), dt)
    k = rng.standard_normal((total, 2, 128), dtype=np.float32)
    v = syn.round_dtype(rng.standard_normal((total, 2, 128), dtype=np.float32), dt)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    for s in range(len(lens)):
        for pos in range(boost_every, lens[s], boost_every):
            k[cu[s] + pos] *= boost
    return q, syn.round_dtype(k, dt), v, cu


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("dt", ["bf16", "fp16"])
def test_row_max_jumps_rescale_the_accumulators(causal, dt, cuda_device):
    import torch

    from mxflashattn_b200 import backend

    lens = [1100, 700]
    q, k, v, cu = _rescale_case(91 + causal, lens, dt)
    tdt = syn.torch_dtype(dt)
    tq, tk, tv = (torch.from_numpy(x).to(cuda_device, tdt) for x in (q, k, v))
    tcu = torch.from_numpy(cu).to(cuda_device)
    out, lse = backend.flash_attn_varlen_func(tq, tk, tv, tcu, tcu, max(lens), max(lens), causal, 128 ** -0.5,
                                              return_lse=True)
    torch.cuda.synchronize()
    ref, ref_lse = oracle.attention_varlen(q, k, v, cu, cu, causal=causal, return_lse=True)
    abs_v = oracle.attention_varlen(q, k, np.abs(v), cu, cu, causal=causal)
    assert_close_out(host(out), ref, dt, f"rescale causal={causal}", extra=p_rounding_bound(dt, abs_v))
    assert_close_lse(host(lse), ref_lse.T, f"rescale lse causal={causal}")


def test_negative_scale_takes_the_row_minimum(cuda_device):
    """A negative softmax scale: the stable exponent is the row's minimum raw score."""
    import torch

    from mxflashattn_b200 import flash_attn_varlen_func

    lens = [300, 45]
    case = syn.varlen_case(93, q_lens=lens, q_heads=8, kv_heads=2, head_dim=128, dtype="bf16", causal=True)
    q, k, v, cu_q, cu_k = _dev(case, cuda_device)
    scale = -0.09
    out = flash_attn_varlen_func(q, k, v, cu_q, cu_k, max(lens), max(lens), softmax_scale=scale, causal=True)
    torch.cuda.synchronize()
    ref = oracle.attention_varlen(case.q, case.k, case.v, case.cu_q, case.cu_k, softmax_scale=scale, causal=True)
    abs_v = oracle.attention_varlen(case.q, case.k, np.abs(case.v), case.cu_q, case.cu_k, softmax_scale=scale,
                                    causal=True)
    assert_close_out(host(out), ref, "bf16", "negative scale", extra=p_rounding_bound("bf16", abs_v))


def test_many_sequences_with_keys_longer_than_queries(cuda_device):
    """200 sequences, q 1-260 tokens, k = q + 0-400 tokens (chunked-prefill shape): bottom-right causal
    masking across several tiles, a grid that is mostly empty query tiles, every row checked."""
    import torch

    from mxflashattn_b200 import flash_attn_varlen_func

    rng = np.random.default_rng(2024)
    q_lens = rng.integers(1, 261, size=200).tolist()
    k_lens = [q + int(rng.integers(0, 401)) for q in q_lens]
    case = syn.varlen_case(2024, q_lens=q_lens, k_lens=k_lens, q_heads=8, kv_heads=2, head_dim=128, dtype="bf16",
                           causal=True)
    q, k, v, cu_q, cu_k = _dev(case, cuda_device)
    out = flash_attn_varlen_func(q, k, v, cu_q, cu_k, max(q_lens), max(k_lens), causal=True)
    torch.cuda.synchronize()
    ref = oracle.attention_varlen(case.q, case.k, case.v, case.cu_q, case.cu_k, causal=True)
    abs_v = oracle.attention_varlen(case.q, case.k, np.abs(case.v), case.cu_q, case.cu_k, causal=True)
    assert_close_out(host(out), ref, "bf16", "many sequences, k longer than q", extra=p_rounding_bound("bf16", abs_v))


def test_cached_tensor_maps_follow_the_shape_at_the_same_address(cuda_device):
    """The library caches the prefill operands' TMA descriptors by address and shape: two calls on the same buffers
    with different row counts must each see their own rows (a map cached for the shorter call would read zeros)."""
    import torch

    from mxflashattn_b200 import backend

    big = syn.varlen_case(81, q_lens=[500], q_heads=8, kv_heads=2, head_dim=128, dtype="bf16", causal=True)
    q, k, v, _, _ = _dev(big, cuda_device)
    for n in (300, 500, 300):
        cu = torch.tensor([0, n], dtype=torch.int32, device=cuda_device)
        out = backend.flash_attn_varlen_func(q[:n], k[:n], v[:n], cu, cu, n, n, True, big.softmax_scale)
        ref = oracle.attention_varlen(big.q[:n], big.k[:n], big.v[:n], np.array([0, n], np.int32),
                                      np.array([0, n], np.int32), softmax_scale=big.softmax_scale, causal=True)
        assert_close_out(host(out), ref, "bf16", f"rows {n}")


def test_captured_replays_and_eager_launches_give_the_same_bits(cuda_device):
    """A forward captured as the first launch on a fresh stream, its graph replays, and later eager launches on
    that stream give the same bits (the kernel keeps no state between launches), within the bound vs the oracle."""
    import torch

    from mxflashattn_b200 import backend

    case = syn.varlen_case(91, q_lens=[3000, 700, 129, 5], q_heads=8, kv_heads=2, head_dim=128, dtype="bf16",
                           causal=True)
    q, k, v, cu_q, cu_k = _dev(case, cuda_device)

    def call():
        return backend.flash_attn_varlen_func(q, k, v, cu_q, cu_k, 3000, 3000, True, case.softmax_scale)

    call()  # kernel attributes and tensor maps set up outside the capture, on another stream
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(cuda_device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        captured = call()
    outs = []
    with torch.cuda.stream(stream):
        for _ in range(2):
            graph.replay()
            outs.append(captured.clone())
        for _ in range(3):
            outs.append(call())
    torch.cuda.synchronize()
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    ref = oracle.attention_varlen(case.q, case.k, case.v, case.cu_q, case.cu_k, causal=True)
    abs_v = oracle.attention_varlen(case.q, case.k, np.abs(case.v), case.cu_q, case.cu_k, causal=True)
    assert_close_out(host(outs[0]), ref, "bf16", "captured and eager launches", extra=p_rounding_bound("bf16", abs_v))
    del graph
