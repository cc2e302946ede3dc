"""The backend passes every C-ABI argument in the slot the header gives it (CPU, no device).

The backend module is driven with CPU tensors against a recording stand-in
for the library (the host-only planning entries still run in the real one).
Each recorded call is matched to the header prototype's parameter names, and
every parameter is checked against the value it must carry: pointers of the
right tensors, the geometry read from the right dimensions, the flags, the
scale and the stream.  A swap of two same-typed arguments (PS and BTW, HQ and
HKV, k and v) that the numerical GPU tests might not expose fails here.
"""

from __future__ import annotations

import contextlib
import os
import re

import pytest
import torch

from mxflashattn_b200 import _lib, backend

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "mxfa_b200.h")
STREAM = 0x5A5A
HOST_ONLY = ("mxfa_kvcache_plan", "mxfa_split_workspace_bytes", "mxfa_split_counter_bytes", "mxfa_last_error")


def _parameter_names():
    text = re.sub(r"/\*.*?\*/|//[^\n]*", " ", open(HEADER).read(), flags=re.S)
    text = re.sub(r"^\s*#.*$", ";", text, flags=re.M)
    text = re.sub(r'extern\s+"C"\s*\{|\}', ";", text)
    names = {}
    for _, name, params in re.findall(r"(?<=;)\s*([A-Za-z_][\w\s]*?\**)\s*\b(mxfa_[a-z0-9_]+)\s*\(([^)]*)\)\s*;",
                                      text):
        params = " ".join(params.split())
        names[name] = [] if params in ("", "void") else [re.findall(r"(\w+)$", a.strip())[0] for a in params.split(",")]
    return names


NAMES = _parameter_names()


class _Recorder:
    def __init__(self, real):
        self.real, self.calls = real, []

    def __getattr__(self, name):
        if name in HOST_ONLY:
            return getattr(self.real, name)

        def launch(*args):
            self.calls.append((name, dict(zip(NAMES[name], args, strict=True))))
            return 0

        return launch


@pytest.fixture
def rec(monkeypatch):
    recorder = _Recorder(_lib.load())
    monkeypatch.setattr(backend, "_LIB", [recorder])
    monkeypatch.setattr(backend, "_on", lambda t: contextlib.nullcontext())
    monkeypatch.setattr(backend, "_stream", lambda t: STREAM)
    return recorder


def _paged(dtype=torch.bfloat16, B=3, HQ=16, HKV=4, D=128, PS=16, pages=40, BTW=7, Sq=1):
    q = torch.zeros(B, Sq, HQ, D, dtype=dtype)
    kc = torch.zeros(pages, PS, HKV, D, dtype=dtype)
    vc = torch.zeros(pages, PS, HKV, D, dtype=dtype)
    seq = torch.tensor([5, 100, 17][:B], dtype=torch.int32)
    bt = torch.arange(B * BTW, dtype=torch.int32).reshape(B, BTW)
    return q, kc, vc, seq, bt


def _check(call, **expected):
    for key, value in expected.items():
        got = call[key]
        if isinstance(value, float):
            assert got == pytest.approx(value, rel=1e-7), key
        else:
            assert got == value, key


@pytest.mark.parametrize("single_launch", [False, True])
@pytest.mark.parametrize("num_splits", [1, 3])
def test_kvcache_attention_arguments(rec, single_launch, num_splits):
    q, kc, vc, seq, bt = _paged()
    out, lse = backend.kvcache_attention(q, kc, vc, seq, bt, 0.125, True, append_len=2, return_lse=True,
                                         num_splits=num_splits, chunk_len=48 if num_splits > 1 else 112,
                                         single_launch=single_launch)
    (name, call), = rec.calls
    assert name == ("mxfa_kvcache_attention_counted_launch" if single_launch and num_splits > 1
                    else "mxfa_kvcache_attention_launch")
    _check(call, q=q.data_ptr(), k_cache=kc.data_ptr(), v_cache=vc.data_ptr(), block_table=bt.data_ptr(),
           seqlens=seq.data_ptr(), out=out.data_ptr(), lse=lse.data_ptr(), B=3, Sq=1, HQ=16, HKV=4, D=128, PS=16,
           BTW=7, num_pages=40, append_len=2, num_splits=num_splits, causal=1, bf16=1, scale=0.125, stream=STREAM)
    if num_splits > 1:
        assert call["workspace_bytes"] == rec.real.mxfa_split_workspace_bytes(3 * 16, 128, num_splits)
    else:
        assert call["workspace"] is None and call["workspace_bytes"] == 0


def test_ordered_and_fp8_arguments(rec):
    fp8 = getattr(torch, "float8_e4m3fn", None)
    if fp8 is None:
        pytest.skip("no float8_e4m3fn in this torch")
    q, kc, vc, seq, bt = _paged(dtype=torch.float16)
    k8, v8 = kc.to(fp8), vc.to(fp8)
    order = torch.tensor([1, 2, 0], dtype=torch.int32)
    out = backend.kvcache_attention(q, k8, v8, seq, bt, 0.5, False, k_scale=0.25, v_scale=4.0, length_order=order)
    backend.kvcache_attention(q, k8, v8, seq, bt, 0.5, False, k_scale=0.25, v_scale=4.0)
    (n1, ordered), (n2, plain) = rec.calls
    assert (n1, n2) == ("mxfa_kvcache_attention_ordered_launch", "mxfa_kvcache_attention_fp8_launch")
    _check(ordered, length_order=order.data_ptr(), out=out.data_ptr(), k_cache=k8.data_ptr(), v_cache=v8.data_ptr(),
           HQ=16, HKV=4, PS=16, BTW=7, num_pages=40, bf16=0, kv_fp8=1, k_scale=0.25, v_scale=4.0, scale=0.5,
           stream=STREAM)
    _check(plain, k_cache=k8.data_ptr(), v_cache=v8.data_ptr(), HQ=16, HKV=4, PS=16, BTW=7, num_pages=40, bf16=0,
           k_scale=0.25, v_scale=4.0, scale=0.5, stream=STREAM)


def test_fused_append_arguments(rec):
    q, kc, vc, seq, bt = _paged(Sq=2)
    k_new = torch.ones(3, 2, 4, 128, dtype=torch.bfloat16)
    v_new = torch.full((3, 2, 4, 128), 2.0, dtype=torch.bfloat16)
    out = backend.kvcache_attention(q, kc, vc, seq, bt, 0.25, True, append_len=2, k_new=k_new, v_new=v_new)
    (name, call), = rec.calls
    assert name == "mxfa_kvcache_append_attention_launch"
    _check(call, k_new=k_new.data_ptr(), v_new=v_new.data_ptr(), out=out.data_ptr(), B=3, Sq=2, HQ=16, HKV=4,
           PS=16, BTW=7, num_pages=40, append_len=2, causal=1, stream=STREAM)


def test_dense_cache_arguments(rec):
    q = torch.zeros(2, 1, 8, 64, dtype=torch.float16)
    kc = torch.zeros(2, 300, 2, 64, dtype=torch.float16)
    vc = torch.zeros(2, 300, 2, 64, dtype=torch.float16)
    seq = torch.tensor([10, 299], dtype=torch.int32)
    backend.kvcache_attention(q, kc, vc, seq, None, 0.1, False, num_splits=1, chunk_len=304)
    (name, call), = rec.calls
    _check(call, block_table=None, B=2, HQ=8, HKV=2, D=64, PS=300, BTW=0, num_pages=2, bf16=0)


def test_append_and_length_update_arguments(rec):
    _, kc, vc, seq, bt = _paged()
    k = torch.ones(3, 5, 4, 128, dtype=torch.bfloat16)
    v = torch.ones(3, 5, 4, 128, dtype=torch.bfloat16)
    backend.kv_append(kc, vc, k, v, seq, bt)
    backend.seqlens_add_(seq, 5)
    (n1, app), (n2, add) = rec.calls
    assert (n1, n2) == ("mxfa_kv_append_launch", "mxfa_seqlens_add_launch")
    _check(app, k_new=k.data_ptr(), v_new=v.data_ptr(), k_cache=kc.data_ptr(), v_cache=vc.data_ptr(),
           block_table=bt.data_ptr(), seqlens=seq.data_ptr(), B=3, Sk=5, HKV=4, D=128, PS=16, BTW=7, num_pages=40,
           elem_bytes=2, stream=STREAM)
    _check(add, seqlens=seq.data_ptr(), is_int64=0, B=3, delta=5, stream=STREAM)


@pytest.mark.parametrize("exact", [False, True])
def test_varlen_and_dense_prefill_arguments(rec, exact):
    q = torch.zeros(40, 8, 128, dtype=torch.bfloat16)
    k = torch.zeros(50, 2, 128, dtype=torch.bfloat16)
    v = torch.ones(50, 2, 128, dtype=torch.bfloat16)
    cu_q = torch.tensor([0, 15, 40], dtype=torch.int32)
    cu_k = torch.tensor([0, 20, 50], dtype=torch.int32)
    out, lse = backend.flash_attn_varlen_func(q, k, v, cu_q, cu_k, 25, 30, True, 0.2, return_lse=True, exact_p=exact)
    qd = torch.zeros(2, 9, 4, 64, dtype=torch.float16)
    kd = torch.zeros(2, 11, 2, 64, dtype=torch.float16)
    vd = torch.ones(2, 11, 2, 64, dtype=torch.float16)
    outd = backend.flash_attn_func(qd, kd, vd, False, 0.3, exact_p=exact)
    (n1, var), (n2, dense) = rec.calls
    name = "mxfa_varlen_fwd_exact_launch" if exact else "mxfa_varlen_fwd_launch"
    assert n1 == n2 == name
    _check(var, q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), cu_q=cu_q.data_ptr(), cu_k=cu_k.data_ptr(),
           out=out.data_ptr(), lse=lse.data_ptr(), B=2, max_q=25, max_k=30, total_q=40, total_k=50, HQ=8, HKV=2,
           D=128, causal=1, bf16=1, scale=0.2, stream=STREAM)
    _check(dense, q=qd.data_ptr(), k=kd.data_ptr(), v=vd.data_ptr(), cu_q=None, cu_k=None, out=outd.data_ptr(),
           lse=None, B=2, max_q=9, max_k=11, total_q=18, total_k=22, HQ=4, HKV=2, D=64, causal=0, bf16=0, scale=0.3)


def test_packed_combine_and_merge_arguments(rec):
    q, kc, vc, seq, bt = _paged()
    packed = backend.kvcache_attention_packed(q, kc, vc, seq, bt, 0.125, num_splits=2, chunk_len=64)
    ows = torch.zeros(48, 2, 128)
    mdws = torch.zeros(48, 2, 2)
    out, lse = backend.split_combine(ows, mdws, 48, 128, 2, torch.float16, lse=True)
    gathered = torch.zeros(4, 48, 129)
    mout, mlse = backend.lse_merge(gathered, 48, 128, torch.bfloat16, lse=True)
    (n1, pk), (n2, cb), (n3, mg) = rec.calls
    assert (n1, n2, n3) == ("mxfa_kvcache_attention_packed_launch", "mxfa_split_combine_launch",
                            "mxfa_lse_merge_launch")
    _check(pk, packed=packed.data_ptr(), B=3, HQ=16, HKV=4, D=128, PS=16, BTW=7, num_pages=40, num_splits=2,
           chunk_len=64, bf16=1, scale=0.125, stream=STREAM)
    _check(cb, ows=ows.data_ptr(), mdws=mdws.data_ptr(), out=out.data_ptr(), out_f32=None, lse=lse.data_ptr(),
           rows=48, D=128, NP=2, bf16=0, stream=STREAM)
    _check(mg, packed=gathered.data_ptr(), out=mout.data_ptr(), lse=mlse.data_ptr(), N=4, rows=48, D=128, bf16=1,
           stream=STREAM)
