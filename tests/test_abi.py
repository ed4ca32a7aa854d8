"""The C-ABI boundary on the CPU: the library loads, exports every entry
point include/nncu.h declares, its host-only logic (spans, cache sizing,
errors) matches the reference's, and compute calls fail loudly without a
GPU instead of falling back to anything."""
from __future__ import annotations

import os
import re
import subprocess

import numpy as np
import pytest

import libllmcpu_b200 as N
from libllmcpu_b200 import build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "nncu.h")


@pytest.fixture(scope="module")
def L():
    if not os.path.exists(N.LIB_PATH):
        build.build()
    return N.lib()


def declared_functions() -> list[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(nncu_[a-z0-9_]+)\s*\(", text)))


def test_header_and_binding_agree():
    assert declared_functions() == sorted(N.EXPORTS)


def test_library_exports_every_declared_symbol(L):
    out = subprocess.run(["nm", "-D", "--defined-only", N.LIB_PATH], capture_output=True, text=True, check=True)
    exported = set(re.findall(r"\bT (nncu_[a-z0-9_]+)$", out.stdout, flags=re.M))
    missing = [f for f in declared_functions() if f not in exported]
    assert not missing, missing
    for f in declared_functions():
        assert hasattr(L, f)


def test_library_is_sm100a_only(L):
    # the device code is built for sm_100a only (no PTX for other targets, no host fallback)
    out = subprocess.run(["cuobjdump", "--list-elf", N.LIB_PATH], capture_output=True, text=True)
    if out.returncode != 0:
        pytest.skip("cuobjdump unavailable")
    arches = set(re.findall(r"sm_(\d+a?)", out.stdout))
    assert arches == {"100a"}, arches


# tests.cpp:1663-1678
SPAN_CASES = [
    (True, 0, 5, 10, 0, 5), (True, 3, 5, 10, 3, 5), (True, 0, 5, 5, 0, 4), (True, 3, 5, 5, 3, 4),
    (False, 0, 5, 10, 0, 9), (False, 4, 5, 10, 3, 7), (False, 4, 0, 10, 0, 2), (False, 4, 9, 10, 7, 9),
    (False, 512, 300, 1000, 44, 556),
]


@pytest.mark.parametrize("causal,window,pos,n_seq,first,last", SPAN_CASES)
def test_attn_span_known_answers(L, causal, window, pos, n_seq, first, last):
    assert N.attn_span(causal, window, pos, n_seq) == (first, last)


def test_attn_span_matches_oracle_everywhere(L):
    import oracle as O
    for causal in (True, False):
        for window in (0, 1, 3, 40, 512):
            for n_seq in (1, 5, 300):
                for pos in range(0, n_seq + 2, 7):
                    assert N.attn_span(causal, window, pos, n_seq) == O.attn_span(causal, window, pos, n_seq)


def test_kv_plan_ring_sizing_matches_reference(L):
    # tests.cpp:2598-2630 (test_sliding_ring_matches_full): a tiny Qwen3 with a sliding layer
    # (window 40) and a global one, n_ctx 1200, n_batch 16 -> ring of 256 rows, max_rewind 216
    layers = [(2, 32, 40, 0), (2, 32, 0, 1)]
    info, max_rewind, nbytes = N.kv_plan(layers, n_ctx=1200, n_batch=16, kv_type=N.KV_BF16)
    assert info[0].rows == 256 and info[0].window == 40
    assert info[1].rows == 1200 and info[1].window == 0
    assert max_rewind == 216
    # bytes: K and V, rows rounded up to whole 256-key blocks in HBM
    assert nbytes == 2 * 2 * 32 * 2 * (256 + 1280)


def test_kv_plan_gemma3_1b(L):
    # 26 layers, every 6th global; window 512, decode batch 1 -> rings of 768 rows
    layers = [(1, 256, 0 if (li + 1) % 6 == 0 else 512, li) for li in range(26)]
    info, max_rewind, _ = N.kv_plan(layers, n_ctx=4097 + 16, n_batch=1, kv_type=N.KV_F32)
    for li, x in enumerate(info):
        assert (x.rows, x.window) == ((4113, 0) if (li + 1) % 6 == 0 else (768, 512))
    assert max_rewind == 256


def test_kv_plan_rules(L):
    # a ring only when it is smaller than n_ctx
    info, mr, _ = N.kv_plan([(1, 64, 512, 0)], n_ctx=600, n_batch=16)
    assert info[0].rows == 600 and info[0].window == 0 and mr == 2 ** 31 - 1
    # a global layer reading a sliding layer's cache keeps it full
    info, mr, _ = N.kv_plan([(1, 64, 40, 0), (1, 64, 0, 0)], n_ctx=1200, n_batch=16)
    assert info[0].rows == 1200 and info[1].buffer == 0
    # bidirectional: one buffer of n_ctx rows for every layer
    info, mr, _ = N.kv_plan([(2, 64, 64, 0), (4, 64, 0, 1)], n_ctx=96, causal=False)
    assert [x.buffer for x in info] == [0, 0] and info[0].rows == 96


@pytest.mark.parametrize("layers,kw", [
    ([], dict(n_ctx=10)),
    ([(1, 64, 0, 0)], dict(n_ctx=0)),
    ([(1, 64, 0, 0)], dict(n_ctx=10, kv_type=7)),
    ([(0, 64, 0, 0)], dict(n_ctx=10)),
    ([(1, 64, 0, 3)], dict(n_ctx=10)),
    ([(1, 64, 0, 1), (1, 64, 0, 0)], dict(n_ctx=10)),
    ([(1, 64, 0, 0), (2, 64, 0, 0)], dict(n_ctx=10)),
])
def test_kv_plan_refuses_bad_arguments(L, layers, kw):
    with pytest.raises(N.NnncError) as e:
        if not layers:
            rc = L.nncu_kv_plan(None, 0, None, None, None, None)
            N._check(rc)
        N.kv_plan(layers, **kw)
    assert e.value.status == N.ERR_INVALID_ARGUMENT


def test_status_strings(L):
    assert L.nncu_status_string(0) == b"ok"
    assert L.nncu_status_string(N.ERR_CONTEXT_FULL) == b"context full"
    assert L.nncu_status_string(N.ERR_TIMEOUT)


def test_no_gpu_means_a_loud_failure(L):
    if L.nncu_device_check(0) == 0:
        pytest.skip("a GPU is present")
    assert L.nncu_last_status() == N.ERR_UNSUPPORTED
    with pytest.raises(N.NnncError) as e:
        N.KVCache([(8, 64, 0, 0)], n_ctx=64)
    assert e.value.status == N.ERR_UNSUPPORTED
    x = np.zeros(64, np.float32)
    with pytest.raises(N.NnncError):
        N.rmsnorm_dev(x, x, 1, 64, 1e-6)  # host memory, no device: refused, not computed


def test_forward_and_logits_refuse_bad_arguments_before_any_device_work(L):
    # argument checks come first: NULL handles and pointers, empty batches,
    # a gate passed in although the q projection makes it
    vp = None
    p = N.params(n_tok=1, pos0=0, n_head=4, n_kv=2, head_dim=64)
    w = N.AttnWeights()
    assert L.nncu_attention_forward_dev(vp, 0, 0, p, w, vp, vp, vp) == N.ERR_INVALID_ARGUMENT
    assert L.nncu_attention_forward_batch_dev(vp, 0, 0, vp, p, w, vp, vp, vp) == N.ERR_INVALID_ARGUMENT
    head = N.Weight(N.W_Q4_S, 64, 64, None, None, None)
    assert L.nncu_logits_batch_dev(head, vp, 1, vp, 0.0, vp, vp) == N.ERR_INVALID_ARGUMENT
    assert L.nncu_argmax_rows_dev(vp, 4, 1, 4, vp, vp) == N.ERR_INVALID_ARGUMENT
    assert b"NULL" in L.nncu_last_error()


def test_forward_bench_parses_its_arguments():
    from libllmcpu_b200 import forward_bench

    with pytest.raises(SystemExit) as e:
        forward_bench.main(["--help"])
    assert e.value.code == 0
    assert set(forward_bench.MODELS) >= {"gemma3-4b", "qwen3-8b", "qwen3.5-4b", "llama3.2-1b"}
