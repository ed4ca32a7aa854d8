"""Causal prefill on the tensor cores (k_prefill.cu: tcgen05 Q K^T and P V,
bf16 operands, fp32 accumulation) against the checker, through the C ABI.

A batch of at least 128 tokens on a bf16 cache of head_dim 128 takes this
path. Its q rows and softmax probabilities are rounded to bf16 for the tensor
cores, which the reference (fp32 q, fp32 probabilities) does not do, so its
tolerance is stated separately from north_star's fp32/fp16 bar:
max-abs <= 2e-2 and relative-L2 <= 1e-2 (the errors measured here are ~10x
smaller). The checker is fed the same bf16-rounded K/V (the cache's type)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from oracle import scenarios as S
from oracle.scenarios import LayerSpec

from gpu_helpers import assert_close, run_product

pytestmark = pytest.mark.gpu

TOL_BF16_ABS, TOL_BF16_REL = 2e-2, 1e-2


def check_prefill(N, case, which="oracle"):
    want, caches = S.run_checker(case, which)
    got, kv = run_product(N, case)
    errs = []
    for s in range(case.n_seqs):
        for li in range(len(case.layers)):
            errs.append(assert_close(got[s][li], want[s][li], f"seq {s} layer {li}", TOL_BF16_ABS, TOL_BF16_REL))
    # the appended rows went through K1 as on every path
    for s in range(case.n_seqs):
        for owner, (Kc, Vc) in caches[s].items():
            p0 = case.pos0[s]
            k_dev, v_dev = kv.read_rows(owner, p0, case.n_tok, seq=s)
            idx = [(p0 + t) % case.rows[owner] for t in range(case.n_tok)]
            assert np.array_equal(v_dev, Vc[idx]), "appended V rows differ"
    kv.close()
    return errs


def test_prefill_qwen3_shape(nncu):
    # BASELINE config 3's layer (32 query heads on 8 KV heads of 128, Q/K
    # RMSNorm, NEOX theta 1e6) at 1024 tokens
    L = [LayerSpec(32, 8, 128, freq_base=1e6, qk_norm=True)]
    case = S.build_case(2, L, n_ctx=1024, n_tok=1024, pos0=0, kv_type=O.KV_BF16)
    check_prefill(nncu, case)


def test_prefill_config3_full(nncu):
    """BASELINE config 3 at its full size: one Qwen3-4B-shaped layer, 2048
    tokens, 32 query heads on 8 KV heads of 128, Q/K RMSNorm, NEOX theta 1e6,
    bf16 cache. The checker is the reference's own compiled kernels where
    they were built (they take a second on the host's cores; the C
    restatement takes about a minute and stands in where they were not)."""
    L = [LayerSpec(32, 8, 128, freq_base=1e6, qk_norm=True)]
    case = S.build_case(2, L, n_ctx=2048, n_tok=2048, pos0=0, kv_type=O.KV_BF16)
    which = "ref" if O.ref() is not None else "oracle"
    (e_abs, e_rel), = check_prefill(nncu, case, which)
    print(f"config 3 prefill vs {which}: max-abs {e_abs:.3e}, rel-L2 {e_rel:.3e} "
          f"(bf16 tolerance {TOL_BF16_ABS:g} / {TOL_BF16_REL:g})")


@pytest.mark.parametrize("n_tok,pos0", [(128, 0), (300, 0), (257, 200), (640, 129)])
def test_prefill_ragged_and_continued(nncu, n_tok, pos0):
    # partial last query tile; a prefill continuing after cached positions
    L = [LayerSpec(8, 2, 128, freq_base=1e4, qk_norm=True)]
    case = S.build_case(20 + n_tok + pos0, L, n_ctx=pos0 + n_tok, n_tok=n_tok, pos0=pos0, kv_type=O.KV_BF16,
                        n_batch=n_tok)
    check_prefill(nncu, case)


def test_prefill_window_softcap_norm_rope(nncu):
    # a sliding layer over a full buffer (ring sizing leaves it whole), soft-cap, NORM RoPE
    L = [LayerSpec(8, 4, 128, window=100, freq_base=1e4, softcap=30.0, rope_mode=O.ROPE_NORM, qk_norm=True)]
    case = S.build_case(31, L, n_ctx=700, n_tok=500, pos0=0, kv_type=O.KV_BF16, n_batch=512)
    assert case.rows[0] >= 700  # not a ring: the tensor-core path takes it
    check_prefill(nncu, case)


def test_prefill_qwen35_gate(nncu):
    # the output gate applied in the tensor-core prefill's output write
    L = [LayerSpec(8, 2, 128, freq_base=1e7, n_rot=64, qk_norm=True, gated=True)]
    case = S.build_case(33, L, n_ctx=384, n_tok=384, pos0=0, kv_type=O.KV_BF16)
    check_prefill(nncu, case)

