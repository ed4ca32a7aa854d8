"""Decode and verify on the tensor cores (k_decode_tc.cu: tcgen05 S^T = K Q^T
and O^T = V^T P^T with q and the weights split into high and low 16-bit
halves) against the checker and against the CUDA-core kernel, through the C
ABI. A 16-bit cache with three or more query rows per KV head takes this
path; nncu_kv_set_tensor_cores(0) keeps it on the CUDA-core kernel for the
comparison. Tolerance: north_star's max-abs 2e-3 and relative-L2 1e-3; the
two kernels agree far closer than that (both accumulate in fp32)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from oracle import scenarios as S
from oracle.scenarios import LayerSpec

from gpu_helpers import assert_close, make_cache, run_product

pytestmark = pytest.mark.gpu


def both_kernels(N, case):
    want, _ = S.run_checker(case, "oracle")
    got_tc, kv = run_product(N, case, per_layer=True)
    kv.close()
    kv = make_cache(N, case)
    kv.set_tensor_cores(False)
    got_cc, kv = run_product(N, case, kv=kv, per_layer=True)
    kv.close()
    for s in range(case.n_seqs):
        for li in range(len(case.layers)):
            assert_close(got_tc[s][li], want[s][li], f"tensor cores, seq {s} layer {li}")
            # bf16 halves keep 16 bits of q and of the weights (f16 halves 22):
            # at scale 1.0 that moves a score by ~1e-4 against the CUDA cores' fp32
            tol = 2e-5 if case.kv_type == O.KV_F16 else 2e-4
            assert_close(got_tc[s][li], got_cc[s][li], f"tensor cores vs CUDA cores, seq {s} layer {li}", tol, tol)
    return got_tc


@pytest.mark.parametrize("kv_type", [O.KV_F16, O.KV_BF16])
def test_tc_smallest(nncu, kv_type):
    # one KV head of 64, four query heads, one token: a single tile of 256 keys
    case = S.build_case(1000, [LayerSpec(4, 1, 64, freq_base=1e4)], n_ctx=200, n_tok=1, pos0=150, kv_type=kv_type)
    both_kernels(nncu, case)


@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("kv_type", [O.KV_F16, O.KV_BF16])
@pytest.mark.parametrize("G_,n_tok", [(4, 1), (2, 4), (8, 1), (4, 4), (3, 1)])
def test_tc_shapes(nncu, D, kv_type, G_, n_tok):
    # spans starting and ending inside tiles, two KV heads, several row
    # groups where G * n_tok > 16, windowed and global layers, two sequences
    L = [LayerSpec(G_ * 2, 2, D, window=700, freq_base=1e4, qk_norm=True),
         LayerSpec(G_ * 2, 2, D, window=0, freq_base=1e6, qk_norm=True)]
    case = S.build_case(1100 + D + 10 * G_ + n_tok, L, n_ctx=3000, n_tok=n_tok, pos0=[2900, 1333], kv_type=kv_type)
    both_kernels(nncu, case)


def test_tc_softcap_norm_rope_freq_factors(nncu):
    ff = (1.0 + np.arange(32, dtype=np.float32) / 8.0).astype(np.float32)
    L = [LayerSpec(8, 2, 128, freq_base=1e4, softcap=30.0, rope_mode=O.ROPE_NORM, qk_norm=True),
         LayerSpec(8, 2, 128, freq_base=1e4, n_rot=64, freq_factors=ff, v_rmsnorm=True, scale=1.0)]
    case = S.build_case(1200, L, n_ctx=2000, n_tok=2, pos0=1900, kv_type=O.KV_BF16)
    both_kernels(nncu, case)


def test_tc_long_chunks(nncu):
    # enough tiles per SM that segments are cut into many chunks, merged in order
    case = S.build_case(1300, [LayerSpec(32, 8, 64, freq_base=5e5, rope_mode=O.ROPE_NORM)], n_ctx=40000, n_tok=1,
                        pos0=39990, kv_type=O.KV_F16)
    both_kernels(nncu, case)


@pytest.mark.parametrize("kv_type", [O.KV_F16, O.KV_BF16])
def test_tc_qwen35_gate(nncu, kv_type):
    # Qwen3.5's output gate (model.cpp:1759-1760) on both kernels: a verify
    # block, partial rotation, Q/K norm
    L = [LayerSpec(8, 2, 256, freq_base=1e7, n_rot=64, qk_norm=True, gated=True),
         LayerSpec(8, 2, 256, window=300, freq_base=1e7, n_rot=64, qk_norm=True, gated=True)]
    case = S.build_case(1400, L, n_ctx=2200, n_tok=2, pos0=[2100, 700], kv_type=kv_type)
    both_kernels(nncu, case)

