"""nncu_attention_noalloc -- the entry point for callers that cannot let the
library allocate device memory (a host whose device memory belongs to its own
arena or caching allocator; a latency-critical loop that must not stall on the
allocator) -- against the allocating path, through the C ABI.

The cache here is the caller's own memory (a torch tensor laid out
[n_kv][rows][head_dim]); the scratch is the library's fixed device array,
shared by every call. Two decode steps in a row use it, so the second one
also checks that what the first one left behind does not leak into it.

This file is collected last on purpose: if it fails, a run that stops at the
first failure has already run every other test.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from oracle import scenarios as S
from oracle.scenarios import LayerSpec

from gpu_helpers import assert_close

pytestmark = pytest.mark.gpu


def test_noalloc_matches_the_allocating_call_twice(nncu, torch_cuda):
    N, torch = nncu, torch_cuda
    # one global Gemma-3-1B-shaped layer: 4 query heads, 1 KV head of 256, Q/K norm, F32 cache
    layer = LayerSpec(4, 1, 256, freq_base=1e6, qk_norm=True)
    D, n_kv = 256, 1
    case = S.build_case(900, [layer], n_ctx=1300, n_tok=1, pos0=1000, kv_type=O.KV_F32, n_batch=1)
    inp = case.inputs[0][0]

    # the allocating path's cache
    kv = N.KVCache(case.layer_descs(), n_ctx=1300, n_batch=1, kv_type=O.KV_F32)
    kv.write_rows(0, 0, inp.past_k, inp.past_v)

    # the caller's own cache: [n_kv][rows][D], rows a multiple of 256, holding the same rows
    rows = 1536
    k_cache = torch.zeros(n_kv, rows, D, device="cuda")
    v_cache = torch.zeros(n_kv, rows, D, device="cuda")
    k_cache[0, :1000] = torch.from_numpy(inp.past_k.reshape(1000, D)).cuda()
    v_cache[0, :1000] = torch.from_numpy(inp.past_v.reshape(1000, D)).cuda()
    qg = torch.from_numpy(inp.q_gamma).cuda()
    kg = torch.from_numpy(inp.k_gamma).cuda()

    rng = O.Rng(901)
    for step in range(2):
        pos = 1000 + step
        q = rng.normal(4 * D).reshape(1, 4 * D)
        k = rng.normal(D).reshape(1, D)
        v = rng.normal(D).reshape(1, D)
        d = case.params_dict(0, 0)
        d.update(pos0=pos, n_seq=pos + 1, q_gamma=inp.q_gamma, k_gamma=inp.k_gamma)
        want = kv.attention(0, N.params(**d), q, k, v)
        kv.commit(pos, 1)

        dq, dk, dv = (torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (q, k, v))
        out = torch.full((1, 4 * D), float("nan"), device="cuda")
        d.update(q_gamma=qg.data_ptr(), k_gamma=kg.data_ptr())
        torch.cuda.synchronize()
        N.attention_noalloc(N.params(**d), dq, dk, dv, out, k_cache, v_cache, O.KV_F32, rows)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert_close(got, want, f"step {step}: no-allocation call vs nncu_attention")
        # and the row it appended is the allocating path's row
        k_row, v_row = kv.read_rows(0, pos, 1)
        assert np.array_equal(v_cache[0, pos].cpu().numpy(), v_row[0])
        assert np.allclose(k_cache[0, pos].cpu().numpy(), k_row[0], rtol=1e-6, atol=1e-6)
    kv.close()


def test_noalloc_refuses_what_does_not_fit(nncu, torch_cuda):
    N, torch = nncu, torch_cuda
    D, rows = 256, 4096
    k_cache = torch.zeros(8, rows, D, device="cuda")
    v_cache = torch.zeros_like(k_cache)
    # 4096 tokens are beyond what the entry point takes (decode and verify). The
    # buffers have the call's full sizes all the same, so that nothing could be
    # read or written out of bounds even if the call were accepted.
    n_tok, n_head, n_kv = 4096, 64, 8
    q = torch.zeros(n_tok, n_head * D, device="cuda")
    out = torch.zeros_like(q)
    kv_new = torch.zeros(n_tok, n_kv * D, device="cuda")
    p = N.params(n_tok=n_tok, pos0=0, n_head=n_head, n_kv=n_kv, head_dim=D)
    with pytest.raises(N.NnncError) as e:
        N.attention_noalloc(p, q, kv_new, kv_new, out, k_cache, v_cache, O.KV_F32, rows)
    assert e.value.status == N.ERR_INVALID_ARGUMENT and "tokens" in str(e.value)
    # a cache whose rows are not whole 256-key blocks is refused too (full-size buffers again)
    p = N.params(n_tok=1, pos0=10, n_head=4, n_kv=1, head_dim=D)
    q1 = torch.zeros(1, 4 * D, device="cuda")
    out1 = torch.zeros_like(q1)
    kv1 = torch.zeros(1, D, device="cuda")
    with pytest.raises(N.NnncError) as e:
        N.attention_noalloc(p, q1, kv1, kv1, out1, k_cache, v_cache, O.KV_F32, 1000)
    assert e.value.status == N.ERR_INVALID_ARGUMENT
    torch.cuda.synchronize()
