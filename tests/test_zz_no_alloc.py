"""nncu_attention_noalloc -- the entry point for callers that cannot let the
library allocate device memory (a host whose device memory belongs to its own
arena or caching allocator; a latency-critical loop that must not stall on the
allocator) -- against the allocating path, through the C ABI.

The cache here is the caller's own memory (a torch tensor laid out
[n_kv][rows][head_dim]); the scratch is the library's fixed device array,
shared by every call. Two decode steps in a row use it, so the second one
also checks that what the first one left behind does not leak into it.

Further cases cover bf16 and f16 caches, several KV heads, a verify block
and a batch long enough that K1 appends first, each against the checker as
well as the allocating path, and nncu_noalloc_check, which reads the shared
array's error word without allocating.

This file is collected last on purpose: if it fails, a run that stops at the
first failure has already run every other test.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from oracle import scenarios as S
from oracle.scenarios import LayerSpec

from gpu_helpers import assert_close, make_cache

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


def _caller_cache(torch, case, layer, rows):
    """The caller's own cache for one layer of sequence 0: [n_kv][rows][D] of
    the cache type's bits, position p at row p % rows, holding the case's
    past rows."""
    L = case.layers[layer]
    inp = case.inputs[0][layer]
    dt = torch.float32 if case.kv_type == O.KV_F32 else torch.int16
    kc = torch.zeros(L.n_kv, rows, L.head_dim, dtype=dt, device="cuda")
    vc = torch.zeros_like(kc)
    n = inp.past_k.shape[0]
    if n:
        r = torch.from_numpy((inp.keep0 + np.arange(n)) % rows).cuda()
        for dst, src in ((kc, inp.past_k), (vc, inp.past_v)):
            bits = O.narrow(src, case.kv_type)
            bits = bits.view(np.int16) if bits.dtype == np.uint16 else bits
            t = torch.from_numpy(np.ascontiguousarray(bits)).cuda().view(n, L.n_kv, L.head_dim).transpose(0, 1)
            dst[:, r] = t
    return kc, vc


# (n_head, n_kv, head_dim, window, kv_type, n_tok): a bf16 sliding layer over
# two KV heads; a Llama-shaped f16 layer of 8 KV heads of 64; a Gemma-3-4B
# verify block on f16; and 8 new tokens of head_dim 256 -- more than the
# attention kernel appends itself, so K1 runs first and the attention kernel
# is its programmatic dependent.
WIDE = [(8, 2, 128, 300, O.KV_BF16, 1), (32, 8, 64, 0, O.KV_F16, 1), (8, 4, 256, 1024, O.KV_F16, 4),
        (4, 1, 256, 0, O.KV_F32, 8)]


@pytest.mark.parametrize("n_head,n_kv,D,window,kv_type,n_tok", WIDE)
def test_noalloc_shapes_against_the_checker(nncu, torch_cuda, n_head, n_kv, D, window, kv_type, n_tok):
    """The no-allocation call against the checker and against the allocating
    call on the same inputs, for each cache type, several KV heads, a verify
    block and the K1 path; then nncu_noalloc_check reports no timeout."""
    N, torch = nncu, torch_cuda
    layer = LayerSpec(n_head, n_kv, D, window=window, freq_base=1e4, qk_norm=True)
    pos0 = 2000
    case = S.build_case(910 + D + n_tok, [layer], n_ctx=pos0 + n_tok, n_tok=n_tok, pos0=pos0, kv_type=kv_type,
                        n_batch=n_tok)
    want, _ = S.run_checker(case, "oracle")
    inp = case.inputs[0][0]
    kv = make_cache(N, case)
    alloc = kv.attention(0, N.params(**case.params_dict(0, 0)), inp.q, inp.k, inp.v)
    kv.close()

    rows = -(-case.rows[0] // 256) * 256
    kc, vc = _caller_cache(torch, case, 0, rows)
    dq, dk, dv = (torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (inp.q, inp.k, inp.v))
    qg, kg = (torch.from_numpy(a).cuda() for a in (inp.q_gamma, inp.k_gamma))
    out = torch.full((n_tok, n_head * D), float("nan"), device="cuda")
    d = case.params_dict(0, 0)
    d.update(q_gamma=qg.data_ptr(), k_gamma=kg.data_ptr())
    torch.cuda.synchronize()
    before = N.launch_count()
    N.attention_noalloc(N.params(**d), dq, dk, dv, out, kc, vc, kv_type, rows)
    N.noalloc_check()
    assert N.launch_count() > before
    got = out.cpu().numpy()
    assert_close(got, want[0][0], "no-allocation call vs the checker")
    assert_close(got, alloc, "no-allocation call vs nncu_attention", 1e-5, 1e-5)


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
