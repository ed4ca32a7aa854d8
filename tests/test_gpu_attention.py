"""Parity of the CUDA attention path (norm + RoPE + append: K1; split-KV
attention with its in-kernel merge: K2+K3) with the checker, through the
C ABI. Tolerance (north_star): max-abs 2e-3 and relative-L2 1e-3 for fp32 and
fp16 caches; fp32 caches are also held to 1e-5, which any indexing or
masking mistake would break."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from oracle import scenarios as S
from oracle.scenarios import LayerSpec

from golden import cases as G
from gpu_helpers import assert_close, make_cache, run_product

pytestmark = pytest.mark.gpu

GOLDEN = np.load(__import__("os").path.join(__import__("os").path.dirname(__file__), "golden", "golden.npz"))


def check_case(N, case, tight=None, batch=False, per_layer=False):
    want, caches = S.run_checker(case, "oracle")
    got, kv = run_product(N, case, batch=batch, per_layer=per_layer)
    if tight is None:
        tight = case.kv_type == O.KV_F32
    for s in range(case.n_seqs):
        for li in range(len(case.layers)):
            assert_close(got[s][li], want[s][li], f"seq {s} layer {li}")
            if tight:
                assert_close(got[s][li], want[s][li], f"seq {s} layer {li} (fp32, tight)", 1e-5, 1e-5)
    # the appended rows: V is a plain rounding (bit-exact), K went through norm + RoPE
    for s in range(case.n_seqs):
        for owner, (Kc, Vc) in caches[s].items():
            if case.layers[owner].kv_layer not in (None, owner):
                continue
            p0 = case.pos0[s]
            rows = case.rows[owner]
            k_dev, v_dev = kv.read_rows(owner, p0, case.n_tok, seq=s) if case.causal else kv.read_rows(owner, 0, case.n_tok, seq=s)
            idx = [(p0 + t) % rows for t in range(case.n_tok)] if case.causal else list(range(case.n_tok))
            if not case.causal and owner != len(case.layers) - 1:
                continue  # a bidirectional model's shared buffer holds the last layer's rows
            if not case.layers[owner].v_rmsnorm:
                assert np.array_equal(v_dev, Vc[idx]), f"appended V rows differ (seq {s}, layer {owner})"
            kd = O.widen(k_dev, case.kv_type).astype(np.float64)
            kw = O.widen(Kc[idx], case.kv_type).astype(np.float64)
            step, floor = {O.KV_F32: (2.0 ** -20, 1.0), O.KV_BF16: (2.0 ** -7, 1e-2), O.KV_F16: (2.0 ** -10, 1e-2)}[
                case.kv_type]
            assert np.all(np.abs(kd - kw) <= step * np.maximum(np.abs(kw), floor)), f"appended K rows (seq {s})"
    kv.close()
    return got


@pytest.mark.parametrize("name", sorted(G.all_cases().keys()))
def test_golden_cases(nncu, name):
    case = G.all_cases()[name]
    got = check_case(nncu, case)
    # and straight against the reference's own outputs
    for s in range(case.n_seqs):
        for li in range(len(case.layers)):
            key = f"{name}.out.{s}.{li}"
            if key in GOLDEN.files:
                assert_close(got[s][li], GOLDEN[key], f"{key} vs the reference")


@pytest.mark.parametrize("name", ["cfg2_stack_f32", "cfg4_verify_bf16", "window_partial_rope_f32"])
def test_batch_call_matches(nncu, name):
    check_case(nncu, G.all_cases()[name], batch=True)


def test_cfg4_verify_f16(nncu):
    g34 = [LayerSpec(8, 4, 256, window=1024, freq_base=1e4, qk_norm=True),
           LayerSpec(8, 4, 256, window=0, freq_base=1e6, qk_norm=True)]
    case = S.build_case(3, g34, n_ctx=4096, n_tok=4, pos0=[2000, 3100, 4092], kv_type=O.KV_F16)
    check_case(nncu, case)


def test_cfg4_verify_f16_full_context(nncu):
    """BASELINE config 4 at its real context: 32768 cached fp16 keys per
    sequence, 4 draft tokens at 32768..32771 (a 4-query causal block), 8
    query heads on 4 KV heads of 256, Q/K RMSNorm; one window-1024 layer (a
    1280-row ring) and one global layer; 2 of the 16 sequences, each layer
    submitted once for both sequences as the benchmark does."""
    g34 = [LayerSpec(8, 4, 256, window=1024, freq_base=1e4, qk_norm=True),
           LayerSpec(8, 4, 256, window=0, freq_base=1e6, qk_norm=True)]
    case = S.build_case(3, g34, n_ctx=32772, n_tok=4, pos0=[32768, 32768], kv_type=O.KV_F16)
    assert case.rows == [1280, 32772]
    check_case(nncu, case, per_layer=True)


def test_gate_cuda_cores_f32(nncu):
    # the output gate in the CUDA-core kernel's direct write and in its merge of pieces
    L = [LayerSpec(4, 1, 256, freq_base=1e6, qk_norm=True, gated=True)]
    case = S.build_case(1500, L, n_ctx=6000, n_tok=1, pos0=5000, kv_type=O.KV_F32, n_batch=1)
    check_case(nncu, case)
    case = S.build_case(1501, L, n_ctx=300, n_tok=1, pos0=200, kv_type=O.KV_F32, n_batch=1)
    check_case(nncu, case)


def test_cfg5_long_f16_reduced(nncu):
    case = S.build_case(4, [LayerSpec(32, 8, 64, freq_base=5e5, rope_mode=O.ROPE_NORM)], n_ctx=16384 + 16,
                        n_tok=1, pos0=16384, kv_type=O.KV_F16)
    check_case(nncu, case)


@pytest.mark.parametrize("D", [64, 128, 256, 512])
@pytest.mark.parametrize("kv_type", [O.KV_F32, O.KV_BF16, O.KV_F16])
@pytest.mark.parametrize("G_,n_tok", [(1, 1), (4, 1), (2, 3), (8, 2)])
def test_shapes_and_types(nncu, D, kv_type, G_, n_tok):
    # spans that start and end inside tiles and blocks, two KV heads
    n_kv = 2
    L = [LayerSpec(G_ * n_kv, n_kv, D, freq_base=1e4, qk_norm=(D != 512))]
    case = S.build_case(100 + D + G_, L, n_ctx=700, n_tok=n_tok, pos0=[257, 3], kv_type=kv_type)
    check_case(nncu, case)


@pytest.mark.parametrize("pos0", [0, 1, 15, 16, 255, 256, 511])
def test_span_edges(nncu, pos0):
    L = [LayerSpec(8, 2, 128, freq_base=1e6), LayerSpec(8, 2, 128, window=100, freq_base=1e4)]
    case = S.build_case(200 + pos0, L, n_ctx=1024, n_tok=2, pos0=pos0, kv_type=O.KV_F32)
    check_case(nncu, case)


def test_softcap_and_norm_rope(nncu):
    L = [LayerSpec(8, 2, 256, freq_base=1e4, rope_mode=O.ROPE_NORM, softcap=50.0, qk_norm=True),
         LayerSpec(8, 2, 256, freq_base=1e4, softcap=20.0, n_rot=128, v_rmsnorm=True, scale=1.0)]
    case = S.build_case(300, L, n_ctx=900, n_tok=3, pos0=800, kv_type=O.KV_BF16)
    check_case(nncu, case)


def test_config1_full(nncu):
    case = S.build_case(0, [LayerSpec(32, 8, 64, freq_base=5e5, rope_mode=O.ROPE_NORM)], n_ctx=1025, n_tok=1,
                        pos0=1024, kv_type=O.KV_F32, rotate_past=True)
    check_case(nncu, case)


def test_config2_full(nncu):
    layers = [LayerSpec(4, 1, 256, window=0 if (li + 1) % 6 == 0 else 512, freq_base=1e6 if (li + 1) % 6 == 0 else 1e4,
                        qk_norm=True) for li in range(26)]
    case = S.build_case(1, layers, n_ctx=4097, n_tok=1, pos0=4096, kv_type=O.KV_F32, n_batch=1)
    check_case(nncu, case, batch=True)


def test_config5_full_f16(nncu):
    case = S.build_case(4, [LayerSpec(32, 8, 64, freq_base=5e5, rope_mode=O.ROPE_NORM)], n_ctx=131073, n_tok=1,
                        pos0=131072, kv_type=O.KV_F16)
    check_case(nncu, case)


def test_verify_rows_match_single_decodes(nncu):
    """tests.cpp:2634-2663 (decode == batch) on the device: 3 tokens in one call
    give what 3 one-token calls give, to within float rounding."""
    L = [LayerSpec(8, 2, 128, freq_base=1e6, qk_norm=True)]
    case = S.build_case(400, L, n_ctx=1200, n_tok=3, pos0=1100, kv_type=O.KV_F32)
    got_batch, kv = run_product(nncu, case)
    kv.close()
    kv = make_cache(nncu, case)
    inp = case.inputs[0][0]
    rows = []
    for t in range(3):
        d = case.params_dict(0, 0)
        d.update(n_tok=1, pos0=1100 + t, n_seq=1101 + t)
        p = nncu.params(**d)
        rows.append(kv.attention(0, p, inp.q[t:t + 1], inp.k[t:t + 1], inp.v[t:t + 1])[0])
    kv.close()
    assert np.abs(np.stack(rows) - got_batch[0][0]).max() <= 1e-6


def test_repeatable_bits(nncu):
    L = [LayerSpec(4, 1, 256, freq_base=1e6, qk_norm=True)]
    case = S.build_case(500, L, n_ctx=5000, n_tok=1, pos0=4000, kv_type=O.KV_F32)
    a, kv = run_product(nncu, case)
    kv.close()
    b, kv = run_product(nncu, case)
    kv.close()
    assert np.array_equal(a[0][0], b[0][0])


def test_sliding_ring_through_wraps_and_rewind(nncu):
    """tests.cpp:2598-2630 on the device: a sliding layer kept as a ring of 256
    rows (window 40, batch 16) attends exactly as over a full buffer, through
    many wraps, a step back, and a refused step back."""
    N = nncu
    layers = [LayerSpec(4, 2, 64, window=40, freq_base=1e4, qk_norm=True),
              LayerSpec(4, 2, 64, window=0, freq_base=1e6, qk_norm=True)]
    kv = N.KVCache([(2, 64, 40, 0), (2, 64, 0, 1)], n_ctx=1200, n_batch=16, kv_type=O.KV_BF16)
    assert kv.layer_info(0).rows == 256 and kv.layer_info(0).window == 40 and kv.state().max_rewind == 216
    full = {li: (np.zeros((1200, 128), np.uint16), np.zeros((1200, 128), np.uint16)) for li in (0, 1)}
    rng = O.Rng(600)
    gam = {li: (rng.normal(64, 1.0, 0.1), rng.normal(64, 1.0, 0.1)) for li in (0, 1)}

    def forward(p0, p1, step):
        for pos in range(p0, p1, step):
            n = min(step, p1 - pos)
            for li, L in enumerate(layers):
                q, k, v = rng.normal(n * 256).reshape(n, 256), rng.normal(n * 128).reshape(n, 128), \
                    rng.normal(n * 128).reshape(n, 128)
                d = dict(n_tok=n, pos0=pos, n_seq=pos + n, n_head=4, n_kv=2, head_dim=64, freq_base=L.freq_base,
                         q_gamma=gam[li][0], k_gamma=gam[li][1], window=L.window)
                got = kv.attention(li, N.params(**d), q, k, v)
                Kc, Vc = full[li]
                want, _, _ = O.attention_forward(O.params(**d), q, k, v, Kc, Vc, O.KV_BF16, 1200)
                assert_close(got, want, f"positions {pos}..{pos + n - 1}, layer {li}")
            kv.commit(pos, n)

    forward(0, 700, 16)
    forward(700, 720, 1)
    assert kv.rewind(705)
    forward(705, 760, 16)
    assert not kv.rewind(760 - 217) and kv.state().cur_pos == 760
    assert kv.rewind(760 - 216) and kv.rewind(0)
    forward(0, 300, 16)
    kv.close()


def test_registered_host_buffers_match_staging(nncu):
    """nncu_host_register: a batch whose host buffers are all registered moves
    them with the gather and scatter kernels through the GPU's mapping of the
    memory; its outputs equal, bit for bit, those of the same batch through the
    pinned staging copies (the same kernels on the same inputs), and the
    checker's within the fp16 bar. A Gemma-3-4B-shaped verify layer (4 draft
    tokens, 8/4 heads of 256, f16 cache) for 12 sequences at context 1500."""
    N = nncu
    L = [LayerSpec(8, 4, 256, window=1024, freq_base=1e4, qk_norm=True)]
    case = S.build_case(77, L, n_ctx=1504, n_tok=4, pos0=[1500] * 12, kv_type=O.KV_F16)
    want, _ = S.run_checker(case, "oracle")

    def run(register):
        # every host buffer a view of one arena (registration pins whole pages)
        arena = np.zeros(1 << 20, np.float32)
        used = [(-arena.ctypes.data // 4) % 4]

        def place(x):
            v = arena[used[0]:used[0] + x.size].reshape(x.shape)
            v[...] = x
            used[0] += (x.size + 3) // 4 * 4
            return v

        kv = make_cache(N, case)
        jobs, outs = [], []
        for s in range(case.n_seqs):
            inp = case.inputs[s][0]
            d = case.params_dict(0, s)
            q, k, v = (place(x) for x in (inp.q, inp.k, inp.v))
            d.update(q_gamma=place(d["q_gamma"]), k_gamma=place(d["k_gamma"]))
            out = place(np.zeros((case.n_tok, 8 * 256), np.float32))
            jobs.append(N.job(0, N.params(**d), q, k, v, out, seq=s))
            outs.append(out)
        if register:
            N.host_register(arena)
        launches = N.launch_count()
        try:
            kv.attention_batch(jobs)
            launches = N.launch_count() - launches
        finally:
            if register:
                N.host_unregister(arena)
            kv.close()
        return [o.copy() for o in outs], launches

    staged, n_staged = run(False)
    mapped, n_mapped = run(True)
    assert n_mapped == n_staged + 2  # the gather and the scatter
    for s in range(case.n_seqs):
        assert np.array_equal(mapped[s], staged[s]), f"sequence {s}"
        assert_close(mapped[s], want[s][0], f"sequence {s}")
    with pytest.raises(N.NnncError):
        N.host_unregister(staged[0])  # never registered
    arena = np.zeros(4096, np.float32)
    N.host_register(arena)
    try:
        with pytest.raises(N.NnncError):
            N.host_register(arena[1024:])  # overlaps a registered range
    finally:
        N.host_unregister(arena)


@pytest.mark.parametrize("kv_type,one_by_one", [(O.KV_F32, False), (O.KV_BF16, False), (O.KV_BF16, True)])
def test_device_pointer_batch_matches_host(nncu, torch_cuda, kv_type, one_by_one):
    # a bf16 cache with 4 query rows per KV head takes the tensor-core kernel;
    # one job alone is a table small enough to travel inline with a launch
    torch = torch_cuda
    N = nncu
    layers = [LayerSpec(4, 1, 256, window=512, freq_base=1e4, qk_norm=True),
              LayerSpec(4, 1, 256, window=0, freq_base=1e6, qk_norm=True)]
    case = S.build_case(700, layers, n_ctx=2048, n_tok=1, pos0=1500, kv_type=kv_type, n_batch=1)
    want, kv_h = run_product(N, case)
    kv_h.close()
    kv = make_cache(N, case)
    st = torch.cuda.Stream()
    keep, outs, jobs = [], [], []
    for li in range(2):
        inp = case.inputs[0][li]
        t = {k: torch.from_numpy(np.ascontiguousarray(getattr(inp, k))).cuda() for k in ("q", "k", "v", "q_gamma", "k_gamma")}
        d = case.params_dict(li, 0)
        d.update(q_gamma=t["q_gamma"].data_ptr(), k_gamma=t["k_gamma"].data_ptr())
        out = torch.empty(1, 4 * 256, device="cuda")
        jobs.append(N.job(li, N.params(**d), t["q"], t["k"], t["v"], out))
        keep.append(t)
        outs.append(out)
    torch.cuda.synchronize()
    if one_by_one:
        for j in jobs:
            kv.attention_batch_dev([j], st)
    else:
        kv.attention_batch_dev(jobs, st)
    kv.sync(st)
    for li in range(2):
        assert np.array_equal(outs[li].cpu().numpy(), want[0][li])
    kv.close()


def test_errors_are_statuses(nncu):
    N = nncu
    kv = N.KVCache([(2, 64, 40, 0), (2, 64, 0, 1)], n_ctx=300, n_batch=4, kv_type=O.KV_F32)
    q = np.zeros((1, 256), np.float32)
    k = np.zeros((1, 128), np.float32)

    def call(layer=1, **kw):
        d = dict(n_tok=1, pos0=0, n_head=4, n_kv=2, head_dim=64, window=0)
        d.update(kw)
        n = d["n_tok"]
        return kv.attention(layer, N.params(**d), np.zeros((n, 4 * d["head_dim"]), np.float32),
                            np.zeros((n, 2 * d["head_dim"]), np.float32), np.zeros((n, 2 * d["head_dim"]), np.float32))

    with pytest.raises(N.NnncError) as e:
        call(pos0=300)
    assert e.value.status == N.ERR_CONTEXT_FULL
    with pytest.raises(N.NnncError) as e:
        call(n_tok=5)
    assert e.value.status == N.ERR_INVALID_ARGUMENT
    with pytest.raises(N.NnncError) as e:
        call(head_dim=32)
    assert e.value.status == N.ERR_INVALID_ARGUMENT
    with pytest.raises(N.NnncError) as e:
        call(layer=0, window=64)  # a ring of window 40 cannot serve window 64
    assert e.value.status == N.ERR_INVALID_ARGUMENT
    with pytest.raises(N.NnncError) as e:
        call(layer=1, reuse_kv=1)
    assert e.value.status == N.ERR_INVALID_ARGUMENT
    with pytest.raises(N.NnncError) as e:
        call(n_head=3)
    assert e.value.status == N.ERR_INVALID_ARGUMENT
    assert not kv.rewind(5)  # beyond cur_pos
    out = call(layer=1)  # and the cache still works
    assert out.shape == (1, 256) and np.all(out == 0.0)
    del q, k
    kv.close()


def test_misaligned_pointers_are_refused(nncu, torch_cuda):
    """Every pointer the kernels bulk-copy from or write with 16-byte stores
    is checked on the host: a misaligned k, out or cache (each inside a
    buffer large enough for the call) fails with NNCU_ERR_INVALID_ARGUMENT
    and nothing is launched."""
    N, torch = nncu, torch_cuda
    D, n_head, n_kv = 256, 4, 1
    kv = N.KVCache([(n_kv, D, 0, 0)], n_ctx=512, n_batch=1, kv_type=O.KV_F32)
    pad = 4  # floats: 16 bytes of room for a 4-byte offset

    def buf(n):
        return torch.zeros(n + pad, device="cuda")

    q, k, v, out = buf(n_head * D), buf(n_kv * D), buf(n_kv * D), buf(n_head * D)
    p = N.params(n_tok=1, pos0=100, n_head=n_head, n_kv=n_kv, head_dim=D)
    good = dict(q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), out=out.data_ptr())
    torch.cuda.synchronize()
    for name in ("k", "out", "q", "v"):
        ptrs = dict(good)
        ptrs[name] += 4  # one float past a 16-byte boundary, still inside its buffer
        before = N.launch_count()
        with pytest.raises(N.NnncError) as e:
            kv.attention_batch_dev([N.job(0, p, ptrs["q"], ptrs["k"], ptrs["v"], ptrs["out"])])
        assert e.value.status == N.ERR_INVALID_ARGUMENT and name in str(e.value), str(e.value)
        assert N.launch_count() == before
    kv.attention_batch_dev([N.job(0, p, good["q"], good["k"], good["v"], good["out"])])  # and the aligned call runs
    kv.sync()
    kv.close()
    # a caller-owned cache (the no-allocation call) whose base is off by 4 bytes
    rows = 512
    k_cache = torch.zeros(n_kv * rows * D + pad, device="cuda")
    v_cache = torch.zeros(n_kv * rows * D + pad, device="cuda")
    for which in ("k_cache", "v_cache"):
        kc = k_cache.data_ptr() + (4 if which == "k_cache" else 0)
        vc = v_cache.data_ptr() + (4 if which == "v_cache" else 0)
        before = N.launch_count()
        with pytest.raises(N.NnncError) as e:
            N.attention_noalloc(p, good["q"], good["k"], good["v"], good["out"], kc, vc, O.KV_F32, rows)
        assert e.value.status == N.ERR_INVALID_ARGUMENT and which in str(e.value), str(e.value)
        assert N.launch_count() == before
    torch.cuda.synchronize()
