"""The checker itself, on the CPU: the C restatement (oracle/oracle.c) against
the reference's own known answers and tests (src/appnnc/tests.cpp), against
the golden vectors in tests/golden/, and -- where oracle/_ref was built --
against the reference's compiled kernels on the same inputs."""
from __future__ import annotations

import os

import numpy as np
import pytest

import oracle as O
from oracle import scenarios as S

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden", "golden.npz")


def close(a, b, tol):
    """tests.cpp:46-51: |a - b| <= tol * max(|a|, |b|, 1)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.all(np.abs(a - b) <= tol * np.maximum(np.maximum(np.abs(a), np.abs(b)), 1.0))


# ---- known answers (the reference's own tables) ----------------------------------------------

# tests.cpp:1663-1678, test_attn_span: (causal, window, pos, n_seq) -> (first, last)
SPAN_CASES = [
    (True, 0, 5, 10, 0, 5), (True, 3, 5, 10, 3, 5), (True, 0, 5, 5, 0, 4), (True, 3, 5, 5, 3, 4),
    (False, 0, 5, 10, 0, 9), (False, 4, 5, 10, 3, 7), (False, 4, 0, 10, 0, 2), (False, 4, 9, 10, 7, 9),
    (False, 512, 300, 1000, 44, 556),
]


@pytest.mark.parametrize("causal,window,pos,n_seq,first,last", SPAN_CASES)
def test_attn_span_known_answers(causal, window, pos, n_seq, first, last):
    assert O.attn_span(causal, window, pos, n_seq) == (first, last)


def test_softcap_known_answers():
    # tests.cpp:1294-1313
    cap = 30.0
    x = np.array([0.0, 1.0, -1.0, 5.0, -5.0, 30.0, 100.0, -100.0, 1e6], np.float32)
    y = O.softcap(x, cap)
    assert close(y, np.tanh(x.astype(np.float64) / cap) * cap, 1e-5)
    assert np.all(np.abs(y) <= cap + 1e-4)
    assert y[0] == 0.0
    assert cap - 1e-3 <= y[8] <= cap


def test_rope_pos0_identity_and_scalar_reference():
    # tests.cpp:1221-1290
    rng = O.Rng(0x5051)
    x = rng.uniform(8 * 64, -1.0, 1.0)
    assert close(O.rope(x, 8, 64, 64, 0.0, 10000.0), x, 1e-6)
    rng = O.Rng(0x5052)
    H, D, R, pos, base = 4, 64, 32, 17, 1e6
    x = rng.uniform(H * D, -1.0, 1.0)
    got = O.rope(x, H, D, R, float(pos), base)
    ref = x.copy().reshape(H, D)
    half = R // 2
    for i in range(half):
        inv = np.float32(base) ** (-np.float32(2 * i) / np.float32(R))
        th = np.float32(pos) * np.float32(inv)
        c, s = np.cos(th), np.sin(th)
        a, b = ref[:, i].copy(), ref[:, i + half].copy()
        ref[:, i] = c * a - s * b
        ref[:, i + half] = s * a + c * b
    assert close(got, ref.ravel(), 1e-5)
    # lanes past n_rot pass through
    assert np.array_equal(got.reshape(H, D)[:, R:], x.reshape(H, D)[:, R:])


def test_rope_preserves_pair_norms():
    rng = O.Rng(0x5053)
    H, D, R = 2, 16, 16
    x = rng.uniform(H * D, -1.0, 1.0)
    y = O.rope(x, H, D, R, 42.0, 10000.0).reshape(H, D)
    x = x.reshape(H, D)
    h = R // 2
    m0 = x[:, :h] ** 2 + x[:, h:R] ** 2
    m1 = y[:, :h] ** 2 + y[:, h:R] ** 2
    assert np.all(np.abs(m0 - m1) <= 1e-4 * np.maximum(m0, 1e-6))


def test_rmsnorm_scalar_reference():
    # tests.cpp:421-466
    rng = O.Rng(0xCAFE)
    for n in (1536, 2560, 256, 13):
        x = rng.uniform(n, -3.0, 3.0)
        y = O.rmsnorm(x, 1e-6)
        s2 = float(np.sum(x.astype(np.float64) ** 2))
        scale = np.float32(1.0 / np.sqrt(s2 / n + 1e-6))
        assert close(y, x * scale, 1e-5)
        assert abs(np.sqrt(np.mean(y.astype(np.float64) ** 2)) - 1.0) <= 1e-3


def test_bf16_round_trip_rne():
    # tests.cpp:469 onwards: exact values survive; ties go to even
    exact = np.array([0.0, 1.0, -1.0, 2.0, 0.5, -0.5, 1024.0, -2048.0], np.float32)
    assert np.array_equal(O.widen(O.narrow(exact, O.KV_BF16), O.KV_BF16), exact)
    L = O.lib()
    for v in (1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -3.14159, 65504.0, 1e-30):
        assert L.orc_f32_to_bf16(v) == O.f32_to_bf16_bits(np.array([v], np.float32))[0]
    # 1 + 2^-8 is a tie between 1 and 1 + 2^-7: even mantissa wins
    assert O.widen(O.narrow(np.array([1.0 + 2 ** -8], np.float32), O.KV_BF16), O.KV_BF16)[0] == 1.0


def ref_attention(q, K, V, group, hd, scale):
    """tests.cpp:2424-2445: scalar double-precision softmax attention."""
    q = q.reshape(group, hd).astype(np.float64)
    s = (q @ K.astype(np.float64).T) * scale
    p = np.exp(s - s.max(axis=1, keepdims=True))
    return ((p @ V.astype(np.float64)) / p.sum(axis=1, keepdims=True)).ravel()


def attn_blocks_case(rng, bf16, hd):
    """The inputs of tests.cpp:2450-2497 (drawn from mt19937(7) in the test's order)."""
    group, n_kv, n_keys = 3, 2, 600
    kv_stride = n_kv * hd
    q = rng.normal(group * hd)
    K = 2.0 * rng.normal(n_keys * kv_stride)
    V = rng.normal(n_keys * kv_stride)
    kt = O.KV_BF16 if bf16 else O.KV_F32
    return q, O.narrow(K, kt), O.narrow(V, kt), kt, group, n_kv, n_keys, kv_stride


def blocked(q, Kb, Vb, kt, group, kv_stride, hd, which, blocks=(100, 256, 244), kv_h=1):
    scale = 1.0 / np.sqrt(hd)
    k0, acc = 0, None
    for n in blocks:
        part = O.attn_block(q, hd, Kb, Vb, kt, kv_stride, n, hd, group, scale, which=which,
                            k_offset_elems=k0 * kv_stride + kv_h * hd)
        acc = part if acc is None else O.attn_merge(acc, part, hd, group, which=which)
        k0 += n
    return O.attn_finish(acc, hd, group, which=which)


def test_attn_blocks_match_full_softmax():
    # tests.cpp:2450-2497: blocks of 100, 256, 244 keys merged in order == softmax over all 600
    rng = O.Rng(7)
    for bf16 in (False, True):
        for hd in (64, 36):
            q, Kb, Vb, kt, group, n_kv, n_keys, kvs = attn_blocks_case(rng, bf16, hd)
            out = blocked(q, Kb, Vb, kt, group, kvs, hd, "oracle")
            Kf = O.widen(Kb, kt).reshape(n_keys, kvs)[:, hd:2 * hd]
            Vf = O.widen(Vb, kt).reshape(n_keys, kvs)[:, hd:2 * hd]
            ref = ref_attention(q, Kf, Vf, group, hd, 1.0 / np.sqrt(hd))
            assert np.all(np.abs(out - ref) <= 1e-4 * (1.0 + np.abs(ref))), (bf16, hd)


def test_ring_rows_rule():
    # model.cpp:1934: round_up(window + n_batch, 256); tests.cpp:2598-2630 expects 256 for (40, 16)
    assert O.ring_rows(40, 16) == 256
    assert O.ring_rows(512, 1) == 768
    assert O.ring_rows(1024, 4) == 1280
    assert O.ring_rows(240, 16) == 256 and O.ring_rows(241, 16) == 512


# ---- golden vectors (made by tests/golden/make_golden.py from the reference's kernels) -----

from golden import cases as G  # noqa: E402


def test_golden_fixture_inputs_are_reproducible():
    gold = np.load(GOLDEN)
    for name, case in G.all_cases().items():
        assert name + ".in_sha" in gold.files, name
        assert G.inputs_digest(case) == str(gold[name + ".in_sha"]), f"{name}: the seeded inputs changed"


@pytest.mark.parametrize("name", sorted(G.all_cases().keys()))
def test_oracle_matches_golden(name):
    gold = np.load(GOLDEN)
    case = G.all_cases()[name]
    outs, _ = S.run_checker(case, "oracle")
    for s in range(case.n_seqs):
        for li in range(len(case.layers)):
            want = gold[f"{name}.out.{s}.{li}"]
            err_abs, err_rel = S.errors(outs[s][li], want)
            assert err_abs <= 2e-6 and err_rel <= 2e-6, (name, s, li, err_abs, err_rel)


@pytest.mark.parametrize("name", sorted(G.UNIT_CASES))
def test_oracle_units_match_golden(name):
    gold = np.load(GOLDEN)
    got = G.run_unit(name, "oracle")
    want = gold[f"unit.{name}"]
    assert got.shape == want.shape
    assert np.allclose(got, want, rtol=2e-6, atol=2e-6), (name, np.abs(got - want).max())


# ---- live comparison with the reference's compiled kernels (where built) ------------------

needs_ref = pytest.mark.skipif(O.ref() is None, reason="oracle/_ref was not built here")


@needs_ref
def test_attn_blocks_restatement_vs_reference_kernels():
    rng = O.Rng(7)
    for bf16 in (False, True):
        for hd in (64, 36):
            q, Kb, Vb, kt, group, n_kv, n_keys, kvs = attn_blocks_case(rng, bf16, hd)
            a = blocked(q, Kb, Vb, kt, group, kvs, hd, "oracle")
            b = blocked(q, Kb, Vb, kt, group, kvs, hd, "ref")
            assert np.abs(a - b).max() <= 1e-6


@needs_ref
@pytest.mark.parametrize("mode,base,pos,n_rot,ff", [
    (O.ROPE_NEOX, 1e6, 17.0, 32, False), (O.ROPE_NORM, 5e5, 1024.0, 64, False),
    (O.ROPE_NORM, 5e5, 131072.0, 64, False), (O.ROPE_NEOX, 1e4, 4096.0, 256, False),
    (O.ROPE_NEOX, 1e6, 4096.0, 256, True)])
def test_rope_restatement_vs_reference(mode, base, pos, n_rot, ff):
    rng = O.Rng(11)
    D = max(n_rot, 64)
    x = rng.normal(4 * D)
    f = (1.0 + np.abs(rng.normal(n_rot // 2))).astype(np.float32) if ff else None
    a = O.rope(x, 4, D, n_rot, pos, base, mode, f)
    b = O.rope(x, 4, D, n_rot, pos, base, mode, f, which="ref")
    # same recurrence, same libm: equal up to the reference's fused multiply-adds
    assert np.abs(a - b).max() <= 2e-6 * max(1.0, np.abs(b).max())


@needs_ref
def test_rmsnorm_gamma_restatement_vs_reference():
    rng = O.Rng(12)
    for dim in (64, 128, 256, 13):
        x = rng.normal(7 * dim)
        g = rng.normal(dim, 1.0, 0.1)
        a = O.rmsnorm_gamma_multi(x, 7, dim, g, 1e-6)
        b = O.rmsnorm_gamma_multi(x, 7, dim, g, 1e-6, which="ref")
        assert np.abs(a - b).max() <= 1e-6 * max(1.0, np.abs(b).max())


@needs_ref
@pytest.mark.parametrize("name", sorted(G.all_cases().keys()))
def test_restatement_vs_reference_scenarios(name):
    case = G.all_cases()[name]
    if case.kv_type == O.KV_F16:
        pytest.skip("the reference has no F16 cache")
    a, ca = S.run_checker(case, "oracle")
    b, cb = S.run_checker(case, "ref")
    for s in range(case.n_seqs):
        for li in range(len(case.layers)):
            err_abs, err_rel = S.errors(a[s][li], b[s][li])
            assert err_abs <= 2e-6 and err_rel <= 2e-6, (name, s, li, err_abs, err_rel)
        # the appended rows: V rows are a plain rounding (bit-exact); K rows went through norm+RoPE
        for owner, (Ka, Va) in ca[s].items():
            Kb, Vb = cb[s][owner]
            assert np.array_equal(Va, Vb), (name, owner)
            ka = O.widen(Ka, case.kv_type).astype(np.float64)
            kb = O.widen(Kb, case.kv_type).astype(np.float64)
            # a rounding step of the cache type apart at most (fp32: a few ulp of
            # values ~N(0,1), where RoPE's a*c - b*s may cancel)
            step, floor = (2.0 ** -7, 1e-2) if case.kv_type == O.KV_BF16 else (2.0 ** -20, 1.0)
            assert np.all(np.abs(ka - kb) <= step * np.maximum(np.abs(kb), floor)), (name, owner)


# ---- the projections' gemvs: the restatement against the reference's own ----------------------

GEMV_SHAPES = [(1, 32, 1), (8, 64, 1), (64, 128, 3), (256, 256, 2), (512, 512, 1), (1024, 2048, 4)]


def _gemv_inputs(rows, cols, nb, seed):
    rng = np.random.default_rng(seed)
    W = O.f32_to_bf16_bits(rng.uniform(-1, 1, (rows, cols)).astype(np.float32))
    X = rng.uniform(-1, 1, (nb, cols)).astype(np.float32)
    qs8 = rng.integers(-128, 128, (rows, cols), dtype=np.int8)
    sc = O.f32_to_bf16_bits((rng.random((rows, cols // 32)) * 0.02).astype(np.float32))
    qs4 = rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
    bi = O.f32_to_bf16_bits((rng.uniform(-1, 1, (rows, cols // 32)) * 0.1).astype(np.float32))
    return W, X, qs8, sc, qs4, bi


def _close(got, want):
    # the reference's own gemv tests: 1e-3 x max(1, |ref|) (tests.cpp:819-880)
    return np.all(np.abs(got - want) <= 1e-3 * np.maximum(1.0, np.abs(want)))


@needs_ref
@pytest.mark.parametrize("rows,cols,nb", GEMV_SHAPES)
def test_gemv_restatement_matches_reference(rows, cols, nb):
    """nnc_gemv_{bf16w,q8_0,q4_s}_f32x_batch, nnc_block_sums_f32 and
    nnc_gemv_bf16w_argmax_f32x (nn_ops.cpp:1000-1446), compiled from the
    reference's sources, against the plain-C restatement on the shapes of the
    reference's own gemv tests."""
    W, X, qs8, sc, qs4, bi = _gemv_inputs(rows, cols, nb, rows * 7 + cols)
    assert _close(O.gemv_bf16w(W, X), O.gemv_bf16w(W, X, "ref"))
    assert _close(O.gemv_q8_0(qs8, sc, X), O.gemv_q8_0(qs8, sc, X, "ref"))
    xs_ref = np.stack([O.block_sums(x, "ref") for x in X])
    xs = np.stack([O.block_sums(x) for x in X])
    assert np.allclose(xs, xs_ref, rtol=1e-5, atol=1e-5)
    assert _close(O.gemv_q4_s(qs4, sc, bi, X, xs_ref), O.gemv_q4_s(qs4, sc, bi, X, xs_ref, "ref"))
    assert O.gemv_bf16w_argmax(W, X[0]) == O.gemv_bf16w_argmax(W, X[0], "ref")


def test_gemv_restatement_scalar_cases():
    # hand-checkable: one row, one block
    W = O.f32_to_bf16_bits(np.arange(32, dtype=np.float32))
    x = np.ones(32, np.float32)
    assert O.gemv_bf16w(W.reshape(1, 32), x)[0, 0] == sum(range(32))
    qs = np.arange(-16, 16, dtype=np.int8).reshape(1, 32)
    sc = O.f32_to_bf16_bits(np.array([[0.5]], np.float32))
    assert O.gemv_q8_0(qs, sc, x)[0, 0] == 0.5 * sum(range(-16, 16))
    q4 = np.array([[k | (15 - k) << 4 for k in range(16)]], np.uint8)  # element k: k, element k + 16: 15 - k
    bi = O.f32_to_bf16_bits(np.array([[2.0]], np.float32))
    xs = O.block_sums(x)
    assert O.gemv_q4_s(q4, sc, bi, x, xs)[0, 0] == 0.5 * (sum(range(16)) + sum(15 - k for k in range(16))) + 2.0 * 32
    # argmax: the first of equal maxima
    W2 = O.f32_to_bf16_bits(np.array([[1.0] * 32, [2.0] * 32, [2.0] * 32], np.float32))
    assert O.gemv_bf16w_argmax(W2, x) == 1


def test_argmax_rows_known_answers():
    # session.cpp:128-134: first maximum under >, -0 ties +0, NaN never
    # replaces the best, a NaN in the first place stays the answer
    x = np.array([[1, 3, 3, 2], [np.nan, 5, 6, 1], [-0.0, 0.0, -1, -2], [1, np.nan, 7, 7],
                  [-np.inf, -np.inf, -np.inf, -np.inf], [0.5, 0.25, np.inf, 1]], np.float32)
    assert O.argmax_rows(x).tolist() == [1, 0, 0, 2, 0, 2]
