"""The projections' gemvs on the device (k_gemv.cu) through the C ABI, against
the checker (oracle.c, pinned to the reference's compiled nn_ops.cpp gemvs in
test_oracle.py): BF16, Q8_0 and Q4_S weights with fp32 activations, one vector
and batches, on the shapes of the reference's own gemv tests
(tests.cpp:819-880) and a Gemma-3-4B-sized projection; the block sums; and the
greedy lm_head's gemv + argmax. Tolerance: the reference tests' 1e-3 x
max(1, |y|)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

# the last three: one vector on tall matrices (Q4_S 4 and 8 rows per warp, Q8_0
# 2 and 4), heights not a multiple of the rows per warp
SHAPES = [(1, 32, 1), (8, 64, 1), (64, 128, 3), (256, 256, 2), (512, 512, 1), (1024, 2048, 4), (2560, 2048, 9),
          (300, 96, 17), (2050, 96, 1), (8195, 64, 1), (12301, 64, 1)]


def _inputs(rows, cols, nb, seed):
    rng = np.random.default_rng(seed)
    W = O.f32_to_bf16_bits(rng.uniform(-1, 1, (rows, cols)).astype(np.float32))
    X = rng.uniform(-1, 1, (nb, cols)).astype(np.float32)
    qs8 = rng.integers(-128, 128, (rows, cols), dtype=np.int8)
    sc = O.f32_to_bf16_bits((rng.random((rows, cols // 32)) * 0.02).astype(np.float32))
    qs4 = rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
    bi = O.f32_to_bf16_bits((rng.uniform(-1, 1, (rows, cols // 32)) * 0.1).astype(np.float32))
    return W, X, qs8, sc, qs4, bi


def _check(got, want, what):
    err = np.abs(got - want) / np.maximum(1.0, np.abs(want))
    assert err.max() <= 1e-3, f"{what}: worst scaled error {err.max():.3g}"


@pytest.mark.parametrize("rows,cols,nb", SHAPES)
def test_gemvs_match_the_checker(nncu, torch_cuda, rows, cols, nb):
    N, torch = nncu, torch_cuda
    W, X, qs8, sc, qs4, bi = _inputs(rows, cols, nb, rows + 13 * cols + nb)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    Xd = d(X)
    Y = torch.full((nb, rows), float("nan"), device="cuda")
    N.gemv_bf16w_dev(d(W.view(np.int16)), Xd, Y, rows, cols, nb)
    torch.cuda.synchronize()
    _check(Y.cpu().numpy(), O.gemv_bf16w(W, X), f"bf16 {rows}x{cols} x{nb}")
    N.gemv_q8_0_dev(d(qs8), d(sc.view(np.int16)), Xd, Y, rows, cols, nb)
    torch.cuda.synchronize()
    _check(Y.cpu().numpy(), O.gemv_q8_0(qs8, sc, X), f"q8_0 {rows}x{cols} x{nb}")
    XS = torch.empty((nb, cols // 32), device="cuda")
    for v in range(nb):
        N.block_sums_dev(Xd[v], XS[v], cols)
    torch.cuda.synchronize()
    xs = np.stack([O.block_sums(x) for x in X])
    assert np.allclose(XS.cpu().numpy(), xs, rtol=1e-5, atol=1e-5)
    N.gemv_q4_s_dev(d(qs4), d(sc.view(np.int16)), d(bi.view(np.int16)), Xd, XS, Y, rows, cols, nb)
    torch.cuda.synchronize()
    _check(Y.cpu().numpy(), O.gemv_q4_s(qs4, sc, bi, X, xs), f"q4_s {rows}x{cols} x{nb}")


def test_gemv_bf16w_odd_columns_and_strides(nncu, torch_cuda):
    # columns not a multiple of 8 (the reference's scalar path), strided batch
    N, torch = nncu, torch_cuda
    rows, cols, nb = 37, 100, 3
    W, X, *_ = _inputs(rows, 128, nb, 5)
    W = np.ascontiguousarray(W[:, :cols])
    Xp = np.zeros((nb, 112), np.float32)
    Xp[:, :cols] = X[:, :cols]
    Y = torch.zeros((nb, 48), device="cuda")
    N.gemv_bf16w_dev(torch.from_numpy(W.view(np.int16)).cuda(), torch.from_numpy(Xp).cuda(), Y, rows, cols, nb,
                     x_stride=112, y_stride=48)
    torch.cuda.synchronize()
    _check(Y.cpu().numpy()[:, :rows], O.gemv_bf16w(W, np.ascontiguousarray(X[:, :cols])), "bf16 odd columns")


@pytest.mark.parametrize("rows,cols", [(4, 64), (1000, 256), (262144 // 64, 2560)])
def test_gemv_argmax(nncu, torch_cuda, rows, cols):
    N, torch = nncu, torch_cuda
    rng = np.random.default_rng(rows)
    W = O.f32_to_bf16_bits(rng.uniform(-1, 1, (rows, cols)).astype(np.float32))
    x = rng.uniform(-1, 1, cols).astype(np.float32)
    scratch = torch.zeros(1, dtype=torch.int64, device="cuda")
    out = torch.full((1,), -7, dtype=torch.int32, device="cuda")
    Wd = torch.from_numpy(W.view(np.int16)).cuda()
    N.gemv_bf16w_argmax_dev(Wd, torch.from_numpy(x).cuda(), rows, cols, scratch, out)
    torch.cuda.synchronize()
    want = O.gemv_bf16w_argmax(W, x)
    got = int(out.item())
    if got != want:  # a near tie decided by summation order: both must be maximal within tolerance
        y = O.gemv_bf16w(W, x)[0]
        assert abs(y[got] - y[want]) <= 1e-3 * max(1.0, abs(y[want])), (got, want)
    # the first of equal maxima
    W2 = np.repeat(O.f32_to_bf16_bits(np.linspace(-1, 1, 8, dtype=np.float32))[None, :], 6, axis=0)
    W2[[2, 4]] = O.f32_to_bf16_bits(np.full(8, 0.5, np.float32))
    x2 = np.ones(8, np.float32)
    N.gemv_bf16w_argmax_dev(torch.from_numpy(W2.view(np.int16)).cuda(), torch.from_numpy(x2).cuda(), 6, 8, scratch,
                            out)
    torch.cuda.synchronize()
    assert int(out.item()) == 2


def test_gemv_refusals(nncu, torch_cuda):
    N, torch = nncu, torch_cuda
    buf = torch.zeros(4096, device="cuda")
    with pytest.raises(N.NnncError):
        N.gemv_q8_0_dev(buf, buf, buf, buf, 4, 48)  # cols not a multiple of 32
    with pytest.raises(N.NnncError):
        N.gemv_q4_s_dev(buf[1:], buf, buf, buf, buf, buf, 4, 64)  # misaligned quants


def test_argmax_rows_match_the_checker(nncu, torch_cuda):
    # session.cpp:128-134 on each row: ties, signed zeros, NaNs, infinities,
    # and random rows of a Gemma-sized vocabulary
    N, torch = nncu, torch_cuda
    rng = np.random.default_rng(3)
    n = 262144
    X = rng.standard_normal((6, n)).astype(np.float32)
    X[1, 77] = X[1, 9000] = 50.0                     # the first of two maxima
    X[2, 0] = np.nan                                 # NaN first: index 0
    X[3, :] = -0.0
    X[3, 5] = 0.0                                    # -0 and +0 tie: index 0
    X[4, 1000:2000] = np.nan
    X[4, 1500] = 1e30                                # NaNs skipped around the max
    X[5, :] = -np.inf                                # all -inf: index 0
    out = torch.full((6,), -7, dtype=torch.int32, device="cuda")
    N.argmax_rows_dev(torch.from_numpy(X).cuda(), 6, n, out)
    torch.cuda.synchronize()
    assert out.cpu().numpy().tolist() == O.argmax_rows(X).tolist()
    # strided rows, a short length
    Xp = np.zeros((3, 40), np.float32)
    Xp[:, :33] = rng.standard_normal((3, 33))
    Xp[:, 33:] = 1e9  # beyond each row's length
    out3 = torch.zeros(3, dtype=torch.int32, device="cuda")
    N.argmax_rows_dev(torch.from_numpy(Xp).cuda(), 3, 33, out3, x_stride=40)
    torch.cuda.synchronize()
    assert out3.cpu().numpy().tolist() == O.argmax_rows(np.ascontiguousarray(Xp[:, :33])).tolist()


@pytest.mark.parametrize("kind", ["bf16", "q8_0", "q4_s"])
def test_verify_logits_match_the_checker(nncu, torch_cuda, kind):
    # model_logits_batch (model.cpp:2198-2208): the lm_head over the n + 1
    # verify rows, then the final soft-cap (sampling) or none (greedy)
    N, torch = nncu, torch_cuda
    rows, cols, n = 5000, 640, 5
    W, X, qs8, sc, qs4, bi = _inputs(rows, cols, n, 17)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    if kind == "bf16":
        w = N.weight(N.W_BF16, rows, cols, d(W.view(np.int16)))
        want = O.gemv_bf16w(W, X)
    elif kind == "q8_0":
        w = N.weight(N.W_Q8_0, rows, cols, d(qs8), d(sc.view(np.int16)))
        want = O.gemv_q8_0(qs8, sc, X)
    else:
        w = N.weight(N.W_Q4_S, rows, cols, d(qs4), d(sc.view(np.int16)), d(bi.view(np.int16)))
        want = O.gemv_q4_s(qs4, sc, bi, X, np.stack([O.block_sums(x) for x in X]))
    keep = w._keep
    xs = torch.empty((n, cols // 32), device="cuda")
    for cap in (0.0, 30.0):
        logits = torch.full((n, rows), float("nan"), device="cuda")
        N.logits_batch_dev(w, d(X), n, logits, cap, xs)
        torch.cuda.synchronize()
        ref = want if cap == 0.0 else O.softcap(want.ravel(), cap).reshape(want.shape)
        _check(logits.cpu().numpy(), ref, f"{kind} logits, cap {cap}")
    if kind == "q4_s":  # without the scratch the gemv forms the block sums itself
        logits = torch.full((n, rows), float("nan"), device="cuda")
        N.logits_batch_dev(w, d(X), n, logits, 0.0, None)
        torch.cuda.synchronize()
        _check(logits.cpu().numpy(), want, "q4_s logits, in-kernel block sums")
    del keep
