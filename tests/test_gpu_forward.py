"""attention_forward on the device (nncu_attention_forward_dev) against the
checker's composition of the reference's steps (model.cpp:1559-1768): the q,
k, v gemvs (gemv_batch, model.cpp:1181-1206, through oracle.c's restatements
of the nn_ops.cpp gemvs, pinned in test_oracle.py), Qwen3.5's query / gate
split, Qwen2's biases, Gemma 4's V = raw K, then orc_attention_forward
(norms, RoPE, append, attend, the gate's sigmoid) and the o gemv.

Tolerance: y is an o gemv over attention rows that are themselves within the
attention's 2e-3 of the checker; y is held to a max-abs error of 2e-3 x
max |y| and a relative L2 error of 1e-3 (the attention's own bar, taken
relative to the output's scale); a prefill on the tensor cores to its own
2e-2 and 1e-2 (bf16 q rows and probabilities). The appended
cache rows are held to one step of the cache type's rounding plus 3e-5 x
max(1, |x|) (the gemvs' sums differ from the checker's in the last bits, so
a 16-bit rounding may land one step away)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


class W:
    """One projection's weights, host copies and their device tensors."""

    def __init__(self, rng, kind, rows, cols, torch):
        self.kind, self.rows, self.cols = kind, rows, cols
        s = 1.0 / np.sqrt(cols)
        if kind == O_BF16:
            self.w = O.f32_to_bf16_bits((rng.uniform(-1, 1, (rows, cols)) * s).astype(np.float32))
            self.sc = self.bi = None
        elif kind == O_Q8:
            self.w = rng.integers(-128, 128, (rows, cols), dtype=np.int8)
            self.sc = O.f32_to_bf16_bits((rng.uniform(0.5, 1.0, (rows, cols // 32)) * s / 128).astype(np.float32))
            self.bi = None
        else:
            self.w = rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
            self.sc = O.f32_to_bf16_bits((rng.uniform(0.5, 1.0, (rows, cols // 32)) * s / 8).astype(np.float32))
            self.bi = O.f32_to_bf16_bits((rng.uniform(-1, 1, (rows, cols // 32)) * s).astype(np.float32))
        dev = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a).view(
            np.int16 if a.dtype == np.uint16 else a.dtype)).cuda()
        self.d = (dev(self.w), dev(self.sc), dev(self.bi))

    def desc(self, N):
        return N.weight(self.kind, self.rows, self.cols, *self.d)

    def apply(self, X):
        """gemv_batch (model.cpp:1181-1206) on the checker."""
        if self.kind == O_BF16:
            return O.gemv_bf16w(self.w, X)
        if self.kind == O_Q8:
            return O.gemv_q8_0(self.w, self.sc, X)
        xs = np.stack([O.block_sums(x) for x in X])
        return O.gemv_q4_s(self.w, self.sc, self.bi, X, xs)


O_BF16, O_Q8, O_Q4 = 0, 1, 2


def _close(got, want, tol_abs=2e-3, tol_rel=1e-3):
    """Relative to the output's own scale: max-abs error within tol_abs of
    max |y| and relative L2 error within tol_rel."""
    assert np.isfinite(got).all()
    scale = float(np.abs(want).max())
    assert scale > 0
    err = np.abs(got.astype(np.float64) - want)
    rel = float(np.linalg.norm(err) / np.linalg.norm(want))
    assert err.max() <= tol_abs * scale and rel <= tol_rel, f"max-abs {err.max():.3g} of {scale:.3g}, rel-L2 {rel:.3g}"


def _checker(p_kw, ws, x, Kc, Vc, kv_type, rows, q_bias=None, k_bias=None, v_bias=None, gated=False, reuse=False):
    """model.cpp:1581-1767 on the checker: returns y; Kc and Vc take the
    appended rows in place."""
    n_tok, n_head, hd = p_kw["n_tok"], p_kw["n_head"], p_kw["head_dim"]
    q_dim = n_head * hd
    qq = ws["q"].apply(x)
    gate = None
    if gated:  # each head's rows: its query, then its gate (model.cpp:1586-1595)
        qg = qq.reshape(n_tok, n_head, 2, hd)
        qq = np.ascontiguousarray(qg[:, :, 0, :].reshape(n_tok, q_dim))
        gate = np.ascontiguousarray(qg[:, :, 1, :].reshape(n_tok, q_dim))
    k = v = np.zeros((n_tok, p_kw["n_kv"] * hd), np.float32)
    if not reuse:
        k = ws["k"].apply(x)
        v = ws["v"].apply(x) if "v" in ws else k.copy()  # Gemma 4: V is the raw K projection
    # biases after the V copy (model.cpp:1610-1617)
    if q_bias is not None:
        qq = (qq + q_bias[None, :]).astype(np.float32)
    if not reuse and k_bias is not None:
        k = (k + k_bias[None, :]).astype(np.float32)
    if not reuse and v_bias is not None:
        v = (v + v_bias[None, :]).astype(np.float32)
    p = O.params(**p_kw, gate=gate)
    attn, _, _ = O.attention_forward(p, qq, k, v, Kc, Vc, kv_type, rows)
    return ws["o"].apply(attn)


def _run(N, torch, rng, *, n_embd, n_head, n_kv, hd, n_tok, pos0, kinds, kv_type=O.KV_BF16, gated=False,
         biases=False, no_v=False, k_bias_only=False, window=0, extra=None, tol=(2e-3, 1e-3)):
    """One layer with `pos0` past rows, then one forward of n_tok tokens,
    against the checker."""
    extra = dict(extra or {})
    q_dim = n_head * hd
    ws = {"q": W(rng, kinds[0], (2 if gated else 1) * q_dim, n_embd, torch),
          "k": W(rng, kinds[1], n_kv * hd, n_embd, torch),
          "o": W(rng, kinds[3], n_embd, q_dim, torch)}
    if not no_v:
        ws["v"] = W(rng, kinds[2], n_kv * hd, n_embd, torch)
    qb = kb = vb = None
    if biases:
        qb = (rng.standard_normal(q_dim) * 0.1).astype(np.float32)
        kb = (rng.standard_normal(n_kv * hd) * 0.1).astype(np.float32)
        vb = None if no_v else (rng.standard_normal(n_kv * hd) * 0.1).astype(np.float32)
    if k_bias_only:
        kb = (rng.standard_normal(n_kv * hd) * 0.1).astype(np.float32)
    n_ctx = max(1024, pos0 + n_tok + 256)
    kv = N.KVCache([(n_kv, hd, window, 0)], n_ctx=n_ctx, n_batch=max(16, n_tok), kv_type=kv_type)
    rows = kv.layer_info(0).rows
    dt = np.float32 if kv_type == O.KV_F32 else np.uint16
    Kc = np.zeros((rows, n_kv * hd), dt)
    Vc = np.zeros_like(Kc)
    if pos0:
        keep0 = max(0, pos0 - rows)
        pk = O.narrow(rng.standard_normal((pos0 - keep0, n_kv * hd)).astype(np.float32), kv_type)
        pv = O.narrow(rng.standard_normal((pos0 - keep0, n_kv * hd)).astype(np.float32), kv_type)
        kv.write_rows(0, keep0, pk, pv)
        r = (keep0 + np.arange(pos0 - keep0)) % rows
        Kc[r], Vc[r] = pk, pv
    x = rng.standard_normal((n_tok, n_embd)).astype(np.float32)
    p_kw = dict(n_tok=n_tok, pos0=pos0, n_head=n_head, n_kv=n_kv, head_dim=hd, freq_base=1e4, window=window)
    p_kw.update(extra)
    host_vec = {k: v for k, v in p_kw.items() if k in ("q_gamma", "k_gamma", "freq_factors")}
    want = _checker(p_kw, ws, x, Kc, Vc, kv_type, rows, qb, kb, vb, gated)

    d = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).cuda()
    keep = {k: d(v) for k, v in host_vec.items()}
    pd = dict(p_kw)
    pd.update({k: t.data_ptr() for k, t in keep.items()})
    p = N.params(**pd)
    bq, bk, bv = d(qb), d(kb), d(vb)
    w = N.AttnWeights(ws["q"].desc(N), ws["k"].desc(N),
                      ws["v"].desc(N) if "v" in ws else N.Weight(0, 0, 0, None, None, None), ws["o"].desc(N),
                      None if bq is None else bq.data_ptr(), None if bk is None else bk.data_ptr(),
                      None if bv is None else bv.data_ptr(), int(gated))
    xd = d(x)
    y = torch.full((n_tok, n_embd), float("nan"), device="cuda")
    kv.attention_forward_dev(0, p, w, xd, y)
    kv.sync()
    got = y.cpu().numpy()
    _close(got, want, *tol)
    # the appended rows
    k_dev, v_dev = kv.read_rows(0, pos0, n_tok)
    idx = [(pos0 + t) % rows for t in range(n_tok)]
    step = {O.KV_F32: 0.0, O.KV_BF16: 2.0 ** -7, O.KV_F16: 2.0 ** -10}[kv_type]
    for got_r, want_r, what in ((k_dev, Kc[idx], "K"), (v_dev, Vc[idx], "V")):
        a = O.widen(got_r, kv_type).astype(np.float64)
        b = O.widen(want_r, kv_type).astype(np.float64)
        tol = step * np.abs(b) + 3e-5 * np.maximum(np.abs(b), 1.0)
        assert np.all(np.abs(a - b) <= tol), f"appended {what} rows"
    kv.close()
    return got, want


def test_llama_bf16_decode(nncu, torch_cuda):
    _run(nncu, torch_cuda, np.random.default_rng(1), n_embd=1024, n_head=8, n_kv=2, hd=128, n_tok=1, pos0=700,
         kinds=(O_BF16,) * 4)


def test_qwen2_q8_biases_verify(nncu, torch_cuda):
    _run(nncu, torch_cuda, np.random.default_rng(2), n_embd=896, n_head=14, n_kv=2, hd=64, n_tok=4, pos0=333,
         kinds=(O_Q8,) * 4, biases=True, kv_type=O.KV_F16)


def test_qwen35_gated_q4_s_qk_norm(nncu, torch_cuda):
    rng = np.random.default_rng(3)
    extra = dict(q_gamma=rng.uniform(0.5, 1.5, 256).astype(np.float32),
                 k_gamma=rng.uniform(0.5, 1.5, 256).astype(np.float32), n_rot=64)
    _run(nncu, torch_cuda, rng, n_embd=1024, n_head=8, n_kv=2, hd=256, n_tok=3, pos0=520,
         kinds=(O_Q4, O_Q4, O_Q8, O_Q4), gated=True, extra=extra)


def test_gemma4_global_v_is_k(nncu, torch_cuda):
    rng = np.random.default_rng(4)
    extra = dict(q_gamma=rng.uniform(0.5, 1.5, 512).astype(np.float32),
                 k_gamma=rng.uniform(0.5, 1.5, 512).astype(np.float32), v_rmsnorm=1, scale=1.0)
    _run(nncu, torch_cuda, rng, n_embd=640, n_head=4, n_kv=1, hd=512, n_tok=2, pos0=260,
         kinds=(O_BF16, O_BF16, O_BF16, O_Q8), no_v=True, kv_type=O.KV_F32, extra=extra)


def test_v_is_k_before_the_k_bias(nncu, torch_cuda):
    # without v_proj the reference copies V before adding the K bias
    _run(nncu, torch_cuda, np.random.default_rng(5), n_embd=256, n_head=2, n_kv=1, hd=128, n_tok=1, pos0=40,
         kinds=(O_BF16,) * 4, no_v=True, k_bias_only=True, kv_type=O.KV_F32)


def test_sliding_softcap_ring(nncu, torch_cuda):
    _run(nncu, torch_cuda, np.random.default_rng(6), n_embd=512, n_head=4, n_kv=2, hd=128, n_tok=2, pos0=1300,
         kinds=(O_Q8, O_BF16, O_Q4, O_BF16), window=512, extra=dict(softcap=30.0))


def test_prefill(nncu, torch_cuda):
    # 256 tokens on a bf16 cache of head_dim 128: the tensor-core prefill, whose
    # bf16 q rows and probabilities carry their own bar (test_gpu_prefill.py)
    _run(nncu, torch_cuda, np.random.default_rng(7), n_embd=512, n_head=4, n_kv=2, hd=128, n_tok=256, pos0=0,
         kinds=(O_BF16,) * 4, tol=(2e-2, 1e-2))


def test_reuse_kv_layer_projects_only_q(nncu, torch_cuda):
    N, torch = nncu, torch_cuda
    rng = np.random.default_rng(8)
    n_embd, n_head, n_kv, hd, pos0 = 256, 4, 1, 128, 90
    kv = N.KVCache([(n_kv, hd, 0, 0), (n_kv, hd, 0, 0)], n_ctx=512, n_batch=16, kv_type=O.KV_F32)
    rows = kv.layer_info(0).rows
    past_k = rng.standard_normal((pos0 + 1, n_kv * hd)).astype(np.float32)
    past_v = rng.standard_normal((pos0 + 1, n_kv * hd)).astype(np.float32)
    kv.write_rows(0, 0, past_k, past_v)  # the owner's rows, its newest token included
    Kc = np.zeros((rows, n_kv * hd), np.float32)
    Vc = np.zeros_like(Kc)
    Kc[:pos0 + 1], Vc[:pos0 + 1] = past_k, past_v
    ws = {"q": W(rng, O_BF16, n_head * hd, n_embd, torch), "o": W(rng, O_Q8, n_embd, n_head * hd, torch)}
    x = rng.standard_normal((1, n_embd)).astype(np.float32)
    p_kw = dict(n_tok=1, pos0=pos0, n_head=n_head, n_kv=n_kv, head_dim=hd, freq_base=1e4, reuse_kv=1)
    want = _checker(p_kw, ws, x, Kc, Vc, O.KV_F32, rows, reuse=True)
    none = N.Weight(0, 0, 0, None, None, None)
    w = N.AttnWeights(ws["q"].desc(N), none, none, ws["o"].desc(N), None, None, None, 0)
    y = torch.empty((1, n_embd), device="cuda")
    kv.attention_forward_dev(1, N.params(**p_kw), w, torch.from_numpy(x).cuda(), y)
    kv.sync()
    _close(y.cpu().numpy(), want)
    kv.close()


def test_refusals(nncu, torch_cuda):
    N, torch = nncu, torch_cuda
    rng = np.random.default_rng(9)
    kv = N.KVCache([(2, 64, 0, 0)], n_ctx=512, n_batch=16, kv_type=O.KV_BF16)
    ws = {k: W(rng, O_BF16, r, c, torch) for k, r, c in (("q", 256, 128), ("k", 128, 128), ("v", 128, 128),
                                                          ("o", 128, 256))}
    x = torch.zeros((1, 128), device="cuda")
    y = torch.zeros((1, 128), device="cuda")
    p = N.params(n_tok=1, pos0=0, n_head=4, n_kv=2, head_dim=64)

    def call(p=p, x=x, y=y, **over):
        d = {k: ws[k].desc(N) for k in ("q", "k", "v", "o")}
        d.update(over)
        w = N.AttnWeights(d["q"], d["k"], d["v"], d["o"], None, None, None, int(over.get("gated", 0)))
        kv.attention_forward_dev(0, p, w, x, y)

    call()
    kv.sync()
    with pytest.raises(N.NnncError, match="weights where"):
        call(q=ws["k"].desc(N))  # 128 rows where 256 are needed
    with pytest.raises(N.NnncError, match="weights where"):
        call(gated=1)  # a gated q has 2 * q_dim rows
    with pytest.raises(N.NnncError, match="unknown weight type"):
        call(o=N.Weight(7, 128, 256, ws["o"].d[0].data_ptr(), None, None))
    with pytest.raises(N.NnncError, match="scales"):
        call(k=N.Weight(N.W_Q8_0, 128, 128, ws["k"].d[0].data_ptr(), None, None))
    with pytest.raises(N.NnncError, match="overlap"):
        call(y=x)
    g = torch.zeros(256, device="cuda")
    with pytest.raises(N.NnncError, match="gate"):
        call(p=N.params(n_tok=1, pos0=1, n_head=4, n_kv=2, head_dim=64, gate=g.data_ptr()))
    kv.close()


def test_second_sequence_of_a_shared_cache(nncu, torch_cuda):
    # a cache of two sequences: the call on sequence 1 appends to and reads
    # only its own rows
    N, torch = nncu, torch_cuda
    rng = np.random.default_rng(10)
    n_embd, n_head, n_kv, hd, pos0 = 256, 4, 2, 64, 70
    kv = N.KVCache([(n_kv, hd, 0, 0)], n_ctx=256, n_batch=16, n_seq=2, kv_type=O.KV_F32)
    rows = kv.layer_info(0).rows
    caches = []
    for s in range(2):
        pk = rng.standard_normal((pos0, n_kv * hd)).astype(np.float32)
        pv = rng.standard_normal((pos0, n_kv * hd)).astype(np.float32)
        kv.write_rows(0, 0, pk, pv, seq=s)
        Kc = np.zeros((rows, n_kv * hd), np.float32)
        Vc = np.zeros_like(Kc)
        Kc[:pos0], Vc[:pos0] = pk, pv
        caches.append((Kc, Vc))
    ws = {k: W(rng, O_Q8, r, c, torch) for k, r, c in (("q", n_head * hd, n_embd), ("k", n_kv * hd, n_embd),
                                                       ("v", n_kv * hd, n_embd), ("o", n_embd, n_head * hd))}
    x = rng.standard_normal((2, n_embd)).astype(np.float32)
    p_kw = dict(n_tok=2, pos0=pos0, n_head=n_head, n_kv=n_kv, head_dim=hd, freq_base=1e4)
    want = _checker(p_kw, ws, x, caches[1][0], caches[1][1], O.KV_F32, rows)
    w = N.AttnWeights(ws["q"].desc(N), ws["k"].desc(N), ws["v"].desc(N), ws["o"].desc(N), None, None, None, 0)
    y = torch.empty((2, n_embd), device="cuda")
    kv.attention_forward_dev(0, N.params(**p_kw), w, torch.from_numpy(x).cuda(), y, seq=1)
    kv.sync()
    _close(y.cpu().numpy(), want)
    k1, _ = kv.read_rows(0, pos0, 2, seq=1)
    k0, _ = kv.read_rows(0, pos0, 2, seq=0)
    assert np.abs(k1 - caches[1][0][pos0:pos0 + 2]).max() < 1e-4  # appended to sequence 1
    assert not np.any(k0)  # sequence 0 untouched past its rows
    kv.close()


def test_batch_of_sequences_in_one_call(nncu, torch_cuda):
    # nncu_attention_forward_batch_dev: three sequences of different lengths
    # and positions through one gated Q4_S layer with Q/K norms; each against
    # the checker's composition on its own cache
    N, torch = nncu, torch_cuda
    rng = np.random.default_rng(12)
    n_embd, n_head, n_kv, hd = 512, 4, 2, 128
    kv = N.KVCache([(n_kv, hd, 0, 0)], n_ctx=512, n_batch=16, n_seq=3, kv_type=O.KV_BF16)
    rows = kv.layer_info(0).rows
    seqs, toks, pos = [2, 0, 1], [4, 1, 2], [250, 100, 30]
    qg = rng.uniform(0.5, 1.5, hd).astype(np.float32)
    kg = rng.uniform(0.5, 1.5, hd).astype(np.float32)
    ws = {"q": W(rng, O_Q4, 2 * n_head * hd, n_embd, torch), "k": W(rng, O_Q4, n_kv * hd, n_embd, torch),
          "v": W(rng, O_Q4, n_kv * hd, n_embd, torch), "o": W(rng, O_Q4, n_embd, n_head * hd, torch)}
    x = rng.standard_normal((sum(toks), n_embd)).astype(np.float32)
    want, params = [], []
    dqg, dkg = torch.from_numpy(qg).cuda(), torch.from_numpy(kg).cuda()
    r0 = 0
    for s, nt, p0 in zip(seqs, toks, pos):
        pk = O.narrow(rng.standard_normal((p0, n_kv * hd)).astype(np.float32), O.KV_BF16)
        pv = O.narrow(rng.standard_normal((p0, n_kv * hd)).astype(np.float32), O.KV_BF16)
        kv.write_rows(0, 0, pk, pv, seq=s)
        Kc = np.zeros((rows, n_kv * hd), np.uint16)
        Vc = np.zeros_like(Kc)
        Kc[:p0], Vc[:p0] = pk, pv
        kw = dict(n_tok=nt, pos0=p0, n_head=n_head, n_kv=n_kv, head_dim=hd, freq_base=1e4)
        want.append(_checker(dict(kw, q_gamma=qg, k_gamma=kg), ws, x[r0:r0 + nt], Kc, Vc, O.KV_BF16, rows,
                             gated=True))
        params.append(N.params(**kw, q_gamma=dqg.data_ptr(), k_gamma=dkg.data_ptr()))
        r0 += nt
    w = N.AttnWeights(ws["q"].desc(N), ws["k"].desc(N), ws["v"].desc(N), ws["o"].desc(N), None, None, None, 1)
    y = torch.full((sum(toks), n_embd), float("nan"), device="cuda")
    kv.attention_forward_batch_dev(0, seqs, params, w, torch.from_numpy(x).cuda(), y)
    kv.sync()
    got = y.cpu().numpy()
    r0 = 0
    for i, nt in enumerate(toks):
        _close(got[r0:r0 + nt], want[i])
        r0 += nt
    with pytest.raises(N.NnncError, match="twice"):
        kv.attention_forward_batch_dev(0, [0, 0], params[:2], w, torch.from_numpy(x[:2]).cuda(), y)
    kv.close()
