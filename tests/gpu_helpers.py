"""Helpers for the GPU parity tests: run a seeded scenario through the
product (libnncu via its C ABI) exactly as through the checker."""
from __future__ import annotations

import numpy as np

import oracle as O
from oracle import scenarios as S

# north_star tolerance for fp32 / fp16 caches: max-abs 2e-3 and relative-L2 1e-3
TOL_ABS, TOL_REL = 2e-3, 1e-3


def make_cache(N, case: S.Case):
    kv = N.KVCache(case.layer_descs(), n_ctx=case.n_ctx, n_batch=case.n_batch, n_seq=case.n_seqs,
                   kv_type=case.kv_type, causal=case.causal)
    for s in range(case.n_seqs):
        for li, L in enumerate(case.layers):
            owner = L.kv_layer if L.kv_layer is not None else li
            if owner != li:
                continue
            inp = case.inputs[s][li]
            if inp.past_k.shape[0]:
                kv.write_rows(li, inp.keep0, O.narrow(inp.past_k, case.kv_type), O.narrow(inp.past_v, case.kv_type),
                              seq=s)
    return kv


def run_product(N, case: S.Case, kv=None, batch: bool = False, per_layer: bool = False):
    """Every layer of every sequence through the product, in the checker's
    order. batch=True submits all layers of a sequence in one
    nncu_attention_batch call (only for cases without shared K/V);
    per_layer=True submits each layer once for all sequences (the drop-in's
    call pattern for a batch of sequences)."""
    kv = kv or make_cache(N, case)
    if per_layer:
        outs = [[None] * len(case.layers) for _ in range(case.n_seqs)]
        for li in range(len(case.layers)):
            jobs = []
            for s in range(case.n_seqs):
                inp = case.inputs[s][li]
                p = N.params(**case.params_dict(li, s))
                out = np.empty((case.n_tok, p.n_head * p.head_dim), np.float32)
                jobs.append(N.job(li, p, np.ascontiguousarray(inp.q), np.ascontiguousarray(inp.k),
                                  np.ascontiguousarray(inp.v), out, seq=s))
                outs[s][li] = out
            kv.attention_batch(jobs)
        return outs, kv
    outs = []
    for s in range(case.n_seqs):
        row = []
        if batch:
            jobs, res = [], []
            for li in range(len(case.layers)):
                inp = case.inputs[s][li]
                p = N.params(**case.params_dict(li, s))
                out = np.empty((case.n_tok, p.n_head * p.head_dim), np.float32)
                jobs.append(N.job(li, p, np.ascontiguousarray(inp.q), np.ascontiguousarray(inp.k),
                                  np.ascontiguousarray(inp.v), out, seq=s))
                res.append(out)
            kv.attention_batch(jobs)
            row = res
        else:
            for li in range(len(case.layers)):
                inp = case.inputs[s][li]
                p = N.params(**case.params_dict(li, s))
                reuse = p.reuse_kv != 0
                row.append(kv.attention(li, p, inp.q, None if reuse else inp.k, None if reuse else inp.v, seq=s))
        outs.append(row)
    return outs, kv


def assert_close(got, want, what, tol_abs=TOL_ABS, tol_rel=TOL_REL):
    e_abs, e_rel = S.errors(got, want)
    assert e_abs <= tol_abs and e_rel <= tol_rel, f"{what}: max-abs {e_abs:.3g}, rel-L2 {e_rel:.3g}"
    return e_abs, e_rel
