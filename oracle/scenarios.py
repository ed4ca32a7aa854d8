"""TEST INFRASTRUCTURE ONLY: seeded attention scenarios and their checker runs.

A scenario is a stack of layers, each with the inputs one attention_forward
call gets (q, k, v projections of n_tok new tokens, Q/K norm gains) and the
cache contents it attends over (the K/V rows of the positions before pos0).
Inputs come from the reference tests' generator -- std::mt19937(seed) through
std::normal_distribution<float> -- drawn per sequence, per layer, in this
order: q, k, v, q_gamma, k_gamma, then the past K rows, then the past V rows,
then (Qwen3.5 layers only) the output gate.
Past keys are optionally rotated at their own positions first, as the
reference's own append would have left them.

The checker runs are ``run_checker(case, which)`` with which = "oracle" (the
C restatement) or "ref" (the reference's compiled kernels, F32/BF16 only).
"""
from __future__ import annotations

import dataclasses as dc

import numpy as np

from . import (KV_BF16, KV_F16, KV_F32, ROPE_NEOX, ROPE_NORM, Rng, attention_forward, narrow, orc_params,
               ring_rows, rope)


@dc.dataclass
class LayerSpec:
    n_head: int
    n_kv: int
    head_dim: int
    window: int = 0            # 0 = global
    freq_base: float = 10000.0
    rope_mode: int = ROPE_NEOX
    qk_norm: bool = False
    n_rot: int | None = None
    rope_scale: float = 1.0
    softcap: float = 0.0
    freq_factors: np.ndarray | None = None
    v_rmsnorm: bool = False
    scale: float | None = None
    kv_layer: int | None = None  # another layer whose cache this one reads (None: its own)
    gated: bool = False          # Qwen3.5: the output multiplied by sigmoid(gate)


@dc.dataclass
class LayerInputs:
    q: np.ndarray              # [n_tok, n_head*D]
    k: np.ndarray              # [n_tok, n_kv*D]
    v: np.ndarray
    q_gamma: np.ndarray | None
    k_gamma: np.ndarray | None
    past_k: np.ndarray         # [n_keep, n_kv*D] fp32 values of positions keep0 .. pos0-1
    past_v: np.ndarray
    keep0: int                 # first past position still held by the buffer
    gate: np.ndarray | None = None  # [n_tok, n_head*D] (Qwen3.5), drawn last


@dc.dataclass
class Case:
    layers: list[LayerSpec]
    n_ctx: int
    n_batch: int
    n_tok: int
    pos0: list[int]            # per sequence
    kv_type: int
    causal: bool
    inputs: list[list[LayerInputs]]  # [seq][layer]
    rows: list[int]            # per layer: the buffer's rows (model_kv_init's sizing)

    @property
    def n_seqs(self) -> int:
        return len(self.pos0)

    def params_dict(self, layer: int, seq: int) -> dict:
        L = self.layers[layer]
        inp = self.inputs[seq][layer]
        d = dict(n_tok=self.n_tok, pos0=self.pos0[seq], n_seq=self.pos0[seq] + self.n_tok, n_head=L.n_head,
                 n_kv=L.n_kv, head_dim=L.head_dim, n_rot=L.n_rot if L.n_rot is not None else L.head_dim,
                 rope_mode=L.rope_mode, freq_base=L.freq_base, rope_scale=L.rope_scale,
                 freq_factors=L.freq_factors, q_gamma=inp.q_gamma, k_gamma=inp.k_gamma,
                 v_rmsnorm=int(L.v_rmsnorm), eps=1e-6,
                 scale=L.scale if L.scale is not None else 1.0 / float(np.sqrt(L.head_dim)),
                 softcap=L.softcap, causal=int(self.causal), window=L.window,
                 reuse_kv=int(L.kv_layer is not None and L.kv_layer != layer), gate=inp.gate)
        if not self.causal:
            d["n_seq"] = self.n_ctx
        return d

    def layer_descs(self):
        return [(L.n_kv, L.head_dim, L.window, L.kv_layer if L.kv_layer is not None else i)
                for i, L in enumerate(self.layers)]


def buffer_rows(layers: list[LayerSpec], n_ctx: int, n_batch: int, causal: bool) -> list[int]:
    """Rows of each layer's buffer under model_kv_init's rules (model.cpp:1929-1962)."""
    if not causal:
        return [n_ctx] * len(layers)
    owner = [L.kv_layer if L.kv_layer is not None else i for i, L in enumerate(layers)]
    win = {}
    ok = {}
    for i, L in enumerate(layers):
        o = owner[i]
        ok.setdefault(o, True)
        if L.window == 0:
            ok[o] = False
        elif win.get(o, 0) == 0:
            win[o] = L.window
        elif win[o] != L.window:
            ok[o] = False
    rows = []
    for i in range(len(layers)):
        o = owner[i]
        w = win.get(o, 0)
        r = ring_rows(w, n_batch)
        rows.append(r if ok[o] and w > 0 and r < n_ctx else n_ctx)
    return rows


def build_case(seed: int, layers: list[LayerSpec], n_ctx: int, n_tok: int, pos0, kv_type: int,
               n_batch: int | None = None, causal: bool = True, rotate_past: bool = False,
               gamma_std: float = 0.1) -> Case:
    """Draw a scenario. pos0: an int or a list (one per sequence)."""
    pos0 = [pos0] if isinstance(pos0, int) else list(pos0)
    n_batch = n_batch if n_batch is not None else max(n_tok, 1)
    rows = buffer_rows(layers, n_ctx, n_batch, causal)
    rng = Rng(seed)
    inputs = []
    for s, p0 in enumerate(pos0):
        per = []
        for li, L in enumerate(layers):
            D = L.head_dim
            q = rng.normal(n_tok * L.n_head * D).reshape(n_tok, L.n_head * D)
            k = rng.normal(n_tok * L.n_kv * D).reshape(n_tok, L.n_kv * D)
            v = rng.normal(n_tok * L.n_kv * D).reshape(n_tok, L.n_kv * D)
            qg = rng.normal(D, 1.0, gamma_std) if L.qk_norm else None
            kg = rng.normal(D, 1.0, gamma_std) if L.qk_norm else None
            reuse = L.kv_layer is not None and L.kv_layer != li
            keep0 = max(0, p0 - rows[li]) if causal else 0
            n_keep = 0 if reuse else (p0 - keep0 if causal else 0)
            pk = rng.normal(n_keep * L.n_kv * D).reshape(n_keep, L.n_kv * D)
            pv = rng.normal(n_keep * L.n_kv * D).reshape(n_keep, L.n_kv * D)
            if rotate_past and n_keep:
                n_rot = L.n_rot if L.n_rot is not None else D
                for t in range(n_keep):
                    pk[t] = rope(pk[t], L.n_kv, D, n_rot, float(keep0 + t) * L.rope_scale, L.freq_base,
                                 L.rope_mode, L.freq_factors)
            # the gate comes after everything else, so ungated cases draw what they always drew
            gate = rng.normal(n_tok * L.n_head * D, 0.0, 2.0).reshape(n_tok, L.n_head * D) if L.gated else None
            per.append(LayerInputs(q, k, v, qg, kg, pk, pv, keep0, gate))
        inputs.append(per)
    return Case(layers, n_ctx, n_batch, n_tok, pos0, kv_type, causal, inputs, rows)


def cache_bits(case: Case, seq: int, layer: int):
    """The layer's buffer (reference layout [rows][n_kv*D], the cache type's
    bits) holding the past rows at position % rows."""
    L = case.layers[layer]
    rows = case.rows[layer]
    dt = np.float32 if case.kv_type == KV_F32 else np.uint16
    Kc = np.zeros((rows, L.n_kv * L.head_dim), dt)
    Vc = np.zeros_like(Kc)
    inp = case.inputs[seq][layer]
    n = inp.past_k.shape[0]
    if n:
        r = (inp.keep0 + np.arange(n)) % rows  # n <= rows: no row is written twice
        Kc[r] = narrow(inp.past_k, case.kv_type)
        Vc[r] = narrow(inp.past_v, case.kv_type)
    return Kc, Vc


def run_checker(case: Case, which: str = "oracle"):
    """Every layer of every sequence through the checker, in layer order (a
    layer that reuses another's cache reads it after that layer appended).
    Returns (outs[seq][layer] [n_tok, n_head*D], caches[seq][owner] (Kc, Vc))."""
    outs, caches = [], []
    for s in range(case.n_seqs):
        bufs = {}
        row = []
        for li, L in enumerate(case.layers):
            owner = L.kv_layer if L.kv_layer is not None else li
            if owner not in bufs:
                bufs[owner] = cache_bits(case, s, owner)
            Kc, Vc = bufs[owner]
            inp = case.inputs[s][li]
            p = orc_params(**case.params_dict(li, s))
            kt = case.kv_type
            if which == "ref" and kt == KV_F16:
                raise ValueError("the reference has no F16 cache")
            out, _, _ = attention_forward(p, inp.q, inp.k, inp.v, Kc, Vc, kt, case.rows[li], which=which)
            row.append(out)
        outs.append(row)
        caches.append(bufs)
    return outs, caches


def errors(got: np.ndarray, want: np.ndarray) -> tuple[float, float]:
    """(max-abs error, relative-L2 error)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    d = got - want
    return float(np.abs(d).max(initial=0.0)), float(np.linalg.norm(d) / max(np.linalg.norm(want), 1e-30))


__all__ = ["LayerSpec", "LayerInputs", "Case", "buffer_rows", "build_case", "cache_bits", "run_checker", "errors",
           "KV_BF16", "KV_F16", "KV_F32", "ROPE_NEOX", "ROPE_NORM"]
