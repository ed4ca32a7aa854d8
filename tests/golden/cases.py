"""The golden cases: small seeded scenarios shaped like the five benchmark
configurations, and unit cases for the kernels of nn_ops.h.

Inputs are never stored: they are redrawn from their seeds with the
reference tests' generator (oracle.Rng), and golden.npz keeps a digest of
them so a changed generator is caught. Only the reference's outputs are
stored. Shapes are cut down from the benchmark's so the checker finishes in
seconds; the full sizes are exercised by the GPU tests' properties.
"""
from __future__ import annotations

import functools
import hashlib

import numpy as np

import oracle as O
from oracle import scenarios as S
from oracle.scenarios import LayerSpec

KV = {"f32": O.KV_F32, "bf16": O.KV_BF16, "f16": O.KV_F16}


@functools.lru_cache(maxsize=None)
def all_cases() -> dict:
    c = {}
    # config 1, Llama-3.2-1B decode: GQA 32:8, head_dim 64, NORM RoPE theta 5e5, F32,
    # cached keys rotated at their positions
    c["cfg1_decode_f32"] = S.build_case(
        0, [LayerSpec(32, 8, 64, freq_base=5e5, rope_mode=O.ROPE_NORM)], n_ctx=512, n_tok=1, pos0=300,
        kv_type=O.KV_F32, rotate_past=True)
    # config 2, Gemma-3-1B: 4:1 heads of 256, Q/K norm; a sliding layer (window 512,
    # theta 1e4, a ring of 768 rows wrapped) and a global one (theta 1e6)
    g3 = [LayerSpec(4, 1, 256, window=512, freq_base=1e4, qk_norm=True),
          LayerSpec(4, 1, 256, window=0, freq_base=1e6, qk_norm=True)]
    c["cfg2_stack_f32"] = S.build_case(1, g3, n_ctx=1024, n_tok=1, pos0=900, kv_type=O.KV_F32, n_batch=1)
    c["cfg2_stack_bf16"] = S.build_case(1, g3, n_ctx=1024, n_tok=1, pos0=900, kv_type=O.KV_BF16, n_batch=1)
    # config 3, Qwen3-4B prefill: causal block from position 0, Q/K norm, theta 1e6, BF16
    c["cfg3_prefill_bf16"] = S.build_case(
        2, [LayerSpec(8, 2, 128, freq_base=1e6, qk_norm=True)], n_ctx=64, n_tok=48, pos0=0, kv_type=O.KV_BF16)
    # config 4, Gemma-3-4B verify: 4 draft tokens per sequence, two sequences, 8:4 heads of 256,
    # a sliding layer (window 1024, a ring of 1280 rows) and a global one
    g34 = [LayerSpec(8, 4, 256, window=1024, freq_base=1e4, qk_norm=True),
           LayerSpec(8, 4, 256, window=0, freq_base=1e6, qk_norm=True)]
    c["cfg4_verify_bf16"] = S.build_case(3, g34, n_ctx=1536, n_tok=4, pos0=[1100, 1301], kv_type=O.KV_BF16)
    # config 5, Llama-3.2-1B long context, cut to 2048 keys (BF16 here: the reference has no F16)
    c["cfg5_long_bf16"] = S.build_case(
        4, [LayerSpec(32, 8, 64, freq_base=5e5, rope_mode=O.ROPE_NORM)], n_ctx=2304, n_tok=1, pos0=2048,
        kv_type=O.KV_BF16)
    # partial rotation, frequency factors, a short window, no grouping, 3 tokens over a block edge
    ff = (1.0 + np.arange(16, dtype=np.float32) / 4.0).astype(np.float32)
    c["window_partial_rope_f32"] = S.build_case(
        5, [LayerSpec(4, 4, 64, window=100, freq_base=1e4, n_rot=32, freq_factors=ff, rope_scale=0.5)],
        n_ctx=600, n_tok=3, pos0=255, kv_type=O.KV_F32)
    # a bidirectional (embedding) model: one call over the whole sequence, symmetric window
    c["bidirectional_f32"] = S.build_case(
        6, [LayerSpec(4, 2, 64, window=64, qk_norm=True), LayerSpec(4, 2, 64, window=0, qk_norm=True)],
        n_ctx=96, n_tok=96, pos0=0, kv_type=O.KV_F32, causal=False)
    # Qwen3.5's gated attention: the output times sigmoid(gate), per element
    # (model.cpp:1759-1760); partial rotation (64 of 256), Q/K norm, theta 1e7,
    # a 3-token verify block
    c["qwen35_gated_bf16"] = S.build_case(
        8, [LayerSpec(8, 2, 256, freq_base=1e7, n_rot=64, qk_norm=True, gated=True)], n_ctx=900, n_tok=3,
        pos0=800, kv_type=O.KV_BF16)
    # a layer reading the cache an earlier layer appended to (Gemma 3n / 4 shared K/V)
    c["reuse_kv_bf16"] = S.build_case(
        7, [LayerSpec(8, 2, 128, freq_base=1e6), LayerSpec(8, 2, 128, freq_base=1e6, kv_layer=0)],
        n_ctx=700, n_tok=2, pos0=600, kv_type=O.KV_BF16)
    return c


def inputs_digest(case) -> str:
    h = hashlib.sha256()
    for per in case.inputs:
        for inp in per:
            for a in (inp.q, inp.k, inp.v, inp.q_gamma, inp.k_gamma, inp.past_k, inp.past_v, inp.gate):
                if a is not None:
                    h.update(np.ascontiguousarray(a, np.float32).tobytes())
    return h.hexdigest()


# ---- unit cases ----------------------------------------------------------------------------

UNIT_CASES = [
    "attn_blocks_f32_64", "attn_blocks_f32_36", "attn_blocks_bf16_64", "attn_blocks_bf16_36",
    "rope_neox_r32_pos17", "rope_norm_pos1024", "rope_norm_pos131072", "rope_neox_d256_pos4096",
    "rope_neox_ff", "rmsnorm_gamma_64", "rmsnorm_gamma_256", "rmsnorm_gamma_13",
]


def unit_inputs(name: str):
    if name.startswith("attn_blocks"):
        _, _, t, hd = name.split("_")
        hd = int(hd)
        rng = O.Rng(7)
        group, n_kv, n_keys = 3, 2, 600
        kvs = n_kv * hd
        q = rng.normal(group * hd)
        K = 2.0 * rng.normal(n_keys * kvs)
        V = rng.normal(n_keys * kvs)
        return dict(q=q, K=O.narrow(K, KV[t]), V=O.narrow(V, KV[t]), kt=KV[t], group=group, hd=hd, kvs=kvs)
    if name.startswith("rope"):
        spec = {
            "rope_neox_r32_pos17": (O.ROPE_NEOX, 1e6, 17.0, 32, 64, False),
            "rope_norm_pos1024": (O.ROPE_NORM, 5e5, 1024.0, 64, 64, False),
            "rope_norm_pos131072": (O.ROPE_NORM, 5e5, 131072.0, 64, 64, False),
            "rope_neox_d256_pos4096": (O.ROPE_NEOX, 1e4, 4096.0, 256, 256, False),
            "rope_neox_ff": (O.ROPE_NEOX, 1e6, 4096.0, 128, 128, True),
        }[name]
        mode, base, pos, n_rot, D, ff = spec
        rng = O.Rng(11)
        x = rng.normal(4 * D)
        f = (1.0 + np.abs(rng.normal(n_rot // 2))).astype(np.float32) if ff else None
        return dict(x=x, H=4, D=D, n_rot=n_rot, pos=pos, base=base, mode=mode, ff=f)
    dim = int(name.split("_")[-1])
    rng = O.Rng(12 + dim)
    return dict(x=rng.normal(7 * dim), g=rng.normal(dim, 1.0, 0.1), n=7, dim=dim)


def run_unit(name: str, which: str) -> np.ndarray:
    a = unit_inputs(name)
    if name.startswith("attn_blocks"):
        hd, kvs, group = a["hd"], a["kvs"], a["group"]
        scale = 1.0 / np.sqrt(hd)
        k0, acc = 0, None
        for n in (100, 256, 244):
            part = O.attn_block(a["q"], hd, a["K"], a["V"], a["kt"], kvs, n, hd, group, scale, which=which,
                                k_offset_elems=k0 * kvs + hd)
            acc = part if acc is None else O.attn_merge(acc, part, hd, group, which=which)
            k0 += n
        return O.attn_finish(acc, hd, group, which=which)
    if name.startswith("rope"):
        return O.rope(a["x"], a["H"], a["D"], a["n_rot"], a["pos"], a["base"], a["mode"], a["ff"], which=which)
    return O.rmsnorm_gamma_multi(a["x"], a["n"], a["dim"], a["g"], 1e-6, which=which)
