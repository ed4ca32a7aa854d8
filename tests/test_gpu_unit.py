"""The unit seam of nn_ops.h on device pointers (nnc_attn_block / merge /
finish, nnc_rope_f32, nnc_rmsnorm*, nnc_softcap_f32) against the checker and
the reference's golden vectors -- the reference's own unit tests re-run on
the GPU."""
from __future__ import annotations

import os

import numpy as np
import pytest

import oracle as O
from golden import cases as G

pytestmark = pytest.mark.gpu

GOLDEN = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("kt", [O.KV_F32, O.KV_BF16, O.KV_F16])
@pytest.mark.parametrize("hd", [64, 36])
def test_attn_blocks_on_device(nncu, torch_cuda, kt, hd):
    """tests.cpp:2450-2497: blocks of 100, 256, 244 keys merged in order equal
    softmax attention over all 600, tolerance 1e-4 * (1 + |ref|)."""
    torch, N = torch_cuda, nncu
    rng = O.Rng(7)
    group, n_kv, n_keys = 3, 2, 600
    kvs = n_kv * hd
    q = rng.normal(group * hd)
    K = 2.0 * rng.normal(n_keys * kvs)
    V = rng.normal(n_keys * kvs)
    Kb, Vb = O.narrow(K, kt), O.narrow(V, kt)
    dq, dK, dV = dev(torch, q), dev(torch, Kb), dev(torch, Vb)
    pw = group * (hd + 2)
    acc = torch.zeros(pw, device="cuda")
    part = torch.zeros(pw, device="cuda")
    es = 4 if kt == O.KV_F32 else 2
    k0 = 0
    for n in (100, 256, 244):
        off = (k0 * kvs + hd) * es
        N.attn_block_dev(dq, hd, dK.data_ptr() + off, dV.data_ptr() + off, kt, kvs, n, hd, group,
                         1.0 / np.sqrt(hd), acc if k0 == 0 else part)
        if k0:
            N.attn_merge_dev(acc, part, hd, group)
        k0 += n
    out = torch.zeros(group * hd, device="cuda")
    N.attn_finish_dev(out, hd, acc, hd, group)
    got = out.cpu().numpy()
    Kf = O.widen(Kb, kt).reshape(n_keys, kvs)[:, hd:2 * hd].astype(np.float64)
    Vf = O.widen(Vb, kt).reshape(n_keys, kvs)[:, hd:2 * hd].astype(np.float64)
    s = (q.reshape(group, hd).astype(np.float64) @ Kf.T) / np.sqrt(hd)
    p = np.exp(s - s.max(1, keepdims=True))
    ref = ((p @ Vf) / p.sum(1, keepdims=True)).ravel()
    assert np.all(np.abs(got - ref) <= 1e-4 * (1.0 + np.abs(ref)))
    name = f"attn_blocks_{'f32' if kt == O.KV_F32 else 'bf16'}_{hd}"
    if kt != O.KV_F16:
        assert np.abs(got - GOLDEN[f"unit.{name}"]).max() <= 1e-5


def test_attn_block_partial_layout(nncu, torch_cuda):
    """A partial is (o, m, l) per head exactly as nnc_attn_block leaves it."""
    torch, N = torch_cuda, nncu
    rng = O.Rng(8)
    hd, group, n = 64, 4, 77
    q, K, V = rng.normal(group * hd), rng.normal(n * hd), rng.normal(n * hd)
    part = torch.zeros(group * (hd + 2), device="cuda")
    N.attn_block_dev(dev(torch, q), hd, dev(torch, K), dev(torch, V), O.KV_F32, hd, n, hd, group, 0.125, part,
                     softcap=30.0)
    want = O.attn_block(q, hd, K, V, O.KV_F32, hd, n, hd, group, 0.125, 30.0)
    got = part.cpu().numpy()
    w = want.reshape(group, hd + 2)
    g = got.reshape(group, hd + 2)
    assert np.allclose(g[:, hd], w[:, hd], atol=1e-6)             # m
    assert np.allclose(g[:, hd + 1], w[:, hd + 1], rtol=1e-5)     # l
    assert np.allclose(g[:, :hd], w[:, :hd], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("name", [n for n in G.UNIT_CASES if n.startswith("rope")])
def test_rope_on_device(nncu, torch_cuda, name):
    torch, N = torch_cuda, nncu
    a = G.unit_inputs(name)
    x = dev(torch, a["x"])
    ff = None if a["ff"] is None else dev(torch, a["ff"])
    # one token of H heads at position pos: pos0 = pos, pos_scale = 1
    N.rope_dev(x, 1, a["H"], a["D"], a["n_rot"], int(a["pos"]), 1.0, a["base"], a["mode"], ff)
    got = x.cpu().numpy()
    want = GOLDEN[f"unit.{name}"]
    assert np.abs(got - want).max() <= 2e-6 * max(1.0, np.abs(want).max()), np.abs(got - want).max()


@pytest.mark.parametrize("name", [n for n in G.UNIT_CASES if n.startswith("rmsnorm")])
def test_rmsnorm_gamma_on_device(nncu, torch_cuda, name):
    torch, N = torch_cuda, nncu
    a = G.unit_inputs(name)
    x, g = dev(torch, a["x"]), dev(torch, a["g"])
    y = torch.empty_like(x)
    N.rmsnorm_gamma_multi_dev(y, x, a["n"], a["dim"], g, 1e-6)
    want = GOLDEN[f"unit.{name}"]
    assert np.abs(y.cpu().numpy() - want).max() <= 1e-6 * max(1.0, np.abs(want).max())


def test_rmsnorm_plain_on_device(nncu, torch_cuda):
    torch, N = torch_cuda, nncu
    rng = O.Rng(0xCAFE)
    for n in (1536, 2560, 256, 13):
        x = rng.uniform(n, -3.0, 3.0)
        y = torch.empty(n, device="cuda")
        N.rmsnorm_dev(y, dev(torch, x), 1, n, 1e-6)
        assert np.allclose(y.cpu().numpy(), O.rmsnorm(x, 1e-6), rtol=1e-6, atol=1e-6)


def test_softcap_on_device(nncu, torch_cuda):
    torch, N = torch_cuda, nncu
    x = np.array([0.0, 1.0, -1.0, 5.0, -5.0, 30.0, 100.0, -100.0, 1e6], np.float32)
    y = torch.empty(9, device="cuda")
    N.softcap_dev(y, dev(torch, x), 9, 30.0)
    got = y.cpu().numpy()
    assert np.allclose(got, O.softcap(x, 30.0), rtol=1e-5, atol=1e-6)
    assert got[0] == 0.0 and 30.0 - 1e-3 <= got[8] <= 30.0
