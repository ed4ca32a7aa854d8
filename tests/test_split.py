"""One sequence split over ranks, host side, on the CPU: the key ranges each
rank holds, and the rank-order log-sum-exp merge of the ranks' partials
(the reference's nnc_attn_block / nnc_attn_merge / nnc_attn_finish over
256-key blocks, nn_ops.cpp:351-499, grouped by rank), over two gloo ranks
that also exchange group handles the way SplitGroup does."""
from __future__ import annotations

import socket

import numpy as np
import pytest

import libllmcpu_b200 as N
import oracle as O


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("n_keys,world", [(131073, 2), (131073, 4), (131073, 8), (4098, 2), (513, 2)])
def test_split_ranges_cover_the_keys_in_256_aligned_runs(n_keys, world):
    ranges = N.split_ranges(n_keys, world)
    assert len(ranges) == world
    assert ranges[0][0] == 0 and ranges[-1][1] == n_keys
    for (lo, hi), (lo2, _) in zip(ranges, ranges[1:]):
        assert hi == lo2 and lo % 256 == 0 and hi > lo
    sizes = [hi - lo for lo, hi in ranges]
    assert all(sz == sizes[0] for sz in sizes[:-1]) and sizes[-1] <= sizes[0]  # equal runs, the last one short
    assert sizes[0] % 256 == 0 and sizes[0] - 256 < -(-n_keys // world)


def test_split_ranges_refuse_an_empty_rank():
    with pytest.raises(ValueError):
        N.split_ranges(300, 4)


def test_two_ranks_merge_like_one(tmp_path):
    import torch.multiprocessing as mp

    import split_workers as W

    D, H, n_keys = 64, 4, 2500
    rng = O.Rng(5)
    q = rng.normal(H * D)
    K = rng.normal(n_keys * D)
    V = rng.normal(n_keys * D)
    scale = 1.0 / 8.0
    # one rank: every 256-key block merged in order (attend_blocks)
    acc = None
    for b0 in range(0, n_keys, 256):
        part = O.attn_block(q, D, K, V, O.KV_F32, D, min(256, n_keys - b0), D, H, scale, k_offset_elems=b0 * D)
        acc = part if acc is None else O.attn_merge(acc, part, D, H)
    want = O.attn_finish(acc, D, H)

    ctx = mp.get_context("spawn")
    qd = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=W.cpu_rank, args=(r, 2, port, q, K, V, n_keys, D, H, scale, qd)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, out, extra = qd.get(timeout=120)
        assert out is not None, extra
        res[r] = (out, extra)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        out, handles = res[r]
        np.testing.assert_allclose(out, want, rtol=0, atol=2e-6)
        assert handles == [1, 2]  # every rank saw every rank's handle, in rank order
