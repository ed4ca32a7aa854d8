"""One sequence split over two GPUs through the C ABI (nncu_group,
nncu_attention_split_dev): BASELINE config 5's shape in small (32 query heads
on 8 KV heads of 64, fp16 cache, 4096 keys), each GPU's merged output against
the checker on the whole sequence. Four decode steps in a row, so both
parities' receive buffers and counters are used twice; and the failure path:
a dropped arrival makes every GPU's bounded merge wait run out (50 ms), the
group stays poisoned until the ranks reset it together, and the calls after
the reset are correct again. Needs two GPUs of one node; skipped otherwise."""
from __future__ import annotations

import socket

import numpy as np
import pytest

import oracle as O
from oracle import scenarios as S
from oracle.scenarios import LayerSpec

from gpu_helpers import assert_close

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run_ranks(target, torch, *extra):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    qd = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, 2, port, qd) + extra) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, outs, err = qd.get(timeout=300)
        assert outs is not None, err
        res[r] = outs
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return res


def _checker(steps):
    """The checker over the whole sequence: decode steps at the given
    (position, inputs step) pairs in order, each appending its token."""
    import split_workers as W

    layer = LayerSpec(32, 8, 64, freq_base=5e5, rope_mode=O.ROPE_NORM)
    n_ctx = 4096 + 8
    case = S.build_case(4, [layer], n_ctx=n_ctx, n_tok=1, pos0=4096, kv_type=O.KV_F16, n_batch=1, rotate_past=True)
    from oracle.scenarios import cache_bits
    Kc, Vc = cache_bits(case, 0, 0)
    want = []
    for pos, step in steps:
        q, k, v = W.step_inputs(step, case)
        d = case.params_dict(0, 0)
        d.update(pos0=pos, n_seq=pos + 1)
        out, _, _ = O.attention_forward(O.orc_params(**d), np.array(q), np.array(k), np.array(v), Kc, Vc, O.KV_F16,
                                        case.rows[0])
        want.append(out.reshape(-1))
    return want


def _need_two(torch):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs of one node")


def test_split_over_two_gpus_matches_the_whole(nncu, torch_cuda):
    _need_two(torch_cuda)
    import split_workers as W

    res = _run_ranks(W.gpu_rank, torch_cuda, 4)
    want = _checker([(4096 + s, s) for s in range(4)])
    for r in range(2):
        for step in range(4):
            assert_close(res[r][step], want[step], f"rank {r} step {step}")


def test_split_timeout_poisons_until_reset(nncu, torch_cuda):
    _need_two(torch_cuda)
    import split_workers as W

    res = _run_ranks(W.gpu_rank_timeout, torch_cuda)
    want = _checker([(4096, 0), (4097, 3), (4098, 4)])
    for r in range(2):
        statuses = [st for _, _, st, _ in res[r]]
        # step 1: the dropped arrival runs every GPU's wait out; step 2: poisoned
        assert statuses == [0, nncu.ERR_TIMEOUT, nncu.ERR_TIMEOUT, 0, 0], (r, statuses)
        ok = [(pos, got) for _, pos, st, got in res[r] if st == 0]
        assert [pos for pos, _ in ok] == [4096, 4097, 4098]
        for (pos, got), w in zip(ok, want):
            assert_close(got, w, f"rank {r} position {pos}")
