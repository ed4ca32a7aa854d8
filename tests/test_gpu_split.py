"""One sequence split over two GPUs through the C ABI (nncu_group,
nncu_attention_split_dev): BASELINE config 5's shape in small (32 query heads
on 8 KV heads of 64, fp16 cache, 4096 keys), two decode steps in a row, each
GPU's merged output against the checker on the whole sequence. Needs two
GPUs of one node; skipped otherwise."""
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


def test_split_over_two_gpus_matches_the_whole(nncu, torch_cuda):
    torch = torch_cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs of one node")
    import torch.multiprocessing as mp

    import split_workers as W

    ctx = mp.get_context("spawn")
    qd = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=W.gpu_rank, args=(r, 2, port, qd)) for r in range(2)]
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

    # the checker over the whole sequence, both steps
    layer = LayerSpec(32, 8, 64, freq_base=5e5, rope_mode=O.ROPE_NORM)
    case = S.build_case(4, [layer], n_ctx=4098, n_tok=1, pos0=4096, kv_type=O.KV_F16, n_batch=1, rotate_past=True)
    outs, caches = S.run_checker(case)
    Kc, Vc = caches[0][0]
    want = [outs[0][0].reshape(-1)]
    q, k, v, _ = res[0][1]
    d = case.params_dict(0, 0)
    d.update(pos0=4097, n_seq=4098)
    out2, _, _ = O.attention_forward(O.orc_params(**d), np.array(q), np.array(k), np.array(v), Kc, Vc, O.KV_F16,
                                     case.rows[0])
    want.append(out2.reshape(-1))
    for r in range(2):
        for step in range(2):
            assert_close(res[r][step][3], want[step], f"rank {r} step {step}")
