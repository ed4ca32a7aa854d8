"""Rank bodies for the split tests (run in child processes; test
infrastructure). A rank sets up its own process group over 127.0.0.1 and
reports through a queue."""
from __future__ import annotations

import os
import traceback

import numpy as np


def _init(rank: int, world: int, port: int, backend: str = "gloo"):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group(backend, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    return dist


def cpu_rank(rank: int, world: int, port: int, q, K, V, n_keys: int, D: int, H: int, scale: float, out_q):
    """This rank's keys through the reference's unit functions (256-key blocks
    merged in order, attend_blocks), the ranks' partials gathered and merged
    in rank order, then finished; also the group-handle exchange."""
    try:
        import torch

        import libllmcpu_b200 as N
        import oracle as O

        dist = _init(rank, world, port)
        try:
            lo, hi = N.split_ranges(n_keys, world)[rank]
            acc = None
            for b0 in range(lo, hi, 256):
                nk = min(256, hi - b0)
                part = O.attn_block(q, D, K, V, O.KV_F32, D, nk, D, H, scale, k_offset_elems=b0 * D)
                acc = part if acc is None else O.attn_merge(acc, part, D, H)
            parts = [torch.zeros(acc.size, dtype=torch.float32) for _ in range(world)]
            dist.all_gather(parts, torch.from_numpy(acc))
            merged = parts[0].numpy()
            for r in range(1, world):
                merged = O.attn_merge(merged, parts[r].numpy(), D, H)
            out = O.attn_finish(merged, D, H)
            handles = N.exchange_handles(bytes([rank + 1]) * N.GROUP_HANDLE_BYTES, world)
            out_q.put((rank, out, [h[0] for h in handles]))
        finally:
            dist.destroy_process_group()
    except Exception:
        out_q.put((rank, None, traceback.format_exc()))


def _split_setup(rank: int, world: int, n_ctx: int):
    import torch

    import libllmcpu_b200 as N
    import oracle as O
    from oracle import scenarios as S
    from oracle.scenarios import LayerSpec

    layer = LayerSpec(32, 8, 64, freq_base=5e5, rope_mode=O.ROPE_NORM)
    case = S.build_case(4, [layer], n_ctx=n_ctx, n_tok=1, pos0=4096, kv_type=O.KV_F16, n_batch=1,
                        rotate_past=True)
    inp = case.inputs[0][0]
    lo, hi = N.split_ranges(n_ctx, world)[rank]
    kv = N.KVCache(case.layer_descs(), n_ctx=n_ctx, n_batch=1, kv_type=O.KV_F16, device=rank)
    own = slice(lo, min(hi, 4096))
    kv.write_rows(0, own.start, O.narrow(inp.past_k[own], O.KV_F16), O.narrow(inp.past_v[own], O.KV_F16))
    grp = N.SplitGroup(rank, world, max_rows=32, head_dim=64, device=rank)
    return case, kv, grp, lo, hi, torch.cuda.Stream()


def step_inputs(step: int, case):
    """The projections of decode step `step` (position 4096 + step): the
    case's own for step 0, then drawn from a fixed stream."""
    import oracle as O

    if step == 0:
        inp = case.inputs[0][0]
        return inp.q, inp.k, inp.v
    rng = O.Rng(40 + step)
    return (rng.normal(32 * 64).reshape(1, 32 * 64), rng.normal(8 * 64).reshape(1, 8 * 64),
            rng.normal(8 * 64).reshape(1, 8 * 64))


def _split_call(N, case, kv, grp, lo, hi, st, step: int, pos: int):
    import torch

    q, k, v = step_inputs(step, case)
    dq, dk, dv = (torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (q, k, v))
    d = case.params_dict(0, 0)
    d.update(pos0=pos, n_seq=pos + 1)
    job = N.job(0, N.params(**d), dq, dk, dv, None, seq=0)
    torch.cuda.synchronize()
    grp.attention(kv, [job], lo, hi, st)
    try:
        kv.sync(st)
        status = 0
    except N.NnncError as e:
        status = e.status
    return status, grp.read_output(32 * 64, st)


def gpu_rank(rank: int, world: int, port: int, out_q, n_steps: int = 4):
    """BASELINE config 5 in small: 32 query heads on 8 KV heads of 64, fp16
    cache, 4096 cached keys; n_steps decode steps (positions 4096, 4097, ...)
    with the keys split over the ranks, so that both parities' receive
    buffers and counters are reused; each rank reports its merged outputs."""
    try:
        import torch

        import libllmcpu_b200 as N

        torch.cuda.set_device(rank)
        dist = _init(rank, world, port)
        try:
            case, kv, grp, lo, hi, st = _split_setup(rank, world, 4096 + n_steps)
            outs = []
            for step in range(n_steps):
                status, got = _split_call(N, case, kv, grp, lo, hi, st, step, 4096 + step)
                if status:
                    raise RuntimeError(f"step {step}: status {status}")
                outs.append(got)
            dist.barrier()
            grp.close()
            kv.close()
            out_q.put((rank, outs, None))
        finally:
            dist.destroy_process_group()
    except Exception:
        out_q.put((rank, None, traceback.format_exc()))


def gpu_rank_timeout(rank: int, world: int, port: int, out_q):
    """The split's failure path on two GPUs, with no device fault: the group's
    merge wait is cut to 50 ms; at step 1 the last rank's partials are stored
    but never counted (a dropped message, injected on the host side), so
    every GPU's merge runs out of time; step 2 then fails at once on the
    poisoned groups; the ranks wait for their calls, meet, reset the group and
    meet again; steps 3 and 4 are correct. Reports each step's status and
    output."""
    try:
        import torch

        import libllmcpu_b200 as N

        torch.cuda.set_device(rank)
        dist = _init(rank, world, port)
        try:
            case, kv, grp, lo, hi, st = _split_setup(rank, world, 4101)
            grp.set_timeout(50)
            res = []
            pos = 4096
            for step in range(5):
                if step == 1 and rank == world - 1:
                    grp.inject_drop(1)
                if step == 3:
                    # recovery at a step boundary: no call in flight anywhere
                    dist.barrier()
                    grp.reset()
                    dist.barrier()
                status, got = _split_call(N, case, kv, grp, lo, hi, st, step, pos)
                res.append((step, pos, status, got))
                if status == 0:
                    kv.commit(pos, 1)
                    pos += 1
            dist.barrier()
            grp.close()
            kv.close()
            out_q.put((rank, res, None))
        finally:
            dist.destroy_process_group()
    except Exception:
        out_q.put((rank, None, traceback.format_exc()))
