#!/usr/bin/env python
"""Benchmark: libnnc's attention hot path on B200, in the reference's metric.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl nncu|reference] [--workload cfgN]

Workloads (synthetic seeded data, no dataset involved):
 cfg4 (default: the largest configuration that fits one GPU) Gemma-3-4B-shaped
      batched verify: 34 layers (5:1 local window 1024 / global), 8/4 heads
      of 256, 16 sequences at 32768 verifying 4 draft tokens, fp16 K/V, per-head
      Q/K RMSNorm. N GPUs: the (sequence, KV head) units sharded, no exchange
      (strong scaling).
 cfg1 Llama-3.2-1B-shaped single-layer decode: 32/8 heads of 64, 1024 cached
      keys (pre-rotated, NORM RoPE theta 5e5), fp32. N GPUs: replicas.
 cfg2 Gemma-3-1B-shaped 26-layer decode: 4 query heads, 1 KV head of 256,
      every 6th layer global (theta 1e6, 4097 keys), the rest sliding (window
      512, theta 1e4, a 768-row ring), per-head Q/K RMSNorm, fp32 K/V holding
      4096 positions, the new token at 4096. N GPUs: replicas.
 cfg3 Qwen3-4B-shaped causal prefill of one layer: 32/8 heads of 128, 2048
      tokens, Q/K RMSNorm, NEOX theta 1e6, bf16 cache. Metric: TFLOP/s.
 cfg5 Llama-3.2-1B-shaped long-context decode: 32/8 heads of 64, 131072
      cached fp16 keys, one new token. N GPUs: the keys split in 256-aligned
      runs, partials merged over NVLink (strong scaling).

One step = one decode (or verify, or prefill) step of the workload in the
drop-in's call pattern: one library call per layer, in layer order (layer
l + 1's inputs come from layer l's output in a real model), each call
holding every sequence of that layer -- nncu_attention_batch_dev, or
nncu_attention_split_dev for cfg5 on N > 1 GPUs.

Reported:
 value     the metric of the whole job (all ranks): algorithmic bytes (K/V of
           every key attended once per KV head, q in, output out) or flops
           (4 * n_head * head_dim per query-key pair) / device time of K steps
           (CUDA events, max over ranks). Inputs stay in HBM; steps rotate over
           R replicas of the workload's caches where one is smaller than L2.
 e2e       the same metric through the host-pointer call (nncu_attention_batch,
           one synchronous call per layer): host fp32 inputs copied up and
           outputs copied down inside every timed step.
 roofline  the attention kernel's achieved GB/s (TFLOP/s for cfg3) = its
           algorithmic work per launch / its mean launch time (CUDA events
           recorded by the library's phase profiler around each launch),
           against MEASURED_PEAKS.json.
 fused_layers  for reference only: every layer of a step in ONE call (a
           launch no real decode step can make, since the layers depend on
           each other through the projections).
 cpu_baseline  the reference's own CPU kernels (oracle/_ref) on the host's
           cores, a bounded sample of the same workload, at all cores and at
           the reference's default of min(8, cores) threads.
With --impl reference only the reference's CPU path runs (rank 0).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

GB = 1e9


# ---- workloads -------------------------------------------------------------------------------

class Layer:
    def __init__(self, n_head, n_kv, D, window, base, qk_norm, rope_mode=0):
        self.n_head, self.n_kv, self.D, self.window, self.base = n_head, n_kv, D, window, base
        self.qk_norm, self.rope_mode = qk_norm, rope_mode


class Workload:
    """The shapes of one benchmark configuration. shard: how N GPUs divide
    it -- "replicas" (each GPU the whole workload), "units" ((sequence, KV
    head) units dealt out), "keys" (the keys of the one sequence split)."""

    def __init__(self, name, title, layers, n_seqs, pos, n_tok, kv_type, dtype, replicas, shard="replicas",
                 metric="kv", seed=1, past_rotated=False):
        self.name, self.title, self.layers = name, title, layers
        self.n_seqs, self.pos, self.n_tok, self.kv_type, self.dtype = n_seqs, pos, n_tok, kv_type, dtype
        self.replicas, self.shard, self.metric, self.seed = replicas, shard, metric, seed
        self.past_rotated = past_rotated
        self.n_ctx = pos + n_tok
        self.esize = 4 if kv_type == 1 else 2

    def span(self, L, t):
        p = self.pos + t
        first = p + 1 - L.window if (L.window > 0 and p + 1 > L.window) else 0
        return first, p

    def union_keys(self, L) -> int:
        first = min(self.span(L, t)[0] for t in range(self.n_tok))
        last = max(self.span(L, t)[1] for t in range(self.n_tok))
        return last - first + 1

    def kv_bytes(self) -> int:
        """Algorithmic K/V bytes of one step: every key of the union of the
        tokens' spans, once per KV head, K and V."""
        return sum(self.union_keys(L) * L.n_kv * L.D * self.esize * 2 for L in self.layers) * self.n_seqs

    def q_out_bytes(self) -> int:
        return sum(2 * self.n_tok * L.n_head * L.D * 4 for L in self.layers) * self.n_seqs

    def step_bytes(self) -> int:
        return self.kv_bytes() + self.q_out_bytes()

    def step_flops(self) -> int:
        """4 * n_head * head_dim per (query, key) pair attended (QK^T and PV)."""
        total = 0
        for L in self.layers:
            for t in range(self.n_tok):
                f, l = self.span(L, t)
                total += 4 * L.n_head * L.D * (l - f + 1)
        return total * self.n_seqs

    def work(self) -> float:
        return float(self.step_flops() if self.metric == "flops" else self.step_bytes())

    @property
    def metric_name(self) -> str:
        return "prefill attn TFLOP/s" if self.metric == "flops" else "decode attn KV GB/s"

    @property
    def unit(self) -> str:
        return "TFLOP/s" if self.metric == "flops" else "GB/s"

    def rate(self, work: float, seconds: float) -> float:
        return work / seconds / (1e12 if self.metric == "flops" else GB)


def cfg1():
    return Workload("cfg1", "Llama-3.2-1B-shaped single-layer decode, 1024 cached keys, fp32 K/V",
                    [Layer(32, 8, 64, 0, 5e5, False, rope_mode=1)], n_seqs=1, pos=1024, n_tok=1, kv_type=1,
                    dtype="f32", replicas=32, seed=0, past_rotated=True)


def cfg2():
    layers = [Layer(4, 1, 256, 0 if (li + 1) % 6 == 0 else 512, 1e6 if (li + 1) % 6 == 0 else 1e4, True)
              for li in range(26)]
    return Workload("cfg2", "Gemma-3-1B-shaped 26-layer decode, context 4096, fp32 K/V", layers, n_seqs=1,
                    pos=4096, n_tok=1, kv_type=1, dtype="f32", replicas=8, seed=1)


def cfg3():
    return Workload("cfg3", "Qwen3-4B-shaped causal prefill of one layer, 2048 tokens, bf16 K/V",
                    [Layer(32, 8, 128, 0, 1e6, True)], n_seqs=1, pos=0, n_tok=2048, kv_type=0, dtype="bf16",
                    replicas=1, metric="flops", seed=2)


def cfg4():
    layers = [Layer(8, 4, 256, 0 if (li + 1) % 6 == 0 else 1024, 1e6 if (li + 1) % 6 == 0 else 1e4, True)
              for li in range(34)]
    return Workload("cfg4", "Gemma-3-4B-shaped batched verify, 16 sequences at 32768, 4 draft tokens, fp16 K/V",
                    layers, n_seqs=16, pos=32768, n_tok=4, kv_type=2, dtype="f32", replicas=1, shard="units",
                    seed=3)


def cfg5():
    return Workload("cfg5", "Llama-3.2-1B-shaped long-context decode, 131072 cached keys, fp16 K/V",
                    [Layer(32, 8, 64, 0, 5e5, False, rope_mode=1)], n_seqs=1, pos=131072, n_tok=1, kv_type=2,
                    dtype="f32", replicas=2, shard="keys", seed=4)


WORKLOADS = {"cfg1": cfg1, "cfg2": cfg2, "cfg3": cfg3, "cfg4": cfg4, "cfg5": cfg5}


KV_NAMES = {0: "bf16", 1: "f32", 2: "f16"}
L2_BYTES = 126e6


# ---- clocks (NVML, sampled in a thread during the timed region) ---------------------------------

class ClockSampler:
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting"}

    def __init__(self, index: int):
        self.samples = []
        self.ok = False
        try:
            import pynvml as nv
            nv.nvmlInit()
            self.nv = nv
            self.h = nv.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # NVML missing: report null clocks, never fake them
            self.err = str(e)
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((time.perf_counter(), mhz, reasons))
            except Exception:
                pass
            time.sleep(0.002)

    def start(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()

    def stop(self):
        if self._t:
            self._stop.set()
            self._t.join()

    def summary(self, t0: float, t1: float):
        if not self.ok:
            return None
        win = [s for s in self.samples if t0 <= s[0] <= t1]
        if not win:  # a very short region: the nearest samples
            win = sorted(self.samples, key=lambda s: abs(s[0] - (t0 + t1) / 2))[:3]
        reasons = set()
        for s in win:
            for bit, name in self.REASONS.items():
                if s[2] & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(s[1] for s in win) if win else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(win), "source": "nvml, 2 ms"}


# ---- what each rank does -----------------------------------------------------------------------

class Share:
    """One rank's part of a workload: its sequences, its KV heads per layer
    (the first kv0 .. kv0+n_kv of each layer's), its key range."""

    def __init__(self, w: Workload, rank: int, world: int):
        self.seqs = list(range(w.n_seqs))
        self.kv_frac = (0, 1)  # (group index, groups): this rank's slice of every layer's KV heads
        self.key_lo, self.key_hi = 0, w.n_ctx
        self.work_frac = 1.0
        if world > 1 and w.shard == "units":
            n_kv = w.layers[0].n_kv
            hg = min(world, n_kv)
            sg = world // hg
            assert n_kv % hg == 0 and w.n_seqs % sg == 0 and hg * sg == world
            self.kv_frac = (rank % hg, hg)
            per = w.n_seqs // sg
            self.seqs = list(range((rank // hg) * per, (rank // hg + 1) * per))
            self.work_frac = 1.0 / world
        elif world > 1 and w.shard == "keys":
            import libllmcpu_b200 as N
            self.key_lo, self.key_hi = N.split_ranges(w.n_ctx, world)[rank]
            self.work_frac = None  # the bytes of its key range

    def layer(self, L: Layer) -> Layer:
        g, n = self.kv_frac
        return Layer(L.n_head // n, L.n_kv // n, L.D, L.window, L.base, L.qk_norm, L.rope_mode)


def ring_rows(window: int, n_batch: int) -> int:
    return (window + max(n_batch, 1) + 255) // 256 * 256


def params_for(N, w: Workload, L: Layer, qg, kg):
    return N.params(n_tok=w.n_tok, pos0=w.pos, n_seq=w.pos + w.n_tok, n_head=L.n_head, n_kv=L.n_kv, head_dim=L.D,
                    rope_mode=L.rope_mode, freq_base=L.base, q_gamma=qg if L.qk_norm else None,
                    k_gamma=kg if L.qk_norm else None, window=L.window, eps=1e-6, scale=1.0 / np.sqrt(L.D))


def keep_range(w: Workload, L: Layer, share: Share):
    """The cached positions this rank's buffer of layer L holds before the step."""
    rows = ring_rows(L.window, w.n_tok) if L.window and ring_rows(L.window, w.n_tok) < w.n_ctx else w.n_ctx
    lo = max(0, w.pos - rows, share.key_lo)
    hi = min(w.pos, share.key_hi)
    return lo, max(lo, hi)


def rank_kv_bytes(w: Workload, share: Share) -> int:
    """K/V bytes this rank reads per step."""
    total = 0
    for L in w.layers:
        Ls = share.layer(L)
        first = max(min(w.span(L, t)[0] for t in range(w.n_tok)), share.key_lo)
        last = min(max(w.span(L, t)[1] for t in range(w.n_tok)), share.key_hi - 1)
        total += max(0, last - first + 1) * Ls.n_kv * Ls.D * w.esize * 2
    return total * len(share.seqs)


# ---- the product arm ---------------------------------------------------------------------------

def run_product(args, w: Workload, rank: int, world: int, local_rank: int):
    import torch

    import libllmcpu_b200 as N

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    share = Share(w, rank, world)
    layers = [share.layer(L) for L in w.layers]
    nsq = len(share.seqs)
    kv_rank = rank_kv_bytes(w, share)
    # steps rotate over R replicas of this rank's caches, together larger than L2
    R = max(w.replicas, int(np.ceil(2 * L2_BYTES / max(kv_rank, 1))))
    split = w.shard == "keys" and world > 1
    descs = [(L.n_kv, L.D, L.window, li) for li, L in enumerate(layers)]
    kv = N.KVCache(descs, n_ctx=w.n_ctx, n_batch=w.n_tok, n_seq=R * nsq, kv_type=w.kv_type, device=local_rank)
    gen = torch.Generator(device=dev)
    gen.manual_seed(w.seed * 1000 + rank)
    cache_dt = {0: torch.bfloat16, 1: torch.float32, 2: torch.float16}[w.kv_type]
    # the cached positions: N(0,1) rows (random keys stand in for rotated ones:
    # rotation does not change the work), the same in every replica
    for li, L in enumerate(layers):
        lo, hi = keep_range(w, L, share)
        for s in range(nsq):
            if hi <= lo:
                continue
            kb = torch.randn(hi - lo, L.n_kv * L.D, generator=gen, device=dev).to(cache_dt).contiguous()
            vb = torch.randn(hi - lo, L.n_kv * L.D, generator=gen, device=dev).to(cache_dt).contiguous()
            for r in range(R):
                kv.write_rows(li, lo, kb, vb, seq=r * nsq + s)
            del kb, vb
    torch.cuda.synchronize()

    # device-resident inputs, one set per replica (distinct memory, same values)
    host = []  # per (seq, layer): the host copies for the e2e leg
    dev_jobs, layer_jobs, keep = [], [], []
    rows_out = sum(w.n_tok * L.n_head for L in layers) * nsq
    for r in range(R):
        jobs = []
        for s in range(nsq):
            for li, L in enumerate(layers):
                if r == 0:
                    g = torch.Generator().manual_seed(w.seed * 7919 + 131 * s + li)
                    d = {"q": torch.randn(w.n_tok, L.n_head * L.D, generator=g),
                         "k": torch.randn(w.n_tok, L.n_kv * L.D, generator=g),
                         "v": torch.randn(w.n_tok, L.n_kv * L.D, generator=g),
                         "qg": 1.0 + 0.1 * torch.randn(L.D, generator=g),
                         "kg": 1.0 + 0.1 * torch.randn(L.D, generator=g)}
                    host.append({k: x.numpy() for k, x in d.items()})
                d = host[s * len(layers) + li]
                t = {k: torch.from_numpy(x).to(dev) for k, x in d.items()}
                out = torch.empty(w.n_tok, L.n_head * L.D, device=dev)
                p = params_for(N, w, L, t["qg"].data_ptr(), t["kg"].data_ptr())
                jobs.append(N.job(li, p, t["q"], t["k"], t["v"], None if split else out, seq=r * nsq + s))
                keep.append((t, out))
        dev_jobs.append((N.AttnJob * len(jobs))(*jobs))
        # the drop-in's pattern: one call per layer, every sequence of the layer in it
        layer_jobs.append([(N.AttnJob * nsq)(*[jobs[s * len(layers) + li] for s in range(nsq)])
                           for li in range(len(layers))])
    stream = torch.cuda.Stream(device=dev)
    dist = None
    if world > 1:
        import torch.distributed as dist
    grp = N.SplitGroup(rank, world, max_rows=rows_out, head_dim=layers[0].D, device=local_rank) if split else None

    def step(i):
        for arr in layer_jobs[i % R]:  # layer by layer, in order
            if grp:
                grp.attention(kv, arr, share.key_lo, share.key_hi, stream)
            else:
                kv.attention_batch_dev(arr, stream)

    def fused_step(i):  # every layer in one call: not a pattern a real decode step allows
        if grp:
            grp.attention(kv, dev_jobs[i % R], share.key_lo, share.key_hi, stream)
        else:
            kv.attention_batch_dev(dev_jobs[i % R], stream)

    for i in range(args.warmup):
        step(i)
    kv.sync(stream)
    torch.cuda.synchronize()

    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.05)
    # ---- the timed region: exactly K steps, barrier + synchronize on both sides ----
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = N.launch_count()
    t_wall0 = time.perf_counter()
    ev0.record(stream)
    for i in range(args.steps):
        step(i)
    ev1.record(stream)
    kv.sync(stream)
    torch.cuda.synchronize()
    t_wall1 = time.perf_counter()
    if dist:
        dist.barrier()
    launches = N.launch_count() - launches0
    ms = ev0.elapsed_time(ev1)
    if dist:
        tm = torch.tensor([ms], device=dev)
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
        ms = float(tm.item())
    time.sleep(0.01)
    sampler.stop()
    clocks = sampler.summary(t_wall0, t_wall1)
    ms_per_step = ms / args.steps
    job_work = w.work() * (world if w.shard == "replicas" else 1)
    value = w.rate(job_work, ms_per_step * 1e-3)

    # ---- roofline: the attention kernel's own launch time, from the phase profiler ----
    N.perf_reset()
    N.perf_enable(True)
    for i in range(args.steps):
        step(i)
    kv.sync(stream)
    ph = N.perf_read()
    N.perf_enable(False)
    core = ph["attn_core"]
    rope = ph["attn_rope"]
    core_us = 1e3 * core["ms"] / max(core["calls"], 1)
    launches_per_step = max(core["calls"], 1) / args.steps
    peaks = measured_peaks()
    if w.metric == "flops":
        flops = w.step_flops() / launches_per_step  # replicas: the whole workload per rank
        achieved = flops / (core_us * 1e-6) / 1e12
        roofline = {"bound": "tensor", "achieved": round(achieved, 3), "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                    "frac": round(achieved / peaks["bf16_tflops"], 5), "traffic": None, "flops_per_launch": int(flops)}
    else:
        core_bytes = core["bytes"] / max(core["calls"], 1)
        achieved = core_bytes / (core_us * 1e-6) / GB
        roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                    "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": profiled_traffic(w.name),
                    "bytes_per_launch": int(core_bytes)}
    # which kernel the library launches for this workload: the tensor-core
    # prefill, the tensor-core decode (16-bit cache, 3+ query rows per KV head,
    # not split), or the CUDA-core decode
    L0 = layers[0]
    rows = (L0.n_head // L0.n_kv) * w.n_tok
    if w.metric == "flops":
        kernel = "prefill_kernel (tcgen05 Q K^T and P V, TMEM softmax), after prefill_prep_kernel"
    elif w.kv_type in (0, 2) and rows >= 3 and not split:
        kernel = "decode_tc_kernel (tcgen05 K Q^T and V^T P^T, split-KV merge, fused append)"
    else:
        kernel = "decode_kernel (CUDA cores: split-KV attention, merge, fused append)"
    roofline.update({"kernel": kernel,
                     "peak_source": peaks["source"], "us_per_launch": round(core_us, 3),
                     "attn_rope_us_per_launch": round(1e3 * rope["ms"] / max(rope["calls"], 1), 3)})

    # ---- for reference: the same steps with every layer in one call ----
    fused = None
    if len(layers) > 1:
        for i in range(args.warmup):
            fused_step(i)
        kv.sync(stream)
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        ev0.record(stream)
        for i in range(args.steps):
            fused_step(i)
        ev1.record(stream)
        kv.sync(stream)
        fms = ev0.elapsed_time(ev1)
        if dist:
            tm = torch.tensor([fms], device=dev)
            dist.all_reduce(tm, op=dist.ReduceOp.MAX)
            fms = float(tm.item())
        fused = {"value": round(w.rate(job_work, fms / args.steps * 1e-3), 3), "unit": w.unit,
                 "ms_per_step": round(fms / args.steps, 5),
                 "note": "all layers of a step in one launch; not the drop-in's call pattern"}

    # ---- e2e: host fp32 inputs up and outputs down inside every step ----
    e2e = run_e2e(args, w, N, kv, layers, share, host, grp, stream, dist, dev)
    e2e["value"] = round(w.rate(job_work, e2e.pop("seconds_per_step")), 3)

    line = {
        "metric": w.metric_name, "value": round(value, 3), "unit": w.unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
        "higher_is_better": True, "scaling": "weak" if w.shard == "replicas" else "strong", "vs_baseline": None,
        "dtype": w.dtype,
        "data": "synthetic (seeded N(0,1) q/k/v and K/V cache; gains 1+N(0,0.1))",
        "config": {"workload": f"{w.name}: {w.title}", "layers": len(w.layers), "n_head": w.layers[0].n_head,
                   "n_kv": w.layers[0].n_kv, "head_dim": w.layers[0].D, "kv_type": KV_NAMES[w.kv_type],
                   "sequences": w.n_seqs, "context": w.pos, "new_tokens": w.n_tok,
                   "work_per_step": int(w.work()), "work_unit": "flop" if w.metric == "flops" else "byte",
                   "l2": f"{R} rotating replicas of the caches ({kv_rank * R / 1e6:.0f} MB read per rotation "
                         f"per GPU) > L2",
                   "parallelism": {"replicas": f"replicas x{world}", "units": f"(sequence, KV head) units / {world}",
                                   "keys": f"keys split / {world}, merge over NVLink"}[w.shard]
                   if world > 1 else "single GPU"},
        "roofline": roofline, "e2e": e2e, "gpu_launches": int(launches), "clocks": clocks,
        "calls_per_step": len(layers),
    }
    if fused:
        line["fused_layers"] = fused
    if w.metric != "flops":
        line["hbm_frac"] = round(value / world / peaks["hbm_gbs"], 4)
    if dist:
        dist.barrier()  # every rank's calls are done before any group memory goes
    if grp:
        grp.close()
    kv.close()
    return line


def _placed(carve, x):
    """x copied into a fresh view of the arena that `carve` cuts."""
    v = carve(x.size).reshape(x.shape)
    v[...] = x
    return v


def run_e2e(args, w: Workload, N, kv, layers, share: Share, host, grp, stream, dist, dev):
    """The same steps through the host-pointer path: nncu_attention_batch with
    host fp32 buffers (views of one arena the caller registered once with
    nncu_host_register: the call gathers the inputs up and scatters the outputs
    down through the GPU's mapping of that memory), or, for a split, pinned
    host inputs copied up, the split call, and the merged output copied down.
    Wall clock of the synchronous steps, max over ranks."""
    import torch

    nsq, nl = len(share.seqs), len(layers)
    h2d = sum(d["q"].nbytes + d["k"].nbytes + d["v"].nbytes + (d["qg"].nbytes + d["kg"].nbytes if L.qk_norm else 0)
              for i, d in enumerate(host) for L in [layers[i % nl]])
    rows_out = sum(w.n_tok * L.n_head for L in layers) * nsq
    d2h = rows_out * layers[0].D * 4
    if grp is None:
        # every host buffer a view of one arena, 16-byte aligned (registration
        # pins whole pages, so small buffers share one registered range)
        sizes = [x.size for d in host for x in d.values()]
        sizes += [w.n_tok * L.n_head * L.D for _ in range(nsq) for L in layers]
        arena = np.zeros(sum((n + 3) // 4 * 4 for n in sizes) + 4, np.float32)
        off = (-arena.ctypes.data // 4) % 4

        def carve(n):
            nonlocal off
            v = arena[off:off + n]
            off += (n + 3) // 4 * 4
            return v

        host = [{k: _placed(carve, x) for k, x in d.items()} for d in host]
        per_layer, outs = [], []
        for li, L in enumerate(layers):
            jobs = []
            for s in range(nsq):
                d = host[s * nl + li]
                out = carve(w.n_tok * L.n_head * L.D).reshape(w.n_tok, L.n_head * L.D)
                p = params_for(N, w, L, d["qg"], d["kg"])
                jobs.append(N.job(li, p, d["q"], d["k"], d["v"], out, seq=s))
                outs.append(out)
            # the job table a caller keeps; its host buffers change per step
            per_layer.append((N.AttnJob * len(jobs))(*jobs))
        # the caller's host buffers live as long as its session: pinned once
        # (nncu_host_register), so each call reads its inputs and writes its
        # outputs through the GPU's mapping of that memory
        N.host_register(arena)

        def one():
            for arr in per_layer:  # layer by layer: each call returns with its outputs in host memory
                kv.attention_batch(arr)
        api = ("nncu_attention_batch (host pointers, one arena registered once with nncu_host_register), "
               "one synchronous call per layer")
    else:
        pinned, devs, jobs = [], [], []
        for s in range(nsq):
            for li, L in enumerate(layers):
                d = host[s * nl + li]
                hp = {k: torch.from_numpy(d[k]).pin_memory() for k in ("q", "k", "v")}
                dd = {k: torch.empty_like(hp[k], device=dev) for k in ("q", "k", "v")}
                g = {k: torch.from_numpy(d[k]).to(dev) for k in ("qg", "kg")}
                p = params_for(N, w, L, g["qg"].data_ptr(), g["kg"].data_ptr())
                jobs.append(N.job(li, p, dd["q"], dd["k"], dd["v"], None, seq=s))
                pinned.append(hp)
                devs.append((dd, g))
        arr = (N.AttnJob * len(jobs))(*jobs)

        def one():
            with torch.cuda.stream(stream):
                for hp, (dd, _) in zip(pinned, devs):
                    for k in ("q", "k", "v"):
                        dd[k].copy_(hp[k], non_blocking=True)
            grp.attention(kv, arr, share.key_lo, share.key_hi, stream)
            grp.read_output(rows_out * layers[0].D, stream)
        api = "host inputs up + nncu_attention_split_dev + nncu_group_copy_output down"
    # warm up to a steady state (the host path's first few hundred calls run
    # slower than the rest): at least W steps and a third of a second on one
    # GPU; a fixed count on several, where every rank must take the same steps
    if dist:
        for _ in range(max(args.warmup, 100)):
            one()
        dist.barrier()
    else:
        n_warm, t_warm = 0, time.perf_counter() + 0.33
        while n_warm < args.warmup or time.perf_counter() < t_warm:
            one()
            n_warm += 1
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one()
    t = time.perf_counter() - t0
    if dist:
        te = torch.tensor([t], device=dev)
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
        t = float(te.item())
    if grp is None:
        N.host_unregister(arena)
    return {"unit": w.unit, "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
            "ms_per_step": round(1e3 * t / args.steps, 4), "api": api, "seconds_per_step": t / args.steps}


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "source": "of measured (MEASURED_PEAKS.json)"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "of fallback"}


def profiled_traffic(workload: str):
    """DRAM bytes per launch of the attention kernel from the committed ncu
    summary (profiles/); None if absent."""
    p = os.path.join(ROOT, "profiles", f"decode_{workload}_traffic.json")
    try:
        with open(p) as f:
            return json.load(f)["dram_bytes_per_launch"]
    except Exception:
        return None


# ---- the reference's CPU path ------------------------------------------------------------------

def default_threads() -> int:
    """The reference's default thread count: min(8, CPUs) (nnc.h:100-104)."""
    return min(8, os.cpu_count() or 1)


def cpu_reference(w: Workload, budget_s: float, threads: int | None):
    """The reference's own kernels (oracle/_ref), parallel through its pool,
    over a bounded sample of the workload (all of it, or one sequence of a
    many-sequence batch); falls back to the C restatement (one thread) where
    the reference was not built. Returns (rate, cores, kind, sample, s/step)."""
    import oracle as O

    which, kind = ("ref", "reference") if O.ref() is not None else ("oracle", "port")
    cores = 1
    if which == "ref":
        n = threads or min(64, os.cpu_count() or 1)
        O.ref().ref_set_num_threads(n)
        cores = O.ref().ref_num_threads()
    n_seqs = 1  # every sequence is the same work; one stands for all
    rng = np.random.default_rng(w.seed)
    kt = w.kv_type if w.kv_type != 2 else 1  # no F16 cache in the reference: the F16 values widened to F32
    layers = []
    for L in w.layers:
        d = {"q": rng.standard_normal((w.n_tok, L.n_head * L.D), np.float32),
             "k": rng.standard_normal((w.n_tok, L.n_kv * L.D), np.float32),
             "v": rng.standard_normal((w.n_tok, L.n_kv * L.D), np.float32),
             "qg": (1.0 + 0.1 * rng.standard_normal(L.D, np.float32)).astype(np.float32),
             "kg": (1.0 + 0.1 * rng.standard_normal(L.D, np.float32)).astype(np.float32)}
        rows = ring_rows(L.window, w.n_tok) if L.window and ring_rows(L.window, w.n_tok) < w.n_ctx else w.n_ctx
        keep0 = max(0, w.pos - rows)
        n = w.pos - keep0
        dt = np.float32 if kt == 1 else np.uint16
        Kc = np.zeros((rows, L.n_kv * L.D), dt)
        Vc = np.zeros_like(Kc)
        if n:
            r = (keep0 + np.arange(n)) % rows
            for buf in (Kc, Vc):
                x = rng.standard_normal((n, L.n_kv * L.D), np.float32)
                if w.kv_type == 2:
                    x = x.astype(np.float16).astype(np.float32)
                buf[r] = O.narrow(x, kt) if kt != 1 else x
        d["Kc"], d["Vc"], d["rows"] = Kc, Vc, rows
        d["p"] = O.params(n_tok=w.n_tok, pos0=w.pos, n_seq=w.pos + w.n_tok, n_head=L.n_head, n_kv=L.n_kv,
                          head_dim=L.D, rope_mode=L.rope_mode, freq_base=L.base,
                          q_gamma=d["qg"] if L.qk_norm else None, k_gamma=d["kg"] if L.qk_norm else None,
                          window=L.window, scale=1.0 / np.sqrt(L.D))
        layers.append(d)

    def one_step():
        for d in layers:
            O.attention_forward(d["p"], d["q"], d["k"], d["v"], d["Kc"], d["Vc"], kt, d["rows"], which=which)

    one_step()  # warm
    n_steps, t0 = 0, time.perf_counter()
    while True:
        one_step()
        n_steps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or n_steps >= 100000:
            break
    work = w.work() / w.n_seqs * n_seqs
    rate = w.rate(work * n_steps, el)
    sample = f"{n_steps} steps ({el:.1f} s) of {w.name}"
    if w.n_seqs > 1:
        sample += f", one of its {w.n_seqs} sequences per step"
    if w.kv_type == 2:
        sample += ", F16 cache widened to F32 (the reference has no F16 cache)"
    return rate, cores, kind, sample, el / n_steps


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["nncu", "reference"], default="nncu")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="cfg4")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline sample length")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sequences", type=int, default=None,
                    help="profiling aid: fewer sequences than the workload names (the line's config says so)")
    args = ap.parse_args(argv)
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    w = WORKLOADS[args.workload]()
    if args.sequences:
        w.n_seqs = args.sequences
        w.title += f" (reduced to {args.sequences} sequences)"

    if args.impl == "reference":
        if rank != 0:
            return 0
        budget = max(5.0, min(60.0, args.cpu_seconds))
        rate, cores, kind, sample, s_per_step = cpu_reference(w, budget, None)
        d_rate, d_cores, _, d_sample, _ = cpu_reference(w, budget / 2, default_threads())
        line = {"impl": "reference", "metric": w.metric_name, "value": round(rate, 4), "unit": w.unit,
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(1e3 * s_per_step, 4), "higher_is_better": True,
                "scaling": "weak" if w.shard == "replicas" else "strong", "vs_baseline": None, "dtype": w.dtype,
                "data": "synthetic", "config": {"workload": f"{w.name}: {w.title}", "work_per_step": int(w.work())},
                "cpu_baseline": {"value": round(rate, 4), "unit": w.unit, "cores": cores, "kind": kind,
                                 "sample": sample, "host_cpus": os.cpu_count(),
                                 "at_default_threads": {"value": round(d_rate, 4), "cores": d_cores,
                                                        "sample": d_sample}},
                "e2e": {"value": round(rate, 4), "unit": w.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    line = run_product(args, w, rank, world, local_rank)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, cores, kind, sample, _ = cpu_reference(w, args.cpu_seconds, None)
        d_rate, d_cores, _, d_sample, _ = cpu_reference(w, args.cpu_seconds / 2, default_threads())
        line["cpu_baseline"] = {"value": round(rate, 4), "unit": w.unit, "cores": cores, "kind": kind,
                                "sample": sample, "host_cpus": os.cpu_count(),
                                "at_default_threads": {"value": round(d_rate, 4), "cores": d_cores,
                                                       "sample": d_sample}}
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
