#!/usr/bin/env python
"""Benchmark: libnnc's decode attention on B200, in the reference's metric.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl nncu|reference] [--workload cfg2]

Workload (the config the metric is quoted on): a
Gemma-3-1B-shaped 26-layer decode step -- 4 query heads, 1 KV head, head_dim
256, every 6th layer global (RoPE theta 1e6, 4097 keys) and the rest sliding
(window 512, theta 1e4, a 768-row ring), per-head Q/K RMSNorm with gains
~1+N(0,0.1), fp32 K/V cache holding 4096 positions, the new token at 4096.
Synthetic seeded data (no public dataset is involved). One step = the
attention of all 26 layers for one token: K1 (norms, RoPE, append) and K2+K3
(split-KV attention with its merge), submitted as one nncu_attention_batch_dev
call (two kernel launches).

Reported:
 value     KV GB/s of the whole job: algorithmic bytes (K/V of every key
           attended, q in, output out) of all ranks / device time of K steps
           (CUDA events, max over ranks). Inputs stay in HBM; consecutive steps
           rotate over R replicas of the whole cache (R * 70 MB > L2), so each
           step reads from HBM, not L2.
 e2e       the same metric through the host-pointer C-ABI call
           (nncu_attention_batch): host fp32 inputs copied up and outputs
           copied down inside every timed step (wall clock of the synchronous
           call).
 roofline  attn_core (K2+K3) achieved GB/s = its algorithmic bytes per launch
           / its mean launch time (CUDA events recorded by the library's phase
           profiler around the launch), against MEASURED_PEAKS.json's HBM copy.
 cpu_baseline  the reference's own CPU kernels (oracle/_ref) on the host's
           cores, a bounded sample of the same workload.
With --impl reference only the reference's CPU path runs (rank 0).
"""
from __future__ import annotations

import argparse
import ctypes as C
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
    """The shapes of one benchmark configuration."""

    def __init__(self, name, title, layers, n_seqs, pos, n_tok, kv_type, dtype, replicas):
        self.name, self.title, self.layers = name, title, layers
        self.n_seqs, self.pos, self.n_tok, self.kv_type, self.dtype = n_seqs, pos, n_tok, kv_type, dtype
        self.replicas = replicas
        self.n_ctx = pos + n_tok
        self.esize = 4 if kv_type == 1 else 2

    def span(self, L, t):
        p = self.pos + t
        first = p + 1 - L.window if (L.window > 0 and p + 1 > L.window) else 0
        return first, p

    def kv_bytes(self) -> int:
        """Algorithmic K/V bytes of one step: every key of the union of the
        tokens' spans, once per KV head, K and V."""
        total = 0
        for L in self.layers:
            first = min(self.span(L, t)[0] for t in range(self.n_tok))
            last = max(self.span(L, t)[1] for t in range(self.n_tok))
            total += (last - first + 1) * L.n_kv * L.D * self.esize * 2
        return total * self.n_seqs

    def q_out_bytes(self) -> int:
        return sum(2 * self.n_tok * L.n_head * L.D * 4 for L in self.layers) * self.n_seqs

    def step_bytes(self) -> int:
        return self.kv_bytes() + self.q_out_bytes()


def gemma3_1b():
    layers = [Layer(4, 1, 256, 0 if (li + 1) % 6 == 0 else 512, 1e6 if (li + 1) % 6 == 0 else 1e4, True)
              for li in range(26)]
    return Workload("cfg2", "Gemma-3-1B-shaped 26-layer decode, context 4096, fp32 K/V", layers, n_seqs=1,
                    pos=4096, n_tok=1, kv_type=1, dtype="f32", replicas=8)


WORKLOADS = {"cfg2": gemma3_1b}


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
                util = nv.nvmlDeviceGetUtilizationRates(self.h).gpu
                self.samples.append((time.perf_counter(), mhz, reasons, util))
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


# ---- the product arm ---------------------------------------------------------------------------

def make_inputs(w: Workload, seed: int):
    """Seeded host data: per layer q, k, v of the new token, the norm gains,
    and the past K/V rows each buffer holds (positions kept by its ring)."""
    rng = np.random.default_rng(seed)
    layers = []
    for L in w.layers:
        d = {}
        d["q"] = rng.standard_normal((w.n_tok, L.n_head * L.D), np.float32)
        d["k"] = rng.standard_normal((w.n_tok, L.n_kv * L.D), np.float32)
        d["v"] = rng.standard_normal((w.n_tok, L.n_kv * L.D), np.float32)
        d["qg"] = (1.0 + 0.1 * rng.standard_normal(L.D, np.float32)).astype(np.float32)
        d["kg"] = (1.0 + 0.1 * rng.standard_normal(L.D, np.float32)).astype(np.float32)
        rows = ring_rows(L.window, w.n_tok) if L.window and ring_rows(L.window, w.n_tok) < w.n_ctx else w.n_ctx
        keep0 = max(0, w.pos - rows)
        n = w.pos - keep0
        d["keep0"], d["rows"] = keep0, rows
        d["pk"] = rng.standard_normal((n, L.n_kv * L.D), np.float32)
        d["pv"] = rng.standard_normal((n, L.n_kv * L.D), np.float32)
        layers.append(d)
    return layers


def ring_rows(window: int, n_batch: int) -> int:
    return (window + max(n_batch, 1) + 255) // 256 * 256


def to_cache_bits(x: np.ndarray, kv_type: int) -> np.ndarray:
    if kv_type == 1:
        return x
    if kv_type == 2:
        return x.astype(np.float16).view(np.uint16)
    u = x.view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def params_for(N, w: Workload, L: Layer, qg, kg):
    return N.params(n_tok=w.n_tok, pos0=w.pos, n_seq=w.pos + w.n_tok, n_head=L.n_head, n_kv=L.n_kv, head_dim=L.D,
                    rope_mode=L.rope_mode, freq_base=L.base, q_gamma=qg if L.qk_norm else None,
                    k_gamma=kg if L.qk_norm else None, window=L.window, eps=1e-6, scale=1.0 / np.sqrt(L.D))


def run_product(args, w: Workload, rank: int, world: int, local_rank: int):
    import torch

    import libllmcpu_b200 as N

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    R = w.replicas
    descs = [(L.n_kv, L.D, L.window, li) for li, L in enumerate(w.layers)]
    kv = N.KVCache(descs, n_ctx=w.n_ctx, n_batch=w.n_tok, n_seq=R * w.n_seqs, kv_type=w.kv_type,
                   device=local_rank)
    data = make_inputs(w, seed=1 + rank)
    for li, d in enumerate(data):
        if d["pk"].shape[0]:
            kb, vb = to_cache_bits(d["pk"], w.kv_type), to_cache_bits(d["pv"], w.kv_type)
            for s in range(R * w.n_seqs):
                kv.write_rows(li, d["keep0"], kb, vb, seq=s)

    # device-resident inputs, one set per replica (distinct memory, same values)
    dev_jobs, keep = [], []
    for r in range(R):
        jobs = []
        for s in range(w.n_seqs):
            seq = r * w.n_seqs + s
            for li, (L, d) in enumerate(zip(w.layers, data)):
                t = {k: torch.from_numpy(d[k]).to(dev) for k in ("q", "k", "v", "qg", "kg")}
                out = torch.empty(w.n_tok, L.n_head * L.D, device=dev)
                p = params_for(N, w, L, t["qg"].data_ptr(), t["kg"].data_ptr())
                jobs.append(N.job(li, p, t["q"], t["k"], t["v"], out, seq=seq))
                keep.append((t, out))
        dev_jobs.append((N.AttnJob * len(jobs))(*jobs))
    stream = torch.cuda.Stream(device=dev)
    dist = torch.distributed if world > 1 else None

    def step(i):
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
    value = world * w.step_bytes() / (ms_per_step * 1e-3) / GB

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
    core_bytes = core["bytes"] / max(core["calls"], 1)
    peaks = measured_peaks()
    achieved = core_bytes / (core_us * 1e-6) / GB
    roofline = {"bound": "hbm", "kernel": "attn_core (decode_kernel: K2+K3)", "achieved": round(achieved, 1),
                "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                "peak_source": peaks["source"], "traffic": profiled_traffic(w.name),
                "bytes_per_launch": int(core_bytes), "us_per_launch": round(core_us, 3),
                "attn_rope_us_per_launch": round(1e3 * rope["ms"] / max(rope["calls"], 1), 3)}

    # ---- e2e: the host-pointer C-ABI call, copies inside every step ----
    host_jobs, host_keep = [], []
    for r in range(R):
        jobs = []
        for s in range(w.n_seqs):
            seq = r * w.n_seqs + s
            for li, (L, d) in enumerate(zip(w.layers, data)):
                out = np.empty((w.n_tok, L.n_head * L.D), np.float32)
                p = params_for(N, w, L, d["qg"], d["kg"])
                jobs.append(N.job(li, p, d["q"], d["k"], d["v"], out, seq=seq))
                host_keep.append(out)
        host_jobs.append(jobs)
    for i in range(args.warmup):
        kv.attention_batch(host_jobs[i % R])
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for i in range(args.steps):
        kv.attention_batch(host_jobs[i % R])
    t_e2e = time.perf_counter() - t0
    if dist:
        te = torch.tensor([t_e2e], device=dev)
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
        t_e2e = float(te.item())
    h2d = sum((d["q"].size + d["k"].size + d["v"].size + (2 * L.D if L.qk_norm else 0)) * 4
              for L, d in zip(w.layers, data)) * w.n_seqs
    d2h = sum(w.n_tok * L.n_head * L.D * 4 for L in w.layers) * w.n_seqs
    e2e = {"value": round(world * w.step_bytes() / (t_e2e / args.steps) / GB, 2), "unit": "GB/s",
           "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
           "ms_per_step": round(1e3 * t_e2e / args.steps, 4), "api": "nncu_attention_batch (host pointers)"}

    line = {
        "metric": "decode attn KV GB/s", "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": w.dtype,
        "data": "synthetic (seeded N(0,1) q/k/v and K/V cache; gains 1+N(0,0.1))",
        "config": {"workload": f"{w.name}: {w.title}", "layers": len(w.layers), "n_head": w.layers[0].n_head,
                   "n_kv": w.layers[0].n_kv, "head_dim": w.layers[0].D, "keys_global": w.pos + 1,
                   "window": 512, "new_tokens": w.n_tok, "bytes_per_step": w.step_bytes(),
                   "l2": f"{R} rotating cache replicas ({kv.state().bytes / R / 1e6:.0f} MB each) > L2",
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU"},
        "hbm_frac": round(value / world / peaks["hbm_gbs"], 4),
        "roofline": roofline, "e2e": e2e, "gpu_launches": int(launches), "clocks": clocks,
    }
    kv.close()
    return line


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
    summary (profiles/), scaled to this workload's launch; None if absent."""
    p = os.path.join(ROOT, "profiles", f"decode_{workload}_traffic.json")
    try:
        with open(p) as f:
            return json.load(f)["dram_bytes_per_launch"]
    except Exception:
        return None


# ---- the reference's CPU path ------------------------------------------------------------------

def cpu_reference(w: Workload, budget_s: float, threads: int | None):
    """The reference's own kernels (oracle/_ref), parallel through its pool,
    over the same workload; falls back to the C restatement (single thread)
    where the reference was not built. Returns (GB/s, cores, kind, sample)."""
    import oracle as O

    which, kind = ("ref", "reference") if O.ref() is not None else ("oracle", "port")
    cores = 1
    if which == "ref":
        n = threads or min(64, os.cpu_count() or 1)
        O.ref().ref_set_num_threads(n)
        cores = O.ref().ref_num_threads()
    data = make_inputs(w, seed=1)
    bufs = []
    for L, d in zip(w.layers, data):
        rows = d["rows"]
        kt = w.kv_type if w.kv_type != 2 else 1  # no F16 cache in the reference: widened F32 rows
        dt = np.float32 if kt == 1 else np.uint16
        Kc = np.zeros((rows, L.n_kv * L.D), dt)
        Vc = np.zeros_like(Kc)
        n = d["pk"].shape[0]
        r = (d["keep0"] + np.arange(n)) % rows
        src_k, src_v = d["pk"], d["pv"]
        if w.kv_type == 2:  # the F16 values, widened
            src_k = src_k.astype(np.float16).astype(np.float32)
            src_v = src_v.astype(np.float16).astype(np.float32)
        Kc[r] = to_cache_bits(src_k, kt)
        Vc[r] = to_cache_bits(src_v, kt)
        bufs.append((Kc, Vc, kt))
    prm = [O.params(n_tok=w.n_tok, pos0=w.pos, n_seq=w.pos + w.n_tok, n_head=L.n_head, n_kv=L.n_kv, head_dim=L.D,
                    rope_mode=L.rope_mode, freq_base=L.base, q_gamma=d["qg"] if L.qk_norm else None,
                    k_gamma=d["kg"] if L.qk_norm else None, window=L.window, scale=1.0 / np.sqrt(L.D))
           for L, d in zip(w.layers, data)]

    def one_step():
        for li, (L, d) in enumerate(zip(w.layers, data)):
            Kc, Vc, kt = bufs[li]
            O.attention_forward(prm[li], d["q"], d["k"], d["v"], Kc, Vc, kt, d["rows"], which=which)

    one_step()  # warm
    n_steps, t0 = 0, time.perf_counter()
    while True:
        one_step()
        n_steps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or n_steps >= 100000:
            break
    gbs = w.step_bytes() * n_steps / el / GB
    sample = f"{n_steps} full {len(w.layers)}-layer steps ({el:.1f} s) of {w.name}"
    if w.kv_type == 2:
        sample += ", F16 cache widened to F32 (the reference has no F16 cache)"
    return gbs, cores, kind, sample, el / n_steps


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["nncu", "reference"], default="nncu")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="cfg2")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline sample length")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args(argv)
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    w = WORKLOADS[args.workload]()

    if args.impl == "reference":
        if rank != 0:
            return 0
        budget = max(5.0, min(60.0, args.cpu_seconds))
        gbs, cores, kind, sample, s_per_step = cpu_reference(w, budget, None)
        line = {"impl": "reference", "metric": "decode attn KV GB/s", "value": round(gbs, 3), "unit": "GB/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * s_per_step, 4),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": w.dtype,
                "data": "synthetic", "config": {"workload": f"{w.name}: {w.title}", "bytes_per_step": w.step_bytes()},
                "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": kind,
                                 "sample": sample},
                "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
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
        gbs, cores, kind, sample, _ = cpu_reference(w, args.cpu_seconds, None)
        line["cpu_baseline"] = {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": kind,
                                "sample": sample}
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
