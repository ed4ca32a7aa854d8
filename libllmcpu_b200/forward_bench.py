"""Time attention_forward on the device (nncu_attention_forward_dev) for one
layer of a named model shape, with seeded random weights in libnnc's formats
and a filled K/V cache:

    python -m libllmcpu_b200.forward_bench --model qwen3-8b --weights q4_s --context 4096 --calls 200

Each call is one decode token (``--tokens`` for a verify block; ``--seqs``
sequences of the layer in one call): the q/k/v gemvs, the attention over
``--context`` keys, the o gemv. L2 is flushed
before every timed call (a 256 MB write) and each call is timed alone with
CUDA events on the launching stream; one JSON line with the median. The
weights are random bytes of the right layout (quants, BF16 scales and
biases), not a checkpoint: the work and the memory traffic are the layer's.
Also ``--gemv ROWSxCOLS`` times one single-vector gemv of that shape instead.
"""
from __future__ import annotations

import argparse
import json

import numpy as np

from . import KV_BF16, KV_F16, KV_F32, W_BF16, W_Q4_S, W_Q8_0, AttnWeights, KVCache, params, weight

# (n_embd, n_head, n_kv, head_dim, gated)
MODELS = {
    "gemma3-4b": (2560, 8, 4, 256, False),
    "qwen3-8b": (4096, 32, 8, 128, False),
    "qwen3.5-4b": (2560, 16, 4, 256, True),
    "llama3.2-1b": (2048, 32, 8, 64, False),
}
WTYPES = {"bf16": W_BF16, "q8_0": W_Q8_0, "q4_s": W_Q4_S}
KVTYPES = {"bf16": KV_BF16, "f16": KV_F16, "f32": KV_F32}


def random_weight(torch, kind: int, rows: int, cols: int, gen):
    """Device tensors of one weight in libnnc's layout, and its descriptor."""
    dev = "cuda"
    if kind == W_BF16:
        data = (torch.rand((rows, cols), generator=gen, device=dev) * 2 - 1).div_(cols ** 0.5).to(torch.bfloat16)
        return weight(kind, rows, cols, data)
    scales = (torch.rand((rows, cols // 32), generator=gen, device=dev) * 0.01).to(torch.bfloat16)
    if kind == W_Q8_0:
        data = torch.randint(-128, 128, (rows, cols), generator=gen, dtype=torch.int8, device=dev)
        return weight(kind, rows, cols, data, scales)
    data = torch.randint(0, 256, (rows, cols // 2), generator=gen, dtype=torch.uint8, device=dev)
    biases = (torch.rand((rows, cols // 32), generator=gen, device=dev) * 0.01 - 0.005).to(torch.bfloat16)
    return weight(kind, rows, cols, data, scales, biases)


def _time(torch, fn, calls: int, flush) -> list[float]:
    st = torch.cuda.current_stream()
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    out = []
    for _ in range(calls):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        fn()
        b.record(st)
        b.synchronize()
        out.append(a.elapsed_time(b) * 1e3)
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--model", choices=sorted(MODELS), default="qwen3-8b")
    ap.add_argument("--weights", choices=sorted(WTYPES), default="q4_s")
    ap.add_argument("--kv", choices=sorted(KVTYPES), default="bf16")
    ap.add_argument("--context", type=int, default=4096)
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--seqs", type=int, default=1, help="sequences of the layer in one call (a serving batch)")
    ap.add_argument("--calls", type=int, default=100)
    ap.add_argument("--gemv", default=None, help="ROWSxCOLS: time one single-vector gemv of this shape instead")
    a = ap.parse_args(argv)

    import torch

    gen = torch.Generator(device="cuda")
    gen.manual_seed(0)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    kind = WTYPES[a.weights]
    if a.gemv:
        rows, cols = (int(v) for v in a.gemv.lower().split("x"))
        w = random_weight(torch, kind, rows, cols, gen)
        x = torch.randn(1, cols, device="cuda")
        y = torch.empty(1, rows, device="cuda")
        # one vector through the logits entry point: the same gemv launch (plus
        # the Q4_S block sums), no soft-cap
        from . import logits_batch_dev

        xs = torch.empty(1, max(cols // 32, 1), device="cuda")
        ts = _time(torch, lambda: logits_batch_dev(w, x, 1, y, 0.0, xs), a.calls, flush)
        med = float(np.median(ts))
        wbytes = sum(int(t.numel() * t.element_size()) for t in w._keep if t is not None)
        print(json.dumps(dict(what="gemv", weights=a.weights, rows=rows, cols=cols, us=round(med, 2),
                              GBs=round(wbytes / med / 1e3, 1))))
        return 0

    n_embd, n_head, n_kv, hd, gated = MODELS[a.model]
    q_dim, kv_dim = n_head * hd, n_kv * hd
    ws = {"q": random_weight(torch, kind, (2 if gated else 1) * q_dim, n_embd, gen),
          "k": random_weight(torch, kind, kv_dim, n_embd, gen),
          "v": random_weight(torch, kind, kv_dim, n_embd, gen),
          "o": random_weight(torch, kind, n_embd, q_dim, gen)}
    kv_type = KVTYPES[a.kv]
    kv = KVCache([(n_kv, hd, 0, 0)], n_ctx=a.context + a.tokens + 256, n_batch=max(16, a.tokens), n_seq=a.seqs,
                 kv_type=kv_type)
    el = {KV_F32: torch.float32, KV_BF16: torch.bfloat16, KV_F16: torch.float16}[kv_type]
    for s in range(a.seqs):
        for p0 in range(0, a.context, 4096):
            n = min(4096, a.context - p0)
            rows_k = torch.randn(n, kv_dim, generator=gen, device="cuda").to(el)
            kv.write_rows(0, p0, rows_k, rows_k, seq=s)
    w = AttnWeights(ws["q"], ws["k"], ws["v"], ws["o"], None, None, None, int(gated))
    p = params(n_tok=a.tokens, pos0=a.context, n_head=n_head, n_kv=n_kv, head_dim=hd, freq_base=1e6)
    x = torch.randn(a.seqs * a.tokens, n_embd, device="cuda")
    y = torch.empty_like(x)
    if a.seqs == 1:
        ts = _time(torch, lambda: kv.attention_forward_dev(0, p, w, x, y), a.calls, flush)
    else:
        seqs, ps = list(range(a.seqs)), [p] * a.seqs
        ts = _time(torch, lambda: kv.attention_forward_batch_dev(0, seqs, ps, w, x, y), a.calls, flush)
    kv.sync()
    kv.close()
    med = float(np.median(ts))
    wbytes = sum(int(t.numel() * t.element_size()) for wt in ws.values() for t in wt._keep if t is not None)
    kvbytes = 2 * a.context * kv_dim * (4 if kv_type == KV_F32 else 2) * a.seqs
    print(json.dumps(dict(what="attention_forward", model=a.model, weights=a.weights, kv=a.kv, context=a.context,
                          tokens=a.tokens, seqs=a.seqs, us=round(med, 2), weight_MB=round(wbytes / 1e6, 2),
                          kv_MB=round(kvbytes / 1e6, 2), GBs=round((wbytes + kvbytes) / med / 1e3, 1))))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
