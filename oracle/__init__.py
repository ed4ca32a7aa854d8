"""TEST INFRASTRUCTURE ONLY: ctypes bindings to the attention checker.

Two libraries, both CPU-only:

* ``liboracle.so`` -- the C restatement of libnnc's attention path
  (``oracle.c``; each function cites the reference file:line it restates).
  Built from this directory with ``make`` wherever gcc exists.
* ``_ref/libnnc_ref.so`` -- the reference's own kernels compiled from the
  reference's sources (``make ref``), wrapped by ``ref_shim.cpp``. Present
  only where it was built; it travels with the repository snapshot.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this package. The product (``libllmcpu_b200``) never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libnnc_ref.so")

KV_BF16, KV_F32, KV_F16 = 0, 1, 2
ROPE_NEOX, ROPE_NORM = 0, 1
ATTN_BLOCK = 256

_lock = threading.Lock()
_lib = None
_ref = None
_ref_tried = False

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")


class AttnParams(C.Structure):
    """orc_attn_params (oracle.h); same fields as nncu_attn_params."""

    _fields_ = [
        ("n_tok", C.c_int32), ("pos0", C.c_int32), ("n_seq", C.c_int32),
        ("n_head", C.c_int32), ("n_kv", C.c_int32), ("head_dim", C.c_int32),
        ("n_rot", C.c_int32), ("rope_mode", C.c_int32),
        ("freq_base", C.c_float), ("rope_scale", C.c_float),
        ("freq_factors", C.c_void_p), ("q_gamma", C.c_void_p), ("k_gamma", C.c_void_p),
        ("v_rmsnorm", C.c_int32),
        ("eps", C.c_float), ("scale", C.c_float), ("softcap", C.c_float),
        ("causal", C.c_int32), ("window", C.c_int32), ("reuse_kv", C.c_int32),
        ("gate", C.c_void_p),
    ]


def _build(target: str = "all") -> None:
    subprocess.run(["make", "-s", "-C", HERE, target], check=True,
                   stdout=subprocess.DEVNULL)


def lib() -> C.CDLL:
    """The restatement, built on first use if missing or stale."""
    global _lib
    with _lock:
        if _lib is None:
            srcs = [os.path.join(HERE, f) for f in ("oracle.c", "oracle.h", "seeded.cpp")]
            if (not os.path.exists(ORACLE_SO)
                    or os.path.getmtime(ORACLE_SO) < max(os.path.getmtime(s) for s in srcs)):
                _build("all")
            L = C.CDLL(ORACLE_SO)
            _declare(L, "orc")
            L.orc_rng_new.restype = C.c_void_p
            L.orc_rng_new.argtypes = [C.c_uint32]
            L.orc_rng_normal.argtypes = [C.c_void_p, _f32p, C.c_size_t, C.c_float, C.c_float]
            L.orc_rng_uniform.argtypes = [C.c_void_p, _f32p, C.c_size_t, C.c_float, C.c_float]
            L.orc_rng_free.argtypes = [C.c_void_p]
            L.orc_argmax_rows.argtypes = [C.c_void_p, C.c_size_t, C.c_int, C.c_uint32, C.c_void_p]
            L.orc_argmax_rows.restype = None
            L.orc_ring_rows.restype = C.c_int
            L.orc_ring_rows.argtypes = [C.c_int, C.c_int]
            L.orc_f32_to_bf16.restype = C.c_uint16
            L.orc_f32_to_bf16.argtypes = [C.c_float]
            L.orc_f32_to_f16.restype = C.c_uint16
            L.orc_f32_to_f16.argtypes = [C.c_float]
            L.orc_attn_block.argtypes = [
                C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p, C.c_int, C.c_size_t, C.c_size_t,
                C.c_size_t, C.c_size_t, C.c_float, C.c_float, C.c_void_p, C.c_void_p]
            _lib = L
        return _lib


def ref():
    """The reference's compiled kernels, or None where they were not built."""
    global _ref, _ref_tried
    with _lock:
        if not _ref_tried:
            _ref_tried = True
            if os.path.exists(REF_SO):
                L = C.CDLL(REF_SO)
                _declare(L, "ref")
                L.ref_set_num_threads.argtypes = [C.c_int]
                L.ref_num_threads.restype = C.c_int
                L.ref_f32_to_bf16.restype = C.c_uint16
                L.ref_f32_to_bf16.argtypes = [C.c_float]
                L.ref_attn_block.argtypes = [
                    C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p, C.c_int, C.c_size_t, C.c_size_t,
                    C.c_size_t, C.c_size_t, C.c_float, C.c_void_p, C.c_void_p]
                _ref = L
        return _ref


def _declare(L, pfx: str) -> None:
    vp, sz, f, i = C.c_void_p, C.c_size_t, C.c_float, C.c_int
    u32 = C.c_uint32
    getattr(L, f"{pfx}_gemv_bf16w").argtypes = [vp, vp, sz, vp, sz, u32, u32, u32]
    getattr(L, f"{pfx}_gemv_q8_0").argtypes = [vp, vp, vp, sz, vp, sz, u32, u32, u32]
    getattr(L, f"{pfx}_gemv_q4_s").argtypes = [vp, vp, vp, vp, sz, vp, sz, vp, sz, u32, u32, u32]
    getattr(L, f"{pfx}_block_sums").argtypes = [vp, vp, sz]
    getattr(L, f"{pfx}_gemv_bf16w_argmax").argtypes = [vp, vp, u32, u32]
    getattr(L, f"{pfx}_gemv_bf16w_argmax").restype = C.c_int
    getattr(L, f"{pfx}_attn_span").argtypes = [i, i, i, i, C.POINTER(C.c_int), C.POINTER(C.c_int)]
    getattr(L, f"{pfx}_rmsnorm_f32").argtypes = [vp, vp, sz, f]
    getattr(L, f"{pfx}_rmsnorm_gamma_multi_f32").argtypes = [vp, vp, sz, sz, vp, f]
    getattr(L, f"{pfx}_rope_f32").argtypes = [vp, C.c_uint32, C.c_uint32, C.c_uint32, f, f, i, vp]
    getattr(L, f"{pfx}_softcap_f32").argtypes = [vp, vp, sz, f]
    getattr(L, f"{pfx}_attn_merge").argtypes = [vp, vp, sz, sz]
    getattr(L, f"{pfx}_attn_finish").argtypes = [vp, sz, vp, sz, sz]
    for fn in ("attend", "attention_forward"):
        g = getattr(L, f"{pfx}_{fn}")
        g.restype = C.c_int
    getattr(L, f"{pfx}_attend").argtypes = [C.POINTER(AttnParams), vp, vp, vp, i, i, vp]
    getattr(L, f"{pfx}_attention_forward").argtypes = [
        C.POINTER(AttnParams), vp, vp, vp, vp, vp, i, i, vp]


def ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


# ---- seeded inputs ----------------------------------------------------------

class Rng:
    """std::mt19937(seed) + std::normal_distribution<float>: the reference tests' stream."""

    def __init__(self, seed: int):
        self._L = lib()
        self._h = self._L.orc_rng_new(seed)

    def normal(self, n: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
        out = np.empty(int(n), np.float32)
        self._L.orc_rng_normal(self._h, out, out.size, mean, std)
        return out

    def uniform(self, n: int, lo: float, hi: float) -> np.ndarray:
        out = np.empty(int(n), np.float32)
        self._L.orc_rng_uniform(self._h, out, out.size, lo, hi)
        return out

    def __del__(self):
        try:
            self._L.orc_rng_free(self._h)
        except Exception:
            pass


# ---- element types ----------------------------------------------------------

def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round to nearest even on the upper 16 bits (runtime.h:106-113)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def narrow(x: np.ndarray, kv_type: int) -> np.ndarray:
    """The cache's stored bits for fp32 values x."""
    if kv_type == KV_F32:
        return np.ascontiguousarray(x, np.float32)
    if kv_type == KV_BF16:
        return f32_to_bf16_bits(x)
    return np.ascontiguousarray(x, np.float32).astype(np.float16).view(np.uint16)


def widen(b: np.ndarray, kv_type: int) -> np.ndarray:
    if kv_type == KV_F32:
        return np.ascontiguousarray(b, np.float32)
    if kv_type == KV_BF16:
        return bf16_bits_to_f32(b)
    return b.view(np.float16).astype(np.float32)


# ---- the attention op ---------------------------------------------------------

def params(**kw) -> AttnParams:
    d = dict(n_tok=1, pos0=0, n_seq=None, n_head=1, n_kv=1, head_dim=64, n_rot=None,
             rope_mode=ROPE_NEOX, freq_base=10000.0, rope_scale=1.0, freq_factors=None,
             q_gamma=None, k_gamma=None, v_rmsnorm=0, eps=1e-6, scale=None, softcap=0.0,
             causal=1, window=0, reuse_kv=0, gate=None)
    d.update(kw)
    if d["n_seq"] is None:
        d["n_seq"] = d["pos0"] + d["n_tok"]
    if d["n_rot"] is None:
        d["n_rot"] = d["head_dim"]
    if d["scale"] is None:
        d["scale"] = 1.0 / float(np.sqrt(d["head_dim"]))
    keep = {}
    p = AttnParams()
    for k, v in d.items():
        if k in ("freq_factors", "q_gamma", "k_gamma", "gate"):
            if v is not None:
                v = np.ascontiguousarray(v, np.float32)
                keep[k] = v
                setattr(p, k, v.ctypes.data)
            else:
                setattr(p, k, None)
        else:
            setattr(p, k, v)
    p._keep = keep  # keep the arrays alive with the struct
    return p


def attention_forward(p: AttnParams, q, k, v, Kc, Vc, kv_type: int, rows: int, which: str = "oracle"):
    """Run norms, RoPE, append and attend. q/k/v are copied (the call modifies
    them); Kc/Vc (the cache's stored bits, reference layout [rows][n_kv*hd])
    are updated in place. Returns (out, q_rotated, k_rotated)."""
    L = lib() if which == "oracle" else ref()
    fn = L.orc_attention_forward if which == "oracle" else L.ref_attention_forward
    q = np.array(q, np.float32, copy=True)
    k = np.array(k, np.float32, copy=True)
    v = np.array(v, np.float32, copy=True)
    out = np.zeros((p.n_tok, p.n_head * p.head_dim), np.float32)
    rc = fn(C.byref(p), ptr(q), ptr(k), ptr(v), ptr(Kc), ptr(Vc), kv_type, rows, ptr(out))
    if rc != 0:
        raise ValueError(f"{which}: attention_forward refused these arguments")
    return out, q, k


def attend(p: AttnParams, q, Kc, Vc, kv_type: int, rows: int, which: str = "oracle"):
    L = lib() if which == "oracle" else ref()
    fn = L.orc_attend if which == "oracle" else L.ref_attend
    q = np.ascontiguousarray(q, np.float32)
    out = np.zeros((p.n_tok, p.n_head * p.head_dim), np.float32)
    rc = fn(C.byref(p), ptr(q), ptr(Kc), ptr(Vc), kv_type, rows, ptr(out))
    if rc != 0:
        raise ValueError(f"{which}: attend refused these arguments")
    return out


def attn_span(causal: bool, window: int, pos: int, n_seq: int, which: str = "oracle"):
    L = lib() if which == "oracle" else ref()
    f, l = C.c_int(), C.c_int()
    getattr(L, "orc_attn_span" if which == "oracle" else "ref_attn_span")(
        int(causal), window, pos, n_seq, C.byref(f), C.byref(l))
    return f.value, l.value


def rope(x, n_heads, head_dim, n_rot, pos, base, mode=ROPE_NEOX, freq_factors=None, which="oracle"):
    L = lib() if which == "oracle" else ref()
    x = np.array(x, np.float32, copy=True)
    ff = None if freq_factors is None else np.ascontiguousarray(freq_factors, np.float32)
    getattr(L, "orc_rope_f32" if which == "oracle" else "ref_rope_f32")(
        ptr(x), n_heads, head_dim, n_rot, pos, base, mode, ptr(ff))
    return x


def rmsnorm_gamma_multi(x, n_groups, dim, gamma, eps, which="oracle"):
    L = lib() if which == "oracle" else ref()
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    g = np.ascontiguousarray(gamma, np.float32)
    getattr(L, "orc_rmsnorm_gamma_multi_f32" if which == "oracle" else "ref_rmsnorm_gamma_multi_f32")(
        ptr(y), ptr(x), n_groups, dim, ptr(g), eps)
    return y


def rmsnorm(x, eps, which="oracle"):
    L = lib() if which == "oracle" else ref()
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    getattr(L, "orc_rmsnorm_f32" if which == "oracle" else "ref_rmsnorm_f32")(ptr(y), ptr(x), x.size, eps)
    return y


def softcap(x, cap, which="oracle"):
    L = lib() if which == "oracle" else ref()
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    getattr(L, "orc_softcap_f32" if which == "oracle" else "ref_softcap_f32")(ptr(y), ptr(x), x.size, cap)
    return y


def attn_block(q, q_stride, K, V, kv_type, kv_stride, n_keys, head_dim, n_heads, scale, softcap_=0.0,
               which="oracle", k_offset_elems=0):
    """One block into a fresh partial [n_heads][head_dim + 2]."""
    L = lib() if which == "oracle" else ref()
    es = 4 if kv_type == KV_F32 else 2
    part = np.zeros(n_heads * (head_dim + 2), np.float32)
    scores = np.zeros(n_heads * max(n_keys, 1), np.float32)
    kp = K.ctypes.data + k_offset_elems * es
    vp = V.ctypes.data + k_offset_elems * es
    if which == "oracle":
        L.orc_attn_block(ptr(q), q_stride, kp, vp, kv_type, kv_stride, n_keys, head_dim, n_heads, scale,
                         softcap_, ptr(scores), ptr(part))
    else:
        if kv_type == KV_F16:
            raise ValueError("the reference has no F16 cache")
        L.ref_attn_block(ptr(q), q_stride, kp, vp, int(kv_type == KV_BF16), kv_stride, n_keys, head_dim,
                         n_heads, scale, ptr(scores), ptr(part))
    return part


def attn_merge(acc, part, head_dim, n_heads, which="oracle"):
    L = lib() if which == "oracle" else ref()
    acc = np.array(acc, np.float32, copy=True)
    getattr(L, "orc_attn_merge" if which == "oracle" else "ref_attn_merge")(
        ptr(acc), ptr(np.ascontiguousarray(part, np.float32)), head_dim, n_heads)
    return acc


def attn_finish(acc, head_dim, n_heads, which="oracle"):
    L = lib() if which == "oracle" else ref()
    out = np.zeros(n_heads * head_dim, np.float32)
    getattr(L, "orc_attn_finish" if which == "oracle" else "ref_attn_finish")(
        ptr(out), head_dim, ptr(np.ascontiguousarray(acc, np.float32)), head_dim, n_heads)
    return out


orc_params = params


def ring_rows(window: int, n_batch: int) -> int:
    """round_up(window + n_batch, 256) (model.cpp:1934)."""
    return int(lib().orc_ring_rows(int(window), int(n_batch)))


# ---- the projections' gemvs (src/libnnc/nn_ops.h:89-170) ----------------------------------------

def _gemv_lib(which: str):
    L = lib() if which == "oracle" else ref()
    return L, ("orc" if which == "oracle" else "ref")


def gemv_bf16w(W_bits: np.ndarray, X: np.ndarray, which: str = "oracle") -> np.ndarray:
    """Y[v] = W X[v] for BF16 weights W_bits [rows][cols] (uint16) and fp32 X [n_batch][cols]."""
    L, p = _gemv_lib(which)
    rows, cols = W_bits.shape
    X = np.ascontiguousarray(X, np.float32).reshape(-1, cols)
    Y = np.empty((X.shape[0], rows), np.float32)
    getattr(L, f"{p}_gemv_bf16w")(ptr(np.ascontiguousarray(W_bits)), ptr(X), cols, ptr(Y), rows, rows, cols, X.shape[0])
    return Y


def gemv_q8_0(qs: np.ndarray, scales: np.ndarray, X: np.ndarray, which: str = "oracle") -> np.ndarray:
    """Q8_0 split layout: qs int8 [rows][cols], scales BF16 [rows][cols / 32]."""
    L, p = _gemv_lib(which)
    rows, cols = qs.shape
    X = np.ascontiguousarray(X, np.float32).reshape(-1, cols)
    Y = np.empty((X.shape[0], rows), np.float32)
    getattr(L, f"{p}_gemv_q8_0")(ptr(np.ascontiguousarray(qs)), ptr(np.ascontiguousarray(scales)), ptr(X), cols,
                                 ptr(Y), rows, rows, cols, X.shape[0])
    return Y


def gemv_q4_s(qs: np.ndarray, scales: np.ndarray, biases: np.ndarray, X: np.ndarray, XSUM: np.ndarray,
              which: str = "oracle") -> np.ndarray:
    """Q4_S split layout: qs uint8 [rows][cols / 2] (byte k of a block: element k low, k + 16 high),
    scales and biases BF16 [rows][cols / 32], XSUM the vectors' block sums [n_batch][cols / 32]."""
    L, p = _gemv_lib(which)
    rows, half = qs.shape
    cols = 2 * half
    X = np.ascontiguousarray(X, np.float32).reshape(-1, cols)
    XSUM = np.ascontiguousarray(XSUM, np.float32).reshape(-1, cols // 32)
    Y = np.empty((X.shape[0], rows), np.float32)
    getattr(L, f"{p}_gemv_q4_s")(ptr(np.ascontiguousarray(qs)), ptr(np.ascontiguousarray(scales)),
                                 ptr(np.ascontiguousarray(biases)), ptr(X), cols, ptr(XSUM), cols // 32, ptr(Y), rows,
                                 rows, cols, X.shape[0])
    return Y


def block_sums(x: np.ndarray, which: str = "oracle") -> np.ndarray:
    L, p = _gemv_lib(which)
    x = np.ascontiguousarray(x, np.float32).ravel()
    out = np.empty(x.size // 32, np.float32)
    getattr(L, f"{p}_block_sums")(ptr(x), ptr(out), x.size)
    return out


def argmax_rows(X: np.ndarray) -> np.ndarray:
    """session.cpp:128-134's argmax of each row of X (the checker's)."""
    X = np.ascontiguousarray(X, np.float32)
    if X.ndim == 1:
        X = X[None, :]
    out = np.zeros(X.shape[0], np.int32)
    lib().orc_argmax_rows(ptr(X), X.shape[1], X.shape[0], X.shape[1], ptr(out))
    return out


def gemv_bf16w_argmax(W_bits: np.ndarray, x: np.ndarray, which: str = "oracle") -> int:
    L, p = _gemv_lib(which)
    rows, cols = W_bits.shape
    x = np.ascontiguousarray(x, np.float32).ravel()
    return int(getattr(L, f"{p}_gemv_bf16w_argmax")(ptr(np.ascontiguousarray(W_bits)), ptr(x), rows, cols))
