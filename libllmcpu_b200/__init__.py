"""libllmcpu_b200 -- libnnc's attention hot path on NVIDIA B200 (sm_100a).

The product is the C-ABI library ``libnncu.so`` built from ``csrc/`` (see
``include/nncu.h``). This module is a thin ctypes binding to it, with the
reference's names, so a Python caller (tests, the benchmark) reads like
libnnc's own code:

==============================  ==========================================
here                            libnnc (ZacWalk/libllmcpu)
==============================  ==========================================
``attn_span``                   ``model_attn_span`` (model.cpp:2300-2316)
``KVCache``                     ``model_kv_cache`` / ``model_kv_init`` /
                                ``model_kv_rewind`` (model.h:231-364)
``KVCache.attention``           ``attention_forward`` after the projections
                                (model.cpp:1616-1757)
``attn_block_dev`` etc.         ``nnc_attn_block`` / ``merge`` / ``finish``
                                (nn_ops.h:31-61) on device pointers
==============================  ==========================================

There is no CPU fallback: importing works without a GPU (so the ABI can be
inspected), but every compute call needs the CUDA library and an sm_100
device and raises ``NnncError`` otherwise.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

__all__ = [
    "NnncError", "lib", "LIB_PATH", "host_register", "host_unregister", "KV_BF16", "KV_F32", "KV_F16", "ROPE_NEOX", "ROPE_NORM",
    "ATTN_BLOCK", "AttnParams", "AttnJob", "LayerDesc", "KVCache", "kv_plan", "job", "attn_span", "params",
    "attn_block_dev", "attn_merge_dev", "attn_finish_dev", "rmsnorm_gamma_multi_dev", "rmsnorm_dev",
    "rope_dev", "softcap_dev", "gemv_bf16w_dev", "gemv_q8_0_dev", "gemv_q4_s_dev", "block_sums_dev",
    "gemv_bf16w_argmax_dev", "Weight", "AttnWeights", "weight", "W_BF16", "W_Q8_0", "W_Q4_S", "logits_batch_dev",
    "argmax_rows_dev", "EXPORTS",
]

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libnncu.so")

KV_BF16, KV_F32, KV_F16 = 0, 1, 2
ROPE_NEOX, ROPE_NORM = 0, 1
ATTN_BLOCK = 256
OK, ERR_INVALID_ARGUMENT, ERR_UNSUPPORTED, ERR_OUT_OF_MEMORY, ERR_CONTEXT_FULL = 0, 1, 2, 6, 7
ERR_DEVICE, ERR_TIMEOUT = 20, 21
W_BF16, W_Q8_0, W_Q4_S = 0, 1, 2

# Every symbol include/nncu.h declares.
EXPORTS = [
    "nncu_status_string", "nncu_last_error", "nncu_last_status", "nncu_clear_error", "nncu_version",
    "nncu_device_check", "nncu_attn_span", "nncu_attn_block_dev", "nncu_attn_merge_dev",
    "nncu_attn_finish_dev", "nncu_rmsnorm_gamma_multi_dev", "nncu_rmsnorm_dev", "nncu_rope_dev",
    "nncu_softcap_dev", "nncu_kv_plan", "nncu_kv_create", "nncu_kv_free", "nncu_kv_layer", "nncu_kv_get_state",
    "nncu_kv_rewind", "nncu_kv_commit", "nncu_kv_write_rows", "nncu_kv_read_rows", "nncu_attention",
    "nncu_attention_batch", "nncu_attention_batch_dev", "nncu_sync", "nncu_perf_enable", "nncu_perf_reset",
    "nncu_perf_read", "nncu_perf_report", "nncu_launch_count", "nncu_attention_noalloc", "nncu_group_create",
    "nncu_group_handle", "nncu_group_open", "nncu_group_output", "nncu_group_copy_output", "nncu_group_free",
    "nncu_attention_split_dev", "nncu_group_set_timeout", "nncu_group_reset", "nncu_group_inject_drop",
    "nncu_noalloc_check", "nncu_kv_set_tensor_cores", "nncu_host_register", "nncu_host_unregister",
    "nncu_gemv_bf16w_f32x_batch_dev", "nncu_gemv_q8_0_f32x_batch_dev", "nncu_gemv_q4_s_f32x_batch_dev",
    "nncu_block_sums_dev", "nncu_gemv_bf16w_argmax_dev", "nncu_attention_forward_dev", "nncu_logits_batch_dev",
    "nncu_attention_forward_batch_dev",
    "nncu_argmax_rows_dev",
]
GROUP_HANDLE_BYTES = 64


class NnncError(RuntimeError):
    """A failed call: ``status`` is the nnc_status value, the message is nncu_last_error()."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[{status}] {message}")
        self.status = status


class AttnParams(C.Structure):
    """nncu_attn_params (include/nncu.h)."""

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


class AttnJob(C.Structure):
    """nncu_attn_job (include/nncu.h)."""

    _fields_ = [("layer", C.c_int32), ("seq", C.c_int32), ("p", AttnParams),
                ("q", C.c_void_p), ("k", C.c_void_p), ("v", C.c_void_p), ("out", C.c_void_p)]


class Weight(C.Structure):
    """nncu_weight (include/nncu.h): one projection's device weights."""

    _fields_ = [("type", C.c_int32), ("rows", C.c_uint32), ("cols", C.c_uint32),
                ("data", C.c_void_p), ("scales", C.c_void_p), ("biases", C.c_void_p)]


class AttnWeights(C.Structure):
    """nncu_attn_weights (include/nncu.h): one layer's q, k, v, o projections."""

    _fields_ = [("q", Weight), ("k", Weight), ("v", Weight), ("o", Weight),
                ("q_bias", C.c_void_p), ("k_bias", C.c_void_p), ("v_bias", C.c_void_p), ("gated", C.c_int32)]


class LayerDesc(C.Structure):
    _fields_ = [("n_kv", C.c_int32), ("head_dim", C.c_int32), ("window", C.c_int32), ("kv_layer", C.c_int32)]


class KVParams(C.Structure):
    _fields_ = [("n_ctx", C.c_int32), ("n_batch", C.c_int32), ("n_seq", C.c_int32), ("kv_type", C.c_int32),
                ("causal", C.c_int32), ("device", C.c_int32)]


class KVLayerInfo(C.Structure):
    _fields_ = [("buffer", C.c_int32), ("rows", C.c_int32), ("window", C.c_int32), ("n_kv", C.c_int32),
                ("head_dim", C.c_int32), ("kv_type", C.c_int32), ("head_bytes", C.c_size_t),
                ("seq_bytes", C.c_size_t), ("k", C.c_void_p), ("v", C.c_void_p)]


class KVState(C.Structure):
    _fields_ = [("cur_pos", C.c_int32), ("kv_written", C.c_int32), ("max_rewind", C.c_int32),
                ("n_ctx", C.c_int32), ("bytes", C.c_size_t)]


class PerfPhase(C.Structure):
    _fields_ = [("ms", C.c_double), ("calls", C.c_int64), ("bytes", C.c_uint64)]


PERF_ATTN_ROPE, PERF_ATTN_CORE = 0, 1


def perf_enable(on: bool = True) -> None:
    """nnc_perf_enable for this path's two phases (attn_rope: K1, attn_core: K2+K3)."""
    lib().nncu_perf_enable(int(on))


def perf_reset() -> None:
    lib().nncu_perf_reset()


def perf_read() -> dict:
    ph = (PerfPhase * 2)()
    _check(lib().nncu_perf_read(ph))
    return {name: dict(ms=p.ms, calls=p.calls, bytes=p.bytes) for name, p in zip(("attn_rope", "attn_core"), ph)}


def perf_report(title: str = "nncu", n_tokens: int = 0) -> str:
    return lib().nncu_perf_report(title.encode(), n_tokens).decode()


def launch_count() -> int:
    return int(lib().nncu_launch_count())


def host_register(arr) -> None:
    """Pin a host numpy array for the host-pointer calls (nncu_host_register):
    a call whose host buffers are all registered moves them with kernels
    through the GPU's mapping of the memory instead of staging copies. Keep
    the array alive until host_unregister(arr)."""
    _check(lib().nncu_host_register(C.c_void_p(arr.ctypes.data), C.c_size_t(arr.nbytes)))


def host_unregister(arr) -> None:
    _check(lib().nncu_host_unregister(C.c_void_p(arr.ctypes.data)))


_lib = None


def lib() -> C.CDLL:
    """Load libnncu.so (built by ``python -m libllmcpu_b200.build``); raise if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise NnncError(ERR_UNSUPPORTED,
                        f"{LIB_PATH} is not built: run `python -m libllmcpu_b200.build` (no CPU fallback exists)")
    L = C.CDLL(LIB_PATH)
    i32, sz, vp, f = C.c_int32, C.c_size_t, C.c_void_p, C.c_float
    L.nncu_status_string.restype = C.c_char_p
    L.nncu_status_string.argtypes = [C.c_int]
    L.nncu_last_error.restype = C.c_char_p
    L.nncu_last_status.restype = C.c_int
    L.nncu_version.restype = C.c_char_p
    L.nncu_device_check.argtypes = [C.c_int]
    L.nncu_attn_span.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int)]
    L.nncu_attn_span.restype = None
    L.nncu_attn_block_dev.argtypes = [vp, sz, vp, vp, C.c_int, sz, sz, sz, sz, f, f, vp, vp]
    L.nncu_attn_merge_dev.argtypes = [vp, vp, sz, sz, vp]
    L.nncu_attn_finish_dev.argtypes = [vp, sz, vp, sz, sz, vp]
    L.nncu_rmsnorm_gamma_multi_dev.argtypes = [vp, vp, sz, sz, vp, f, vp]
    L.nncu_rmsnorm_dev.argtypes = [vp, vp, sz, sz, f, vp]
    L.nncu_rope_dev.argtypes = [vp, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_int32, f, f, C.c_int, vp,
                                vp]
    L.nncu_softcap_dev.argtypes = [vp, vp, sz, f, vp]
    u32 = C.c_uint32
    L.nncu_gemv_bf16w_f32x_batch_dev.argtypes = [vp, vp, sz, vp, sz, u32, u32, u32, vp]
    L.nncu_gemv_q8_0_f32x_batch_dev.argtypes = [vp, vp, vp, sz, vp, sz, u32, u32, u32, vp]
    L.nncu_gemv_q4_s_f32x_batch_dev.argtypes = [vp, vp, vp, vp, sz, vp, sz, vp, sz, u32, u32, u32, vp]
    L.nncu_block_sums_dev.argtypes = [vp, vp, sz, vp]
    L.nncu_gemv_bf16w_argmax_dev.argtypes = [vp, vp, u32, u32, vp, vp, vp]
    L.nncu_kv_plan.argtypes = [C.POINTER(LayerDesc), i32, C.POINTER(KVParams), C.POINTER(KVLayerInfo),
                               C.POINTER(i32), C.POINTER(sz)]
    L.nncu_kv_create.argtypes = [C.POINTER(LayerDesc), i32, C.POINTER(KVParams), C.POINTER(vp)]
    L.nncu_kv_free.argtypes = [vp]
    L.nncu_kv_free.restype = None
    L.nncu_kv_layer.argtypes = [vp, i32, C.POINTER(KVLayerInfo)]
    L.nncu_kv_get_state.argtypes = [vp, i32, C.POINTER(KVState)]
    L.nncu_kv_rewind.argtypes = [vp, i32, i32]
    L.nncu_kv_commit.argtypes = [vp, i32, i32, i32]
    L.nncu_kv_write_rows.argtypes = [vp, i32, i32, i32, i32, vp, vp]
    L.nncu_kv_read_rows.argtypes = [vp, i32, i32, i32, i32, vp, vp]
    L.nncu_attention.argtypes = [vp, i32, i32, C.POINTER(AttnParams), vp, vp, vp, vp]
    L.nncu_attention_batch.argtypes = [vp, C.POINTER(AttnJob), i32]
    L.nncu_attention_batch_dev.argtypes = [vp, C.POINTER(AttnJob), i32, vp]
    L.nncu_attention_forward_dev.argtypes = [vp, i32, i32, C.POINTER(AttnParams), C.POINTER(AttnWeights), vp, vp,
                                             vp]
    L.nncu_logits_batch_dev.argtypes = [C.POINTER(Weight), vp, i32, vp, f, vp, vp]
    L.nncu_attention_forward_batch_dev.argtypes = [vp, i32, i32, vp, C.POINTER(AttnParams), C.POINTER(AttnWeights),
                                                   vp, vp, vp]
    L.nncu_argmax_rows_dev.argtypes = [vp, sz, i32, C.c_uint32, vp, vp]
    L.nncu_host_register.argtypes = [vp, sz]
    L.nncu_host_unregister.argtypes = [vp]
    L.nncu_sync.argtypes = [vp, vp]
    L.nncu_perf_enable.argtypes = [C.c_int]
    L.nncu_perf_enable.restype = None
    L.nncu_perf_reset.restype = None
    L.nncu_perf_read.argtypes = [C.POINTER(PerfPhase)]
    L.nncu_perf_report.argtypes = [C.c_char_p, i32]
    L.nncu_perf_report.restype = C.c_char_p
    L.nncu_launch_count.restype = C.c_uint64
    L.nncu_attention_noalloc.argtypes = [C.POINTER(AttnParams), vp, vp, vp, vp, vp, vp, i32, i32, vp]
    L.nncu_group_create.argtypes = [i32, i32, i32, i32, i32, C.POINTER(vp)]
    L.nncu_group_handle.argtypes = [vp, vp]
    L.nncu_group_open.argtypes = [vp, i32, vp]
    L.nncu_group_output.argtypes = [vp]
    L.nncu_group_output.restype = vp
    L.nncu_group_copy_output.argtypes = [vp, vp, sz, vp]
    L.nncu_group_free.argtypes = [vp]
    L.nncu_group_free.restype = None
    L.nncu_attention_split_dev.argtypes = [vp, vp, C.POINTER(AttnJob), i32, i32, i32, vp]
    L.nncu_group_set_timeout.argtypes = [vp, C.c_uint32]
    L.nncu_group_reset.argtypes = [vp]
    L.nncu_group_inject_drop.argtypes = [vp, i32]
    L.nncu_noalloc_check.argtypes = [vp]
    L.nncu_kv_set_tensor_cores.argtypes = [vp, C.c_int]
    _lib = L
    return L


def _check(rc: int) -> None:
    if rc != OK:
        raise NnncError(rc, lib().nncu_last_error().decode(errors="replace"))


def _ptr(a):
    if a is None:
        return None
    if isinstance(a, int):
        return a
    if isinstance(a, np.ndarray):
        assert a.flags["C_CONTIGUOUS"], "arrays passed to the library must be C-contiguous"
        return a.ctypes.data
    return a.data_ptr()  # a torch tensor (device memory)


def attn_span(causal: bool, window: int, pos: int, n_seq: int) -> tuple[int, int]:
    """model_attn_span: the keys [first, last] the query at pos attends to."""
    f, l = C.c_int(), C.c_int()
    lib().nncu_attn_span(int(causal), int(window), int(pos), int(n_seq), C.byref(f), C.byref(l))
    return f.value, l.value


def params(**kw) -> AttnParams:
    """An nncu_attn_params with the reference's defaults filled in. Array
    arguments (freq_factors, q_gamma, k_gamma, gate) may be numpy arrays (host
    calls) or device pointers / tensors (device calls)."""
    d = dict(n_tok=1, pos0=0, n_seq=None, n_head=1, n_kv=1, head_dim=64, n_rot=None, rope_mode=ROPE_NEOX,
             freq_base=10000.0, rope_scale=1.0, freq_factors=None, q_gamma=None, k_gamma=None, v_rmsnorm=0,
             eps=1e-6, scale=None, softcap=0.0, causal=1, window=0, reuse_kv=0, gate=None)
    d.update(kw)
    if d["n_seq"] is None:
        d["n_seq"] = d["pos0"] + d["n_tok"]
    if d["n_rot"] is None:
        d["n_rot"] = d["head_dim"]
    if d["scale"] is None:
        d["scale"] = 1.0 / float(np.sqrt(d["head_dim"]))
    p = AttnParams()
    keep = {}
    for k, v in d.items():
        if k in ("freq_factors", "q_gamma", "k_gamma", "gate"):
            if isinstance(v, np.ndarray):
                v = np.ascontiguousarray(v, np.float32)
                keep[k] = v
            setattr(p, k, _ptr(v))
        else:
            setattr(p, k, v)
    p._keep = keep
    return p


def kv_plan(layers, n_ctx: int, n_batch: int = 16, n_seq: int = 1, kv_type: int = KV_BF16, causal: bool = True):
    """model_kv_init's sizing without a device: (per-layer KVLayerInfo list, max_rewind, bytes)."""
    descs = (LayerDesc * len(layers))(*[LayerDesc(*map(int, t)) for t in layers])
    prm = KVParams(int(n_ctx), int(n_batch), int(n_seq), int(kv_type), int(causal), 0)
    info = (KVLayerInfo * len(layers))()
    mr, nbytes = C.c_int32(), C.c_size_t()
    _check(lib().nncu_kv_plan(descs, len(layers), C.byref(prm), info, C.byref(mr), C.byref(nbytes)))
    return list(info), mr.value, nbytes.value


class KVCache:
    """The HBM K/V cache of one model (model_kv_cache), for n_seq sequences."""

    def __init__(self, layers, n_ctx: int, n_batch: int = 16, n_seq: int = 1, kv_type: int = KV_BF16,
                 causal: bool = True, device: int = 0):
        """layers: a list of (n_kv, head_dim, window, kv_layer) tuples."""
        L = lib()
        descs = (LayerDesc * len(layers))(*[LayerDesc(*map(int, t)) for t in layers])
        prm = KVParams(int(n_ctx), int(n_batch), int(n_seq), int(kv_type), int(causal), int(device))
        h = C.c_void_p()
        _check(L.nncu_kv_create(descs, len(layers), C.byref(prm), C.byref(h)))
        self._h = h
        self.n_layer = len(layers)
        self.kv_type = kv_type
        self.layers = [tuple(t) for t in layers]

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().nncu_kv_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    def set_tensor_cores(self, enabled: bool) -> None:
        """Decode / verify of several rows per KV head on a 16-bit cache on the
        tensor cores (the default) or on the CUDA-core kernel."""
        _check(lib().nncu_kv_set_tensor_cores(self._h, int(enabled)))

    def layer_info(self, layer: int) -> KVLayerInfo:
        info = KVLayerInfo()
        _check(lib().nncu_kv_layer(self._h, layer, C.byref(info)))
        return info

    def state(self, seq: int = 0) -> KVState:
        st = KVState()
        _check(lib().nncu_kv_get_state(self._h, seq, C.byref(st)))
        return st

    def rewind(self, pos: int, seq: int = 0) -> bool:
        """model_kv_rewind: False (and nothing changed) when refused."""
        rc = lib().nncu_kv_rewind(self._h, seq, pos)
        if rc == ERR_INVALID_ARGUMENT:
            return False
        _check(rc)
        return True

    def commit(self, pos0: int, n_tok: int, seq: int = 0) -> None:
        _check(lib().nncu_kv_commit(self._h, seq, pos0, n_tok))

    def write_rows(self, layer: int, pos0: int, k_rows: np.ndarray, v_rows: np.ndarray, seq: int = 0) -> None:
        """Load rows [n][n_kv*head_dim] of the cache type's bits at positions pos0..
        (numpy arrays, or contiguous device tensors)."""
        n = k_rows.shape[0]
        if isinstance(k_rows, np.ndarray):
            k_rows, v_rows = np.ascontiguousarray(k_rows), np.ascontiguousarray(v_rows)
        _check(lib().nncu_kv_write_rows(self._h, layer, seq, pos0, n, _ptr(k_rows), _ptr(v_rows)))

    def read_rows(self, layer: int, pos0: int, n: int, seq: int = 0):
        info = self.layer_info(layer)
        dt = np.float32 if self.kv_type == KV_F32 else np.uint16
        k = np.empty((n, info.n_kv * info.head_dim), dt)
        v = np.empty_like(k)
        _check(lib().nncu_kv_read_rows(self._h, layer, seq, pos0, n, _ptr(k), _ptr(v)))
        return k, v

    def attention(self, layer: int, p: AttnParams, q: np.ndarray, k=None, v=None, seq: int = 0) -> np.ndarray:
        """attention_forward from the norms on: host fp32 rows in, host fp32 rows out."""
        q = np.ascontiguousarray(q, np.float32)
        k = None if k is None else np.ascontiguousarray(k, np.float32)
        v = None if v is None else np.ascontiguousarray(v, np.float32)
        out = np.empty((p.n_tok, p.n_head * p.head_dim), np.float32)
        _check(lib().nncu_attention(self._h, layer, seq, C.byref(p), _ptr(q), _ptr(k), _ptr(v), _ptr(out)))
        return out

    def attention_batch(self, jobs) -> None:
        """Many jobs, host pointers, one round trip. jobs: AttnJob sequence or
        ctypes array (outputs filled in place)."""
        arr = jobs if isinstance(jobs, C.Array) else (AttnJob * len(jobs))(*jobs)
        _check(lib().nncu_attention_batch(self._h, arr, len(arr)))

    def attention_batch_dev(self, jobs, stream=None) -> None:
        """Many jobs, device pointers, asynchronous on `stream` (an int handle or a torch stream)."""
        arr = jobs if isinstance(jobs, C.Array) else (AttnJob * len(jobs))(*jobs)
        _check(lib().nncu_attention_batch_dev(self._h, arr, len(arr), _stream(stream)))

    def attention_forward_dev(self, layer: int, p: AttnParams, w: AttnWeights, x, y, seq: int = 0,
                              stream=None) -> None:
        """nncu_attention_forward_dev: one layer's q / k / v projections,
        attention and output projection for p.n_tok tokens of `seq`; x and y
        are device arrays [n_tok][n_embd], asynchronous on `stream`."""
        _check(lib().nncu_attention_forward_dev(self._h, layer, seq, C.byref(p), C.byref(w), _ptr(x), _ptr(y),
                                                _stream(stream)))

    def attention_forward_batch_dev(self, layer: int, seqs, ps, w: AttnWeights, x, y, stream=None) -> None:
        """nncu_attention_forward_batch_dev: one layer for several sequences;
        ps: one AttnParams per sequence; x, y: the sequences' token rows one
        after another."""
        sa = (C.c_int32 * len(seqs))(*[int(s_) for s_ in seqs])
        pa = (AttnParams * len(ps))(*ps)
        _check(lib().nncu_attention_forward_batch_dev(self._h, layer, len(seqs), C.cast(sa, C.c_void_p), pa,
                                                      C.byref(w), _ptr(x), _ptr(y), _stream(stream)))

    def sync(self, stream=None) -> None:
        """Wait for `stream` and report a kernel's timed-out wait."""
        _check(lib().nncu_sync(self._h, _stream(stream)))


def attention_noalloc(p: AttnParams, q, k, v, out, k_cache, v_cache, kv_type: int, rows: int, stream=None) -> None:
    """nncu_attention_noalloc: one layer's attention on caller-owned device
    buffers (the cache laid out [n_kv][rows][head_dim]), with no allocation."""
    _check(lib().nncu_attention_noalloc(C.byref(p), _ptr(q), _ptr(k), _ptr(v), _ptr(out), _ptr(k_cache),
                                        _ptr(v_cache), int(kv_type), int(rows), _stream(stream)))


def noalloc_check(stream=None) -> None:
    """nncu_noalloc_check: wait for `stream`; raise (ERR_TIMEOUT) if a no-allocation
    call on the current device timed out since the last check."""
    _check(lib().nncu_noalloc_check(_stream(stream)))


def weight(kind: int, rows: int, cols: int, data, scales=None, biases=None) -> Weight:
    """A Weight over device arrays (torch tensors or raw pointers)."""
    w = Weight(int(kind), int(rows), int(cols), _ptr(data), _ptr(scales), _ptr(biases))
    w._keep = (data, scales, biases)
    return w


def logits_batch_dev(lm_head: Weight, hidden, n: int, logits, final_softcap: float = 0.0, xsum=None,
                     stream=None) -> None:
    """nncu_logits_batch_dev: model_logits_batch on the device."""
    _check(lib().nncu_logits_batch_dev(C.byref(lm_head), _ptr(hidden), int(n), _ptr(logits), float(final_softcap),
                                       _ptr(xsum), _stream(stream)))


def argmax_rows_dev(x, n_rows: int, n: int, out, x_stride=None, stream=None) -> None:
    """nncu_argmax_rows_dev: greedy verify's argmax of each row."""
    _check(lib().nncu_argmax_rows_dev(_ptr(x), int(x_stride if x_stride is not None else n), int(n_rows), int(n),
                                      _ptr(out), _stream(stream)))


def job(layer: int, p: AttnParams, q, k, v, out, seq: int = 0) -> AttnJob:
    j = AttnJob(layer, seq, p, _ptr(q), _ptr(k), _ptr(v), _ptr(out))
    j._keep = (p, q, k, v, out)
    return j


def _stream(s):
    if s is None:
        return None
    if isinstance(s, int):
        return s
    return s.cuda_stream  # torch.cuda.Stream


# ---- unit seam (device pointers) -------------------------------------------------------

def attn_block_dev(q, q_stride, K, V, kv_type, kv_stride, n_keys, head_dim, n_heads, scale, part, softcap=0.0,
                   stream=None):
    _check(lib().nncu_attn_block_dev(_ptr(q), q_stride, _ptr(K), _ptr(V), kv_type, kv_stride, n_keys, head_dim,
                                     n_heads, scale, softcap, _ptr(part), _stream(stream)))


def attn_merge_dev(acc, part, head_dim, n_heads, stream=None):
    _check(lib().nncu_attn_merge_dev(_ptr(acc), _ptr(part), head_dim, n_heads, _stream(stream)))


def attn_finish_dev(out, out_stride, acc, head_dim, n_heads, stream=None):
    _check(lib().nncu_attn_finish_dev(_ptr(out), out_stride, _ptr(acc), head_dim, n_heads, _stream(stream)))


def rmsnorm_gamma_multi_dev(y, x, n_groups, dim, gamma, eps, stream=None):
    _check(lib().nncu_rmsnorm_gamma_multi_dev(_ptr(y), _ptr(x), n_groups, dim, _ptr(gamma), eps, _stream(stream)))


def rmsnorm_dev(y, x, n_groups, dim, eps, stream=None):
    _check(lib().nncu_rmsnorm_dev(_ptr(y), _ptr(x), n_groups, dim, eps, _stream(stream)))


def rope_dev(x, n_tok, n_heads, head_dim, n_rot, pos0, pos_scale, freq_base, mode=ROPE_NEOX, freq_factors=None,
             stream=None):
    _check(lib().nncu_rope_dev(_ptr(x), n_tok, n_heads, head_dim, n_rot, pos0, pos_scale, freq_base, mode,
                               _ptr(freq_factors), _stream(stream)))


def softcap_dev(y, x, n, cap, stream=None):
    _check(lib().nncu_softcap_dev(_ptr(y), _ptr(x), n, cap, _stream(stream)))


def gemv_bf16w_dev(W, X, Y, rows, cols, n_batch=1, x_stride=None, y_stride=None, stream=None):
    """nnc_gemv_bf16w_f32x_batch on device buffers (tensors or pointers)."""
    _check(lib().nncu_gemv_bf16w_f32x_batch_dev(_ptr(W), _ptr(X), x_stride or cols, _ptr(Y), y_stride or rows, rows,
                                                cols, n_batch, _stream(stream)))


def gemv_q8_0_dev(qs, scales, X, Y, rows, cols, n_batch=1, x_stride=None, y_stride=None, stream=None):
    _check(lib().nncu_gemv_q8_0_f32x_batch_dev(_ptr(qs), _ptr(scales), _ptr(X), x_stride or cols, _ptr(Y),
                                               y_stride or rows, rows, cols, n_batch, _stream(stream)))


def gemv_q4_s_dev(qs, scales, biases, X, XSUM, Y, rows, cols, n_batch=1, x_stride=None, xsum_stride=None,
                  y_stride=None, stream=None):
    _check(lib().nncu_gemv_q4_s_f32x_batch_dev(_ptr(qs), _ptr(scales), _ptr(biases), _ptr(X), x_stride or cols,
                                               _ptr(XSUM), xsum_stride or cols // 32, _ptr(Y), y_stride or rows,
                                               rows, cols, n_batch, _stream(stream)))


def block_sums_dev(x, out, n, stream=None):
    _check(lib().nncu_block_sums_dev(_ptr(x), _ptr(out), n, _stream(stream)))


def gemv_bf16w_argmax_dev(W, x, rows, cols, scratch, out_index, stream=None):
    _check(lib().nncu_gemv_bf16w_argmax_dev(_ptr(W), _ptr(x), rows, cols, _ptr(scratch), _ptr(out_index),
                                            _stream(stream)))


# ---- one sequence split over the GPUs of a node (nncu_group) ----------------------------------

def split_ranges(n_keys: int, world: int, block: int = 256):
    """The key range of each rank: equal 256-aligned runs of the n_keys keys
    (the last one short). Raises if a rank would be left without keys."""
    per = -(-n_keys // world)
    chunk = -(-per // block) * block
    ranges = [(r * chunk, min((r + 1) * chunk, n_keys)) for r in range(world)]
    if any(hi <= lo for lo, hi in ranges):
        raise ValueError(f"{n_keys} keys leave a rank of {world} without keys")
    return ranges


def exchange_handles(handle: bytes, world: int):
    """Every rank's group handle, through the default torch.distributed group
    (host plumbing only: the handles are a few bytes)."""
    import torch.distributed as dist
    out = [None] * world
    dist.all_gather_object(out, handle)
    return out


class SplitGroup:
    """This GPU's part of a sequence split over `world` GPUs (nncu_group):
    rank r reads keys [key_lo, key_hi) and every GPU ends with the merged
    attention in its output rows."""

    def __init__(self, rank: int, world: int, max_rows: int, head_dim: int, device: int = 0, exchange=None):
        L = lib()
        h = C.c_void_p()
        _check(L.nncu_group_create(int(device), int(rank), int(world), int(max_rows), int(head_dim), C.byref(h)))
        self._h, self.rank, self.world, self.head_dim, self.max_rows = h, rank, world, head_dim, max_rows
        buf = C.create_string_buffer(GROUP_HANDLE_BYTES)
        _check(L.nncu_group_handle(self._h, buf))
        handles = (exchange or exchange_handles)(buf.raw, world)
        for r, hb in enumerate(handles):
            if r != rank:
                _check(L.nncu_group_open(self._h, r, C.create_string_buffer(hb, GROUP_HANDLE_BYTES)))

    def output_ptr(self) -> int:
        """Device address of this GPU's merged output rows (float32, head_dim each)."""
        return int(lib().nncu_group_output(self._h))

    def read_output(self, n_floats: int, stream=None) -> np.ndarray:
        """The first n_floats of this GPU's merged output, on the host (waits for `stream`)."""
        out = np.empty(int(n_floats), np.float32)
        _check(lib().nncu_group_copy_output(self._h, out.ctypes.data, out.size, _stream(stream)))
        import torch
        torch.cuda.synchronize()
        return out

    def attention(self, kv: "KVCache", jobs, key_lo: int, key_hi: int, stream=None) -> None:
        arr = jobs if isinstance(jobs, C.Array) else (AttnJob * len(jobs))(*jobs)
        _check(lib().nncu_attention_split_dev(kv._h, self._h, arr, len(arr), int(key_lo), int(key_hi),
                                               _stream(stream)))

    def set_timeout(self, ms: int) -> None:
        """The bounded wait of this GPU's end-of-call merge."""
        _check(lib().nncu_group_set_timeout(self._h, int(ms)))

    def reset(self) -> None:
        """nncu_group_reset: only at a step boundary every rank has reached."""
        _check(lib().nncu_group_reset(self._h))

    def inject_drop(self, n_calls: int) -> None:
        """Test injection: this rank's next n_calls calls never count their partials."""
        _check(lib().nncu_group_inject_drop(self._h, int(n_calls)))

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().nncu_group_free(self._h)
            self._h = None
