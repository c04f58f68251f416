"""ctypes binding of the B200 backend's C ABI (include/ffwd_b200.h).

Mirrors the reference backend's operator interface (libffwd/cuda.h: load,
config, encode_into, encode_batch, encode_spans_batch; and the public
libffwd/ffwd.h API through :class:`FfwdApi`) with the same argument meaning and
error behaviour: calls return -1 / raise on invalid input, never fall back.
There is no CPU path here: if the CUDA library is missing the import fails.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libffwd_b200.so")
API_LIB_PATH = os.path.join(_HERE, "lib", "libffwd_b200_api.so")


class FfwdError(RuntimeError):
    pass


class ffwd_input_t(ctypes.Structure):
    _fields_ = [("ids", ctypes.POINTER(ctypes.c_int)), ("n_tokens", ctypes.c_int)]


class ffwd_span_t(ctypes.Structure):
    _fields_ = [("start", ctypes.c_int), ("n_tokens", ctypes.c_int)]


class ffwd_context_input_t(ctypes.Structure):
    _fields_ = [("input", ffwd_input_t), ("spans", ctypes.POINTER(ffwd_span_t)),
                ("n_spans", ctypes.c_int)]


class ffwd_config_t(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in (
        "family", "ffn_act", "hidden_size", "n_layers", "n_heads", "n_kv_heads", "head_dim",
        "q_dim", "kv_dim", "intermediate_size", "vocab_size", "max_position_embeddings",
        "position_id_offset", "type_vocab_size")] + [
        ("rms_norm_eps", ctypes.c_float), ("layer_norm_eps", ctypes.c_float),
        ("rope_theta", ctypes.c_float)] + [(n, ctypes.c_int) for n in (
            "qk_norm", "qkv_bias", "attention_mode", "pooling_mode", "normalize_embeddings",
            "append_terminal_token")]


class ffwd_rerank_input_t(ctypes.Structure):
    _fields_ = [("query_ids", ctypes.POINTER(ctypes.c_int)), ("query_n_tokens", ctypes.c_int),
                ("query_n_keep", ctypes.c_int),
                ("doc_ids", ctypes.POINTER(ctypes.POINTER(ctypes.c_int))),
                ("doc_n_tokens", ctypes.POINTER(ctypes.c_int)),
                ("doc_keep", ctypes.POINTER(ctypes.POINTER(ctypes.c_int))),
                ("doc_n_keep", ctypes.POINTER(ctypes.c_int)), ("n_docs", ctypes.c_int)]


class ffwd_options_t(ctypes.Structure):
    _fields_ = [("n_threads", ctypes.c_int), ("gpu_quant_bits", ctypes.c_int),
                ("gpu_quant_group_size", ctypes.c_int), ("gpu_gemm_mode", ctypes.c_char_p),
                ("gpu_weight_dtype", ctypes.c_char_p), ("memory_utilization", ctypes.c_double)]


# Every exported function of include/ffwd_b200.h: (restype, argtypes).
ABI = {
    "ffwd_b200_set_fast_gemm": (ctypes.c_int, [ctypes.c_char_p]),
    "ffwd_b200_set_weights_bf16": (ctypes.c_int, [ctypes.c_int]),
    "ffwd_b200_set_weights_f16": (ctypes.c_int, [ctypes.c_int]),
    "ffwd_b200_set_weights_default": (ctypes.c_int, []),
    "ffwd_b200_load": (ctypes.c_void_p, [ctypes.c_char_p]),
    "ffwd_b200_free": (None, [ctypes.c_void_p]),
    "ffwd_b200_config": (ctypes.POINTER(ffwd_config_t), [ctypes.c_void_p]),
    "ffwd_b200_encode_into": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                             ctypes.c_void_p]),
    "ffwd_b200_encode": (ctypes.c_void_p, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]),
    "ffwd_b200_encode_batch": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                              ctypes.c_void_p]),
    "ffwd_b200_encode_spans_batch": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p,
                                                    ctypes.c_int, ctypes.c_void_p]),
    "ffwd_b200_set_devices": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "ffwd_b200_set_max_tokens": (ctypes.c_int, [ctypes.c_int]),
    "ffwd_b200_encode_device": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                               ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                               ctypes.c_int]),
    "ffwd_b200_encode_device_noalloc": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int,
                                                       ctypes.c_void_p, ctypes.c_void_p,
                                                       ctypes.c_int, ctypes.c_void_p]),
    "ffwd_b200_stream": (ctypes.c_void_p, [ctypes.c_void_p, ctypes.c_int]),
    "ffwd_b200_shard_stats": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                             ctypes.c_void_p, ctypes.c_int]),
    "ffwd_b200_test_inject": (ctypes.c_int, [ctypes.c_int, ctypes.c_int]),
    "ffwd_b200_selftest_wait": (ctypes.c_int, [ctypes.c_int, ctypes.c_int]),
    "ffwd_b200_run_op": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_int]),
    "ffwd_b200_launch_count": (ctypes.c_longlong, []),
    "ffwd_b200_last_error": (ctypes.c_char_p, []),
    "ffwd_b200_precision": (ctypes.c_int, [ctypes.c_void_p]),
    "ffwd_b200_lpt_partition": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                               ctypes.c_void_p]),
    "ffwd_b200_attention_items": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                 ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                                 ctypes.c_void_p, ctypes.c_int]),
    "ffwd_b200_gemm_bf16": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                           ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                           ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    "ffwd_b200_gemm_tf32": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                           ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    "ffwd_b200_encode_batch_as": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                                 ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                 ctypes.c_void_p]),
    "ffwd_b200_late_load": (ctypes.c_void_p, [ctypes.c_char_p]),
    "ffwd_b200_late_free": (None, [ctypes.c_void_p]),
    "ffwd_b200_late_config": (ctypes.POINTER(ffwd_config_t), [ctypes.c_void_p]),
    "ffwd_b200_late_token_dim": (ctypes.c_int, [ctypes.c_void_p]),
    "ffwd_b200_late_encode_tokens": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                                    ctypes.c_int, ctypes.c_void_p]),
    "ffwd_b200_late_encode_docs": (ctypes.c_int, [ctypes.c_void_p] + [ctypes.c_void_p] * 4 + [
        ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]),
    "ffwd_b200_late_rerank": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
}

# The reference-facing public API (include/ffwd_b200_api.h).
API_ABI = {
    "ffwd_init": (ctypes.c_int, [ctypes.POINTER(ffwd_options_t), ctypes.c_char_p, ctypes.c_size_t]),
    "ffwd_open": (ctypes.c_void_p, [ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(ffwd_options_t),
                                    ctypes.c_char_p, ctypes.c_size_t]),
    "ffwd_activate": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]),
    "ffwd_worker_free": (None, [ctypes.c_void_p]),
    "ffwd_free": (None, [ctypes.c_void_p]),
    "ffwd_config": (ctypes.POINTER(ffwd_config_t), [ctypes.c_void_p]),
    "ffwd_token_dim": (ctypes.c_int, [ctypes.c_void_p]),
    "ffwd_uses_dense_batches": (ctypes.c_int, [ctypes.c_void_p]),
    "ffwd_encode_batch": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                         ctypes.c_void_p]),
    "ffwd_encode_spans_batch": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                               ctypes.c_void_p]),
    "ffwd_rerank": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "ffwd_scratch_nbytes": (ctypes.c_size_t, [ctypes.c_void_p]),
    "ffwd_capability": (ctypes.c_char_p, []),
    "ffwd_default_batch_wait_us": (ctypes.c_int, []),
    "ffwd_preflight": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                      ctypes.c_char_p, ctypes.c_size_t]),
    "ffwd_l2_normalize": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "ffwd_cosine_similarity": (ctypes.c_float, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]),
    "ffwd_b200_api_context": (ctypes.c_void_p, [ctypes.c_void_p]),
}

_lib = None
_api = None


def _bind(path, table):
    if not os.path.exists(path):
        raise ImportError(f"ffwd_b200 native library missing: {path} (run ffwd_b200/build.py)")
    lib = ctypes.CDLL(path)
    for name, (res, args) in table.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


def lib():
    global _lib
    if _lib is None:
        _lib = _bind(LIB_PATH, ABI)
    return _lib


def api():
    global _api
    if _api is None:
        _api = _bind(API_LIB_PATH, {**ABI, **API_ABI})
    return _api


INJECT_NONE, INJECT_SHARD, INJECT_ALLOC = 0, 1, 2


def test_inject(kind: int, value: int = 0, library=None) -> int:
    """Host-side fault injection (ffwd_b200_test_inject) in `library` (default
    libffwd_b200.so; the API library keeps its own copy of the switches)."""
    return (library or lib()).ffwd_b200_test_inject(int(kind), int(value))


def shard_stats(ctx, library=None):
    """[(sequences, tokens, host ms)] per device entry of the last encode_batch."""
    L = library or lib()
    n = L.ffwd_b200_shard_stats(ctx, None, None, None, 0)
    if n <= 0:
        return []
    seqs = np.zeros(n, np.int32)
    toks = np.zeros(n, np.int64)
    ms = np.zeros(n, np.float64)
    L.ffwd_b200_shard_stats(ctx, seqs.ctypes.data, toks.ctypes.data, ms.ctypes.data, n)
    return [(int(a), int(b), float(c)) for a, b, c in zip(seqs, toks, ms)]


def last_error() -> str:
    return (lib().ffwd_b200_last_error() or b"").decode()


def _pack_inputs(seqs):
    arrs = [np.ascontiguousarray(np.asarray(s, dtype=np.int32)) for s in seqs]
    ins = (ffwd_input_t * len(arrs))()
    for i, a in enumerate(arrs):
        ins[i].ids = a.ctypes.data_as(ctypes.POINTER(ctypes.c_int)) if a.size else None
        ins[i].n_tokens = int(a.size)
    return ins, arrs


def set_fast_gemm(mode: str) -> int:
    return lib().ffwd_b200_set_fast_gemm(mode.encode())


class B200Model:
    """One loaded model (the reference's ffwd_cuda_ctx_t)."""

    def __init__(self, model_dir: str, gemm_mode: str | None = None,
                 weight_dtype: str | None = None, devices=None, max_tokens: int | None = None):
        L = lib()
        if gemm_mode is not None and L.ffwd_b200_set_fast_gemm(gemm_mode.encode()) != 0:
            raise FfwdError("--gpu-gemm-mode must be f32, tf32, bf16, or 16f")
        if weight_dtype is not None:
            if weight_dtype == "bf16":
                L.ffwd_b200_set_weights_bf16(1)
            elif weight_dtype in ("f16", "fp16"):
                L.ffwd_b200_set_weights_f16(1)
            elif weight_dtype == "f32":
                L.ffwd_b200_set_weights_bf16(0)
            elif weight_dtype == "file":
                L.ffwd_b200_set_weights_default()
            else:
                raise FfwdError("--gpu-weight-dtype must be f32, bf16, or f16")
        if devices is not None:
            d = (ctypes.c_int * len(devices))(*devices)
            if L.ffwd_b200_set_devices(d, len(devices)) != 0:
                raise FfwdError("bad device list")
        if max_tokens is not None:
            L.ffwd_b200_set_max_tokens(int(max_tokens))
        self._l = L
        self.h = L.ffwd_b200_load(model_dir.encode())
        if not self.h:
            raise FfwdError(f"failed to load model: {last_error()}")
        self.config = L.ffwd_b200_config(self.h).contents
        self.hidden = self.config.hidden_size
        self.precision = L.ffwd_b200_precision(self.h)

    def encode_batch(self, seqs) -> np.ndarray:
        ins, keep = _pack_inputs(seqs)
        out = np.zeros((len(seqs), self.hidden), dtype=np.float32)
        rc = self._l.ffwd_b200_encode_batch(self.h, ins, len(seqs), out.ctypes.data)
        if rc != 0:
            raise FfwdError(f"encode_batch failed: {last_error()}")
        return out

    ENCODINGS = {"f32": (0, np.float32), "int8": (1, np.int8), "binary": (2, np.uint8)}

    def encode_batch_as(self, seqs, dims: int, renormalize: bool, encoding: str) -> np.ndarray:
        """Embeddings in a wire form made on the device: f32 [n, dims], int8
        [n, dims] or binary [n, dims / 8] bytes."""
        enc, dt = self.ENCODINGS[encoding]
        ins, keep = _pack_inputs(seqs)
        width = dims // 8 if encoding == "binary" else dims
        out = np.zeros((len(seqs), max(width, 1)), dtype=dt)
        if self._l.ffwd_b200_encode_batch_as(self.h, ins, len(seqs), int(dims), int(renormalize),
                                             enc, out.ctypes.data) != 0:
            raise FfwdError(f"encode_batch_as failed: {last_error()}")
        return out

    def try_encode_batch(self, seqs):
        """Return code + output (reference-style -1 on failure)."""
        ins, keep = _pack_inputs(seqs)
        out = np.zeros((max(len(seqs), 1), self.hidden), dtype=np.float32)
        rc = self._l.ffwd_b200_encode_batch(self.h, ins, len(seqs), out.ctypes.data)
        return rc, out

    def encode_into(self, ids) -> np.ndarray:
        a = np.ascontiguousarray(np.asarray(ids, dtype=np.int32))
        out = np.zeros(self.hidden, dtype=np.float32)
        if self._l.ffwd_b200_encode_into(self.h, a.ctypes.data, int(a.size), out.ctypes.data) != 0:
            raise FfwdError(f"encode_into failed: {last_error()}")
        return out

    def encode_spans_batch(self, docs, spans) -> np.ndarray:
        """docs: list of id arrays; spans: list (per doc) of (start, n_tokens)."""
        arrs = [np.ascontiguousarray(np.asarray(d, dtype=np.int32)) for d in docs]
        sp = [(ffwd_span_t * len(s))(*[ffwd_span_t(a, b) for a, b in s]) for s in spans]
        ins = (ffwd_context_input_t * len(docs))()
        for i, a in enumerate(arrs):
            ins[i].input.ids = a.ctypes.data_as(ctypes.POINTER(ctypes.c_int))
            ins[i].input.n_tokens = int(a.size)
            ins[i].spans = ctypes.cast(sp[i], ctypes.POINTER(ffwd_span_t))
            ins[i].n_spans = len(spans[i])
        total = sum(len(s) for s in spans)
        out = np.zeros((total, self.hidden), dtype=np.float32)
        if self._l.ffwd_b200_encode_spans_batch(self.h, ins, len(docs), out.ctypes.data) != 0:
            raise FfwdError(f"encode_spans_batch failed: {last_error()}")
        return out

    def encode_device(self, d_ids: int, offsets, d_out: int, dev: int = 0, sync: bool = True):
        off = np.ascontiguousarray(np.asarray(offsets, dtype=np.int32))
        rc = self._l.ffwd_b200_encode_device(self.h, dev, d_ids, off.ctypes.data, len(off) - 1,
                                             d_out, 1 if sync else 0)
        if rc != 0:
            raise FfwdError(f"encode_device failed: {last_error()}")

    def encode_device_noalloc(self, d_ids: int, offsets, d_out: int, dev: int = 0) -> int:
        """Return code of the no-allocation entry (0 or -1)."""
        off = np.ascontiguousarray(np.asarray(offsets, dtype=np.int32))
        return self._l.ffwd_b200_encode_device_noalloc(self.h, dev, d_ids, off.ctypes.data,
                                                       len(off) - 1, d_out)

    def run_op(self, op: int, layer: int = 0, reps: int = 1, dev: int = 0):
        if self._l.ffwd_b200_run_op(self.h, dev, op, layer, reps) != 0:
            raise FfwdError(f"run_op failed: {last_error()}")

    def stream(self, dev: int = 0) -> int:
        return self._l.ffwd_b200_stream(self.h, dev) or 0

    def close(self):
        if getattr(self, "h", None):
            self._l.ffwd_b200_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class _DocArrays:
    """Pointer arrays (int *const *) over a list of int32 arrays, kept alive."""

    def __init__(self, arrays):
        self.arrs = [np.ascontiguousarray(np.asarray(a, dtype=np.int32)) for a in arrays]
        self.ptrs = (ctypes.POINTER(ctypes.c_int) * len(self.arrs))(
            *[a.ctypes.data_as(ctypes.POINTER(ctypes.c_int)) for a in self.arrs])
        self.lens = np.ascontiguousarray(np.array([a.size for a in self.arrs], dtype=np.int32))


def rerank_input(query, query_n_keep, docs, keeps):
    """ffwd_rerank_input_t over numpy arrays; returns (struct, keep-alive)."""
    q = np.ascontiguousarray(np.asarray(query, dtype=np.int32))
    d, k = _DocArrays(docs), _DocArrays(keeps)
    rin = ffwd_rerank_input_t(q.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), int(q.size),
                              int(query_n_keep), d.ptrs,
                              d.lens.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), k.ptrs,
                              k.lens.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), len(d.arrs))
    return rin, (q, d, k)


class B200Late:
    """A late-interaction model (the reference's ffwd_cuda_late_ctx_t)."""

    def __init__(self, model_dir: str, gemm_mode: str | None = None):
        L = lib()
        if gemm_mode is not None and L.ffwd_b200_set_fast_gemm(gemm_mode.encode()) != 0:
            raise FfwdError("--gpu-gemm-mode must be f32, tf32, bf16, or 16f")
        self._l = L
        self.h = L.ffwd_b200_late_load(model_dir.encode())
        if not self.h:
            raise FfwdError(f"failed to load late model: {last_error()}")
        self.config = L.ffwd_b200_late_config(self.h).contents
        self.dim = L.ffwd_b200_late_token_dim(self.h)

    def encode_tokens(self, ids, normalize=True) -> np.ndarray:
        a = np.ascontiguousarray(np.asarray(ids, dtype=np.int32))
        out = np.zeros((a.size, self.dim), dtype=np.float32)
        if self._l.ffwd_b200_late_encode_tokens(self.h, a.ctypes.data, int(a.size),
                                                int(normalize), out.ctypes.data) != 0:
            raise FfwdError(f"late_encode_tokens failed: {last_error()}")
        return out

    def encode_docs(self, docs, keeps, normalize=True):
        d, k = _DocArrays(docs), _DocArrays(keeps)
        out = np.zeros((int(k.lens.sum()), self.dim), dtype=np.float32)
        offs = np.zeros(len(docs) + 1, dtype=np.int32)
        if self._l.ffwd_b200_late_encode_docs(self.h, d.ptrs, d.lens.ctypes.data, k.ptrs,
                                              k.lens.ctypes.data, len(docs), int(normalize),
                                              out.ctypes.data, offs.ctypes.data) != 0:
            raise FfwdError(f"late_encode_docs failed: {last_error()}")
        return out, offs

    def rerank(self, query, query_n_keep, docs, keeps) -> np.ndarray:
        rin, keep = rerank_input(query, query_n_keep, docs, keeps)
        scores = np.zeros(len(docs), dtype=np.float32)
        if self._l.ffwd_b200_late_rerank(self.h, ctypes.byref(rin), scores.ctypes.data) != 0:
            raise FfwdError(f"late_rerank failed: {last_error()}")
        return scores

    def close(self):
        if getattr(self, "h", None):
            self._l.ffwd_b200_late_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def launch_count() -> int:
    return int(lib().ffwd_b200_launch_count())


def lpt_partition(costs, n_parts: int) -> np.ndarray:
    c = np.ascontiguousarray(np.asarray(costs, dtype=np.float64))
    part = np.zeros(len(c), dtype=np.int32)
    if lib().ffwd_b200_lpt_partition(c.ctypes.data, len(c), n_parts, part.ctypes.data) != 0:
        raise FfwdError("lpt_partition failed")
    return part


def attention_items(lens, n_heads, n_kv_heads, causal=True, windows=False) -> np.ndarray:
    """The forward's attention work list for sequences of these lengths:
    [n, 7] int32 rows (seq, qt0, h0, qt1, h1, key tiles, window sequences).
    windows=True: the 16-bit plans' list, short neighbours sharing items."""
    offs = np.ascontiguousarray(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32))
    L = lib()
    n = L.ffwd_b200_attention_items(int(causal), int(windows), n_heads, n_kv_heads,
                                    offs.ctypes.data, len(lens), None, 0)
    if n < 0:
        raise FfwdError("attention_items failed")
    out = np.zeros((max(n, 1), 7), np.int32)
    got = L.ffwd_b200_attention_items(int(causal), int(windows), n_heads, n_kv_heads,
                                      offs.ctypes.data, len(lens), out.ctypes.data, n)
    if got < 0 or got > n:
        raise FfwdError("attention_items failed")
    return out[:got]


def gemm_bf16(x_ptr, w_ptr, y_ptr, M, N, K, bn=256, x_lo_ptr=None, w_lo_ptr=None):
    rc = lib().ffwd_b200_gemm_bf16(x_ptr, x_lo_ptr, w_ptr, w_lo_ptr, y_ptr, M, N, K, bn)
    if rc != 0:
        raise FfwdError(f"gemm failed: {last_error()}")


def gemm_tf32(x_ptr, w_ptr, y_ptr, M, N, K, bn=256):
    rc = lib().ffwd_b200_gemm_tf32(x_ptr, w_ptr, y_ptr, M, N, K, bn)
    if rc != 0:
        raise FfwdError(f"gemm failed: {last_error()}")


class FfwdApi:
    """The reference's public API (libffwd/ffwd.h) served by libffwd_b200_api.so."""

    def __init__(self, model_dir: str, gemm_mode: str | None = None,
                 weight_dtype: str | None = None, is_late: bool = False):
        A = api()
        self._a = A
        err = ctypes.create_string_buffer(256)
        opts = ffwd_options_t(0, 0, 0, gemm_mode.encode() if gemm_mode else None,
                              weight_dtype.encode() if weight_dtype else None, 0.0)
        if A.ffwd_init(ctypes.byref(opts), err, 256) != 0:
            raise FfwdError(err.value.decode())
        self.e = A.ffwd_open(model_dir.encode(), int(is_late), ctypes.byref(opts), err, 256)
        if not self.e:
            raise FfwdError(err.value.decode())
        if A.ffwd_activate(self.e, err, 256) != 0:
            A.ffwd_free(self.e)
            self.e = None
            raise FfwdError(err.value.decode())
        self.config = A.ffwd_config(self.e).contents
        self.hidden = self.config.hidden_size

    def token_dim(self) -> int:
        return self._a.ffwd_token_dim(self.e)

    def rerank(self, query, query_n_keep, docs, keeps) -> np.ndarray:
        rin, keep = rerank_input(query, query_n_keep, docs, keeps)
        scores = np.zeros(len(docs), dtype=np.float32)
        if self._a.ffwd_rerank(self.e, ctypes.byref(rin), scores.ctypes.data) != 0:
            raise FfwdError("ffwd_rerank failed")
        return scores

    def encode_batch_into(self, ins, n, out) -> int:
        return self._a.ffwd_encode_batch(self.e, ins, n, out)

    def shard_stats(self):
        """Per device entry of the last encode: (sequences, tokens, host ms)."""
        return shard_stats(self._a.ffwd_b200_api_context(self.e), self._a)

    def encode_batch(self, seqs) -> np.ndarray:
        ins, keep = _pack_inputs(seqs)
        out = np.zeros((len(seqs), self.hidden), dtype=np.float32)
        if self._a.ffwd_encode_batch(self.e, ins, len(seqs), out.ctypes.data) != 0:
            raise FfwdError("ffwd_encode_batch failed")
        return out

    def close(self):
        if getattr(self, "e", None):
            self._a.ffwd_worker_free(self.e)
            self._a.ffwd_free(self.e)
            self.e = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
