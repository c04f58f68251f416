"""ctypes binding to the reference's own CPU forward (oracle/_ref/libffwd_ref.so).

TEST INFRASTRUCTURE ONLY: the checker and the timed CPU baseline.  The library
is built from the unmodified reference sources by oracle/Makefile and wraps
``ffwd_model_load`` / ``ffwd_model_encode_batch`` (libffwd/forward.c:628-652).
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_ref", "libffwd_ref.so")
_lib = None


def available() -> bool:
    return os.path.exists(LIB_PATH)


def lib():
    global _lib
    if _lib is None:
        l = ctypes.CDLL(LIB_PATH)
        l.ref_load.restype = ctypes.c_void_p
        l.ref_load.argtypes = [ctypes.c_char_p]
        l.ref_free.argtypes = [ctypes.c_void_p]
        l.ref_set_threads.argtypes = [ctypes.c_int]
        l.ref_config.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        l.ref_encode.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                 ctypes.c_void_p]
        l.ref_encode_spans.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] + [
            ctypes.c_void_p] * 4
        l.ref_forward.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
        l.ref_late_load.restype = ctypes.c_void_p
        l.ref_late_load.argtypes = [ctypes.c_char_p]
        l.ref_late_free.argtypes = [ctypes.c_void_p]
        l.ref_late_token_dim.argtypes = [ctypes.c_void_p]
        l.ref_late_encode_tokens.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                             ctypes.c_int, ctypes.c_void_p]
        l.ref_late_encode_docs.argtypes = [ctypes.c_void_p] + [ctypes.c_void_p] * 4 + [
            ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
        l.ref_late_maxsim_batch.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                            ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_void_p]
        _lib = l
    return _lib


class RefModel:
    def __init__(self, model_dir: str, threads: int = 1):
        self.l = lib()
        self.l.ref_set_threads(int(threads))
        self.h = self.l.ref_load(model_dir.encode())
        if not self.h:
            raise RuntimeError(f"reference failed to load {model_dir}")
        ints = np.zeros(18, dtype=np.int32)
        floats = np.zeros(3, dtype=np.float32)
        self.l.ref_config(self.h, ints.ctypes.data, floats.ctypes.data)
        self.ints, self.floats = ints, floats
        self.hidden = int(ints[2])

    def set_threads(self, n: int):
        self.l.ref_set_threads(int(n))

    def encode_batch(self, seqs) -> np.ndarray:
        ids = np.ascontiguousarray(np.concatenate([np.asarray(s, np.int32) for s in seqs]))
        lens = np.ascontiguousarray(np.array([len(s) for s in seqs], dtype=np.int32))
        out = np.zeros((len(seqs), self.hidden), dtype=np.float32)
        rc = self.l.ref_encode(self.h, ids.ctypes.data, lens.ctypes.data, len(seqs), out.ctypes.data)
        if rc != 0:
            raise RuntimeError("reference encode failed")
        return out

    def encode_spans(self, docs, spans) -> np.ndarray:
        """ffwd_model_encode_spans_batch: docs (id arrays), spans per doc as
        (start, n_tokens) pairs; one unnormalised mean row per span."""
        ids = np.ascontiguousarray(np.concatenate([np.asarray(d, np.int32) for d in docs]))
        lens = np.ascontiguousarray(np.array([len(d) for d in docs], np.int32))
        ns = np.ascontiguousarray(np.array([len(sp) for sp in spans], np.int32))
        st = np.ascontiguousarray(np.array([a for sp in spans for a, _ in sp], np.int32))
        ln = np.ascontiguousarray(np.array([n for sp in spans for _, n in sp], np.int32))
        out = np.zeros((int(ns.sum()), self.hidden), dtype=np.float32)
        if self.l.ref_encode_spans(self.h, ids.ctypes.data, lens.ctypes.data, len(docs),
                                   ns.ctypes.data, st.ctypes.data, ln.ctypes.data,
                                   out.ctypes.data) != 0:
            raise RuntimeError("reference encode_spans failed")
        return out

    def forward_states(self, ids) -> np.ndarray:
        ids = np.ascontiguousarray(np.asarray(ids, np.int32))
        out = np.zeros((len(ids), self.hidden), dtype=np.float32)
        if self.l.ref_forward(self.h, ids.ctypes.data, len(ids), out.ctypes.data) != 0:
            raise RuntimeError("reference forward failed")
        return out

    def close(self):
        if self.h:
            self.l.ref_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class RefLate:
    """The reference's CPU late-interaction model (libffwd/late.c, late_blas.c)."""

    def __init__(self, model_dir: str, threads: int = 1):
        self.l = lib()
        self.l.ref_set_threads(int(threads))
        self.h = self.l.ref_late_load(model_dir.encode())
        if not self.h:
            raise RuntimeError(f"reference failed to load late model {model_dir}")
        self.dim = int(self.l.ref_late_token_dim(self.h))

    def encode_tokens(self, ids, normalize=True) -> np.ndarray:
        ids = np.ascontiguousarray(np.asarray(ids, np.int32))
        out = np.zeros((len(ids), self.dim), np.float32)
        if self.l.ref_late_encode_tokens(self.h, ids.ctypes.data, len(ids), int(normalize),
                                         out.ctypes.data) != 0:
            raise RuntimeError("reference late encode_tokens failed")
        return out

    def encode_docs(self, docs, keeps, normalize=True):
        ids = np.ascontiguousarray(np.concatenate([np.asarray(d, np.int32) for d in docs]))
        lens = np.ascontiguousarray(np.array([len(d) for d in docs], np.int32))
        keep = np.ascontiguousarray(np.concatenate([np.asarray(k, np.int32) for k in keeps]))
        nk = np.ascontiguousarray(np.array([len(k) for k in keeps], np.int32))
        out = np.zeros((int(nk.sum()), self.dim), np.float32)
        offs = np.zeros(len(docs) + 1, np.int32)
        if self.l.ref_late_encode_docs(self.h, ids.ctypes.data, lens.ctypes.data, keep.ctypes.data,
                                       nk.ctypes.data, len(docs), int(normalize), out.ctypes.data,
                                       offs.ctypes.data) != 0:
            raise RuntimeError("reference late encode_docs failed")
        return out, offs

    def maxsim_batch(self, q, docs, offs) -> np.ndarray:
        q = np.ascontiguousarray(q, np.float32)
        docs = np.ascontiguousarray(docs, np.float32)
        offs = np.ascontiguousarray(offs, np.int32)
        scores = np.zeros(len(offs) - 1, np.float32)
        if self.l.ref_late_maxsim_batch(q.ctypes.data, len(q), docs.ctypes.data, offs.ctypes.data,
                                        len(offs) - 1, q.shape[1], scores.ctypes.data) != 0:
            raise RuntimeError("reference maxsim failed")
        return scores

    def rerank(self, query, query_n_keep, docs, keeps) -> np.ndarray:
        """The reference's ffwd_rerank (backend_cuda.c:132-156) on its CPU path."""
        qv = self.encode_tokens(query, True)
        dv, offs = self.encode_docs(docs, keeps, True)
        return self.maxsim_batch(qv[:query_n_keep], dv, offs)

    def close(self):
        if self.h:
            self.l.ref_late_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
