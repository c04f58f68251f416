"""ctypes binding to the reference's own CUDA backend (oracle/_ref/libffwd_refcuda.so).

TEST INFRASTRUCTURE ONLY: built by ``make -C oracle cuda`` from the unmodified
libffwd/cuda.cu and cuda_sdpa.cu (cuBLAS / cuBLASLt GEMMs, the reference's
mma.sync attention kernels, cuDNN SDPA when libcudnn loads) for sm_100a.  It
is timed beside this backend on the same GPU and its rows are compared with
the CPU reference; nothing in ffwd_b200 loads it.  Entry points follow
libffwd/cuda.h:22-68 (``ffwd_cuda_set_fast_gemm``, ``ffwd_cuda_load``,
``ffwd_cuda_encode_batch``, ``ffwd_cuda_free``).

Run it in a process of its own: a failure inside it must not take down the
caller's CUDA context.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_ref", "libffwd_refcuda.so")


class _Input(ctypes.Structure):  # ffwd_input_t (libffwd/ffwd.h:91-94)
    _fields_ = [("ids", ctypes.POINTER(ctypes.c_int)), ("n_tokens", ctypes.c_int)]


def available() -> bool:
    return os.path.exists(LIB_PATH)


class RefCudaModel:
    def __init__(self, model_dir: str, gemm_mode: str = "bf16"):
        l = ctypes.CDLL(LIB_PATH)
        l.ffwd_cuda_set_fast_gemm.argtypes = [ctypes.c_char_p]
        l.ffwd_cuda_load.restype = ctypes.c_void_p
        l.ffwd_cuda_load.argtypes = [ctypes.c_char_p]
        l.ffwd_cuda_free.argtypes = [ctypes.c_void_p]
        l.ffwd_cuda_encode_batch.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                             ctypes.c_void_p]
        l.ffwd_cuda_config.restype = ctypes.POINTER(ctypes.c_int * 4)
        l.ffwd_cuda_config.argtypes = [ctypes.c_void_p]
        self.l = l
        if l.ffwd_cuda_set_fast_gemm(gemm_mode.encode()) != 0:
            raise RuntimeError(f"reference CUDA backend rejected gemm mode {gemm_mode}")
        self.h = l.ffwd_cuda_load(model_dir.encode())
        if not self.h:
            raise RuntimeError(f"reference CUDA backend failed to load {model_dir}")
        self.hidden = int(l.ffwd_cuda_config(self.h).contents[2])  # ffwd_config_t.hidden_size

    def pack(self, seqs):
        arrs = [np.ascontiguousarray(np.asarray(s, np.int32)) for s in seqs]
        ins = (_Input * len(arrs))()
        for i, a in enumerate(arrs):
            ins[i].ids = a.ctypes.data_as(ctypes.POINTER(ctypes.c_int))
            ins[i].n_tokens = int(a.size)
        return ins, arrs

    def encode_packed(self, ins, n, out) -> int:
        return self.l.ffwd_cuda_encode_batch(self.h, ins, n, out.ctypes.data)

    def encode_batch(self, seqs) -> np.ndarray:
        ins, keep = self.pack(seqs)
        out = np.zeros((len(seqs), self.hidden), np.float32)
        if self.encode_packed(ins, len(seqs), out) != 0:
            raise RuntimeError("reference ffwd_cuda_encode_batch failed")
        return out

    def close(self):
        if self.h:
            self.l.ffwd_cuda_free(self.h)
            self.h = None


def main(argv=None):
    """python -m oracle.refcuda MODEL_DIR STEPS WARMUP SEED [OUT.npy [CONFIG [MODE [BATCH]]]]:
    time the reference CUDA backend's ffwd_cuda_encode_batch on a seeded batch
    of a BASELINE config (default the Qwen3-0.6B bench batch, bf16 GEMMs; host
    ids in, host rows out, synchronous: the call a server makes) and print one
    JSON line; the rows of the last call go to OUT.npy."""
    import json
    import sys
    import time

    sys.path.insert(0, os.path.dirname(_HERE))
    from ffwd_b200 import synth

    a = argv if argv is not None else sys.argv[1:]
    model_dir, steps, warmup, seed = a[0], int(a[1]), int(a[2]), int(a[3])
    config = a[5] if len(a) > 5 else "qwen3-0.6b"
    mode = a[6] if len(a) > 6 else "bf16"
    batch = int(a[7]) if len(a) > 7 else None
    seqs = synth.token_batch(config, seed=seed, batch=batch)
    m = RefCudaModel(model_dir, mode)
    ins, keep = m.pack(seqs)
    out = np.zeros((len(seqs), m.hidden), np.float32)
    for _ in range(warmup):
        if m.encode_packed(ins, len(seqs), out) != 0:
            raise RuntimeError("reference ffwd_cuda_encode_batch failed")
    t0 = time.perf_counter()
    for _ in range(steps):
        if m.encode_packed(ins, len(seqs), out) != 0:
            raise RuntimeError("reference ffwd_cuda_encode_batch failed")
    dt = (time.perf_counter() - t0) / steps
    m.close()
    if len(a) > 4 and a[4] != "-":
        np.save(a[4], out)
    tokens = sum(len(s) for s in seqs)
    print(json.dumps({"value": tokens / dt, "unit": "tokens/s", "ms_per_call": 1000 * dt,
                      "tokens_per_call": tokens, "calls": steps}), flush=True)


if __name__ == "__main__":
    main()
