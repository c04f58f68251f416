"""The no-allocation entry point (ffwd_b200_encode_device_noalloc), called
through the C ABI, against the existing device-resident entry point
(ffwd_b200_encode_device) on the same inputs, on two calls in a row, and
against the CPU checker.

It serves callers that cannot allocate device memory while serving (a host
that owns all GPU memory through its own pool, or a latency-sensitive caller
that must not hit cudaMalloc / cudaFree on the request path); its scratch is a
fixed arena reserved in device memory.  Both entries run the same kernels on
the same inputs, so their outputs must be bitwise equal; every precision plan
is covered, since each one carves the arena differently (split-bf16 lo
buffers, 4-byte tf32 operands, f32 qkv).  This file is collected last so that
a stop-at-first-failure run has already run every other test."""

import numpy as np
import pytest

from ffwd_b200 import native, synth
from oracle import forward as of

from helpers import small_spec, small_batch, cos_rows

pytestmark = pytest.mark.gpu

# Gates of the parity tests: exact plans against the reference CPU path,
# tf32 and 16-bit plans by cosine.
GATES = {3: (1e-4, 0.99999), 2: (1e-4, 0.99999), 4: (2e-3, 0.9999), 0: (None, 0.999),
         1: (None, 0.999)}

CASES = [
    # (model, gemm mode, expected precision plan)
    ("qwen3-2l", "bf16", 0),
    ("qwen3-f32-2l", "f32", 3),
    ("qwen3-f32-2l", "tf32", 4),
    ("qwen3-f32-2l", "16f", 1),
    ("minilm-2l", "f32", 3),
    ("minilm-2l", "tf32", 4),
    ("minilm-2l", "bf16", 0),
    ("bge-bf16-2l", "f32", 2),
]


def _run(key, mode, prec, n, max_len):
    import torch

    s = small_spec(key)
    d = synth.ensure_model(s)
    m = native.B200Model(d, gemm_mode=mode, devices=[0])
    assert m.precision == prec
    seqs = small_batch(key, n=n, max_len=max_len, seed=11)
    offs = np.concatenate([[0], np.cumsum([len(q) for q in seqs])]).astype(np.int32)
    ids = torch.from_numpy(np.concatenate(seqs).astype(np.int32)).cuda()
    ref = torch.empty((len(seqs), s.hidden), dtype=torch.float32, device="cuda")
    m.encode_device(ids.data_ptr(), offs, ref.data_ptr(), sync=True)
    ref = ref.cpu().numpy()
    for call in range(2):
        out = torch.full((len(seqs), s.hidden), float("nan"), dtype=torch.float32, device="cuda")
        rc = m.encode_device_noalloc(ids.data_ptr(), offs, out.data_ptr())
        assert rc == 0, native.last_error()
        out = out.cpu().numpy()
        assert np.array_equal(out, ref), f"call {call}: not bitwise equal to encode_device"
    return m, s, d, seqs, ref


@pytest.mark.parametrize("key,mode,prec", CASES)
def test_noalloc_bitwise_equals_encode_device_and_matches_checker(key, mode, prec):
    m, s, d, seqs, out = _run(key, mode, prec, n=3, max_len=160)
    m.close()
    want = of.OracleModel(d).encode_batch(seqs)
    max_abs, min_cos = GATES[prec]
    assert np.isfinite(out).all()
    if max_abs is not None:
        assert np.abs(out - want).max() <= max_abs
    assert cos_rows(out, want).min() >= min_cos


def test_noalloc_rejects_oversized_request():
    import torch

    m, s, _, _, _ = _run("qwen3-2l", "bf16", 0, n=2, max_len=64)
    T = 4000  # ~24.6 KB of scratch per token for this shape: beyond the 32 MiB arena
    offs = np.array([0, 2000, T], np.int32)
    ids = torch.zeros(T, dtype=torch.int32, device="cuda")
    out = torch.empty((2, s.hidden), dtype=torch.float32, device="cuda")
    assert m.encode_device_noalloc(ids.data_ptr(), offs, out.data_ptr()) == -1
    assert "scratch maximum" in native.last_error()
    # a rejected request leaves the arena usable
    m2, _, _, _, _ = _run("qwen3-2l", "bf16", 0, n=2, max_len=64)
    m2.close()
    m.close()
