"""The no-allocation entry point (ffwd_b200_encode_device_noalloc), called
through the C ABI, against the existing device-resident entry point
(ffwd_b200_encode_device) on the same inputs, on two calls in a row.

It serves callers that cannot allocate device memory while serving (a host
that owns all GPU memory through its own pool, or a latency-sensitive caller
that must not hit cudaMalloc / cudaFree on the request path); its scratch is a
fixed arena reserved in device memory.  This file is collected last so that a
stop-at-first-failure run has already run every other test."""

import numpy as np
import pytest

from ffwd_b200 import native, synth

from helpers import small_spec, small_batch, cos_rows

pytestmark = pytest.mark.gpu

BF16_COS = 0.999
F32_MAXABS = 1e-4
F32_COS = 0.99999


def _run(key, mode, n, max_len, exact):
    import torch

    s = small_spec(key)
    d = synth.ensure_model(s)
    m = native.B200Model(d, gemm_mode=mode, devices=[0])
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
        assert np.isfinite(out).all(), f"call {call}"
        cos = cos_rows(out, ref)
        if exact:
            assert np.abs(out - ref).max() <= F32_MAXABS, f"call {call}"
            assert cos.min() >= F32_COS, f"call {call}"
        else:
            assert cos.min() >= BF16_COS, f"call {call}"
    return m, s


def test_noalloc_matches_encode_device_bf16():
    m, s = _run("qwen3-2l", "bf16", n=4, max_len=300, exact=False)
    m.close()


def test_noalloc_matches_encode_device_exact_mode():
    m, s = _run("minilm-2l", "f32", n=6, max_len=None, exact=True)
    m.close()


def test_noalloc_rejects_oversized_request():
    import torch

    m, s = _run("qwen3-2l", "bf16", n=2, max_len=64, exact=False)
    T = 4000  # ~24.6 KB of scratch per token for this shape: beyond the 32 MiB arena
    offs = np.array([0, 2000, T], np.int32)
    ids = torch.zeros(T, dtype=torch.int32, device="cuda")
    out = torch.empty((2, s.hidden), dtype=torch.float32, device="cuda")
    assert m.encode_device_noalloc(ids.data_ptr(), offs, out.data_ptr()) == -1
    assert "scratch maximum" in native.last_error()
    m.close()
