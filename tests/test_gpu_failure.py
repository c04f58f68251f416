"""Failure detection on the host side of the path, with no GPU fault.

* A per-device shard worker forced to fail (ffwd_b200_test_inject): the
  encode call returns -1 with the shard's message, the failing shard writes no
  output row, and the context stays usable.  Two device entries on one GPU
  (devices=[0, 0]) run the sharder's thread-per-device path on a 1-GPU lease.
* A workspace allocation that fails (a fake out-of-memory error): -1 with the
  CUDA error text, then a normal call succeeds and matches.
* The kernels' bounded waits: a self-test kernel waits on an mbarrier that
  nothing arrives at, with a 2 ms limit; the call returns -1 with "device wait
  timed out" and the GPU stays usable.

Reference error contract: every CUDA call checked and -1 returned
(libffwd/cuda.cu:151-167, launch_check 2710-2717)."""

import ctypes

import numpy as np
import pytest

from ffwd_b200 import native, synth

from helpers import small_spec, small_batch

pytestmark = pytest.mark.gpu


@pytest.fixture
def reset_devices():
    yield
    native.test_inject(native.INJECT_NONE)
    native.lib().ffwd_b200_set_devices((ctypes.c_int * 1)(0), 1)


def test_shard_failure_on_one_device_entry(reset_devices, model_root):
    s = small_spec("qwen3-2l")
    d = synth.ensure_model(s, model_root)
    seqs = small_batch("qwen3-2l", n=9, max_len=400, seed=13)
    single = native.B200Model(d, gemm_mode="bf16", devices=[0])
    want = single.encode_batch(seqs)
    single.close()
    m = native.B200Model(d, gemm_mode="bf16", devices=[0, 0])
    ins, keep = native._pack_inputs(seqs)
    L = native.lib()

    # Which entry gets which sequence (LPT over the same costs the sharder uses).
    assert L.ffwd_b200_encode_batch(m.h, ins, len(seqs), np.zeros((9, s.hidden), np.float32)
                                    .ctypes.data) == 0
    stats = native.shard_stats(m.h)
    assert len(stats) == 2 and sum(st[0] for st in stats) == 9
    assert all(st[0] > 0 for st in stats)

    sentinel = np.float32(-7.0)
    out = np.full((9, s.hidden), sentinel, np.float32)
    assert native.test_inject(native.INJECT_SHARD, 1) == 0
    rc = L.ffwd_b200_encode_batch(m.h, ins, len(seqs), out.ctypes.data)
    assert rc == -1
    assert "injected failure of the shard on device entry 1" in native.last_error()
    untouched = np.all(out == sentinel, axis=1)
    written = ~untouched
    # entry 1's rows are never written; entry 0's rows are complete and correct
    assert untouched.sum() == stats[1][0]
    assert written.sum() == stats[0][0]
    assert np.array_equal(out[written], want[written])

    # the injection is one-shot and the context stays usable
    assert np.array_equal(m.encode_batch(seqs), want)
    m.close()


def test_multi_entry_same_gpu_matches_single(reset_devices, model_root):
    """The sharder's LPT split, one host thread per entry and the row placement,
    exercised with two entries on GPU 0: bitwise equal to one entry."""
    s = small_spec("qwen3-2l")
    d = synth.ensure_model(s, model_root)
    seqs = small_batch("qwen3-2l", n=9, max_len=400, seed=13)
    a = native.B200Model(d, gemm_mode="bf16", devices=[0])
    want = a.encode_batch(seqs)
    a.close()
    b = native.B200Model(d, gemm_mode="bf16", devices=[0, 0])
    assert np.array_equal(b.encode_batch(seqs), want)
    b.close()


def test_workspace_allocation_failure(reset_devices, model_root):
    s = small_spec("minilm-2l")
    d = synth.ensure_model(s, model_root)
    seqs = small_batch("minilm-2l", n=4)
    big = small_batch("minilm-2l", n=32, seed=5)
    want_big = None
    for n_fail in (1, 3):
        m = native.B200Model(d, gemm_mode="f32", devices=[0])
        want = m.encode_batch(seqs)
        # The larger batch makes the workspace grow; its first allocations fail.
        assert native.test_inject(native.INJECT_ALLOC, n_fail) == 0
        rc, _ = m.try_encode_batch(big)
        assert rc == -1
        assert "out of memory" in native.last_error()
        native.test_inject(native.INJECT_NONE)
        # the next call allocates again and computes the right thing
        got_big = m.encode_batch(big)
        if want_big is None:
            want_big = got_big
        assert np.array_equal(got_big, want_big)
        assert np.array_equal(m.encode_batch(seqs), want)
        m.close()


def test_bounded_wait_expires_and_gpu_stays_usable(model_root):
    L = native.lib()
    assert L.ffwd_b200_selftest_wait(0, 2000) == -1
    assert "device wait timed out" in native.last_error()
    s = small_spec("minilm-2l")
    d = synth.ensure_model(s, model_root)
    m = native.B200Model(d, gemm_mode="f32", devices=[0])
    out = m.encode_batch(small_batch("minilm-2l", n=2))
    assert np.isfinite(out).all()
    m.close()
