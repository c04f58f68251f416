"""C-ABI boundary checks that need no GPU: every entry point declared in
include/*.h is exported by the built libraries, the bindings agree with the
headers, and host-side logic (LPT sharding, option parsing) behaves."""

import os
import re

import numpy as np
import pytest

from ffwd_b200 import native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared(header):
    lines = open(os.path.join(ROOT, "include", header)).read().splitlines()
    text = "\n".join(l for l in lines if not l.lstrip().startswith("#"))
    names = re.findall(r"FFWD_B200_API\s+[^;(]*?\b(\w+)\s*\(", text)
    return set(names)


def _exported(path):
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line or " B " in line
            or " D " in line}


def test_core_library_exports_header():
    decl = _declared("ffwd_b200.h")
    assert len(decl) >= 18
    exp = _exported(native.LIB_PATH)
    assert decl <= exp, decl - exp
    assert set(native.ABI) == decl


def test_api_library_exports_reference_api():
    decl = _declared("ffwd_b200_api.h") | _declared("ffwd_b200.h")
    exp = _exported(native.API_LIB_PATH)
    assert decl <= exp, decl - exp
    assert "ffwd_verbose" in exp


def test_library_loads_and_binds():
    L = native.lib()
    A = native.api()
    for name in native.ABI:
        assert getattr(L, name) is not None
    for name in native.API_ABI:
        assert getattr(A, name) is not None


def test_lpt_partition_balances():
    rng = np.random.default_rng(0)
    cost = rng.integers(1, 1000, size=200).astype(np.float64)
    for parts in (1, 2, 4, 8):
        p = native.lpt_partition(cost, parts)
        assert p.min() >= 0 and p.max() < parts
        loads = np.bincount(p, weights=cost, minlength=parts)
        # LPT bound: max load <= mean + max item
        assert loads.max() <= cost.sum() / parts + cost.max()
        assert abs(loads.sum() - cost.sum()) < 1e-6


def test_lpt_partition_errors():
    L = native.lib()
    assert L.ffwd_b200_lpt_partition(None, 3, 2, None) == -1
    assert L.ffwd_b200_lpt_partition(None, 0, 0, None) == -1


def test_gemm_mode_parsing():
    L = native.lib()
    for m in (b"f32", b"tf32", b"bf16", b"16f"):
        assert L.ffwd_b200_set_fast_gemm(m) == 0
    assert L.ffwd_b200_set_fast_gemm(b"fp64") == -1
    assert L.ffwd_b200_set_fast_gemm(b"f32") == 0


def test_api_option_errors_match_reference():
    # backend_cuda.c:45-65 messages
    import ctypes
    A = native.api()
    err = ctypes.create_string_buffer(256)
    o = native.ffwd_options_t(0, 0, 0, b"fp64", None, 0.0)
    assert A.ffwd_init(ctypes.byref(o), err, 256) == -1
    assert err.value.decode() == "--gpu-gemm-mode must be f32, tf32, bf16, or 16f"
    o = native.ffwd_options_t(0, 0, 0, None, b"int8", 0.0)
    assert A.ffwd_init(ctypes.byref(o), err, 256) == -1
    assert err.value.decode() == "--gpu-weight-dtype must be f32, bf16, or f16"
    o = native.ffwd_options_t(0, 0, 0, b"f32", b"f32", 0.0)
    assert A.ffwd_init(ctypes.byref(o), err, 256) == 0
    assert A.ffwd_default_batch_wait_us() == 1000
    assert A.ffwd_scratch_nbytes(None) == 0
    assert A.ffwd_uses_dense_batches(None) == 0


def test_api_math_helpers():
    A = native.api()
    v = np.array([3.0, 4.0], np.float32)
    assert A.ffwd_l2_normalize(v.ctypes.data, 2) == 0
    assert np.allclose(v, [0.6, 0.8])
    z = np.zeros(2, np.float32)
    assert A.ffwd_l2_normalize(z.ctypes.data, 2) == -1
    a = np.array([1.0, 0.0], np.float32)
    b = np.array([1.0, 1.0], np.float32)
    assert abs(A.ffwd_cosine_similarity(a.ctypes.data, b.ctypes.data, 2) - 0.70710677) < 1e-6


def test_load_failure_is_loud(tmp_path):
    L = native.lib()
    assert not L.ffwd_b200_load(str(tmp_path).encode())
    assert "config.json" in native.last_error()


def test_device_entries_reject_offsets_not_starting_at_zero():
    # A nonzero first offset would make the id copy read past the caller's
    # buffer; both device-resident entries refuse it before touching a GPU.
    L = native.lib()
    offs = np.array([3, 10, 20], np.int32)
    assert L.ffwd_b200_encode_device(None, 0, 1, offs.ctypes.data, 2, 1, 1) == -1
    assert "row offsets must start at 0" in native.last_error()
    assert L.ffwd_b200_encode_device_noalloc(None, 0, 1, offs.ctypes.data, 2, 1) == -1
    assert "row offsets must start at 0" in native.last_error()
    offs[0] = -4
    assert L.ffwd_b200_encode_device_noalloc(None, 0, 1, offs.ctypes.data, 2, 1) == -1
    assert "row offsets must start at 0" in native.last_error()


def test_fault_injection_switches():
    L = native.lib()
    assert native.test_inject(native.INJECT_SHARD, 1) == 0
    assert native.test_inject(native.INJECT_ALLOC, 2) == 0
    assert native.test_inject(native.INJECT_NONE) == 0
    assert native.test_inject(99) == -1
    assert L.ffwd_b200_selftest_wait(0, 0) == -1  # limit out of range, no launch
    assert "limit_us" in native.last_error()
    assert native.shard_stats(None) == []
