"""Host-side helpers of bench.py that need no GPU: the parity summary the
bench line carries and the CPU description of its baseline."""

import numpy as np

import bench


def test_parity_rows_gate():
    rng = np.random.default_rng(0)
    a = rng.standard_normal((3, 64)).astype(np.float32)
    p = bench.parity_rows(a, a)
    assert p["ok"] and p["rows"] == 3 and p["max_abs"] == 0.0
    assert abs(p["min_cos"] - 1.0) < 1e-12
    b = a.copy()
    b[1] = -b[1]
    p = bench.parity_rows(a, b)
    assert not p["ok"] and p["min_cos"] < 0
    b = a.copy()
    b[0, 0] = np.nan
    assert not bench.parity_rows(b, a)["ok"]


def test_cpu_info():
    info = bench.cpu_info()
    assert info["nproc"] >= 1 and 1 <= info["physical_cores"] <= info["nproc"]


def test_flops_per_token_of_the_bench_model():
    # Qwen3-0.6B: 880.8 MFLOP/token in the projections (2 x MAC, 28 layers)
    spec, seqs = bench.workload(0)
    total, lin, attn = bench.flops_per_token(spec, seqs)
    assert abs(lin / 1e6 - 880.8) < 0.5
    assert attn > 0 and abs(total - lin - attn) < 1


def test_config_sweep_covers_every_baseline_config():
    """`bench.py --configs` times every BASELINE configuration (the 8B shape at
    reduced depth, with the same per-layer shapes) in the GEMM mode the
    configuration names."""
    from ffwd_b200 import synth

    names = {name for name, _, _, _ in bench.SWEEP}
    assert names == set(synth.CONFIGS)
    modes = {name: mode for name, mode, _, _ in bench.SWEEP}
    assert modes["minilm"] == "f32" and modes["bge-base"] == "f32"
    assert all(modes[n] == "bf16" for n in ("bge-base-bf16", "xlmr-large", "qwen3-0.6b", "qwen3-8b"))
    for name, _, _, over in bench.SWEEP:
        spec = synth.spec(name, **over) if over else synth.CONFIGS[name]
        base = synth.CONFIGS[name]
        assert (spec.hidden, spec.n_heads, spec.n_kv_heads, spec.head_dim, spec.intermediate) == \
            (base.hidden, base.n_heads, base.n_kv_heads, base.head_dim, base.intermediate)
