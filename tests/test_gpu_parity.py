"""End-to-end parity of the B200 forward (through the C ABI) against the
reference's CPU path: the golden fixtures it produced, and the CPU checker on
further seeded batches.  Gates: f32 mode max-abs <= 1e-4
and cosine >= 0.99999 per row; bf16 mode cosine >= 0.999 per row."""

import ctypes

import numpy as np
import pytest

from ffwd_b200 import native, synth
from oracle import forward as of

from golden_util import fixtures, load, span_fixtures, load_spans
from helpers import small_spec, small_batch, cos_rows

pytestmark = pytest.mark.gpu

F32_MAXABS = 1e-4
F32_COS = 0.99999
BF16_COS = 0.999

_models = {}


def model(d, gemm_mode, weight_dtype=None):
    key = (d, gemm_mode, weight_dtype)
    if key not in _models:
        _models[key] = native.B200Model(d, gemm_mode=gemm_mode, weight_dtype=weight_dtype)
    return _models[key]


def check(out, ref, exact):
    cos = cos_rows(out, ref)
    if exact:
        err = np.abs(out - ref).max()
        assert err <= F32_MAXABS, f"max-abs {err}"
        assert cos.min() >= F32_COS, f"cos {cos.min()}"
    else:
        assert cos.min() >= BF16_COS, f"cos {cos.min()}"
    assert np.isfinite(out).all()


@pytest.mark.parametrize("name", fixtures())
@pytest.mark.parametrize("mode", ["f32", "bf16"])
def test_golden(name, mode, model_root):
    spec, d, seqs, expected = load(name, model_root)
    m = model(d, mode)
    out = m.encode_batch(seqs)
    exact = m.precision >= 2
    # Decoders with bf16 weights run 16-bit regardless of the GEMM mode
    # (libffwd/cuda.cu:5010-5019); everything else follows the mode.
    if spec.family in ("qwen3", "qwen2") and spec.dtype == "bf16":
        assert m.precision == 0
    elif mode == "f32":
        assert m.precision in (2, 3)
    check(out, expected, exact)


@pytest.mark.parametrize("key", ["qwen3-f32-2l", "minilm-2l", "bge-2l"])
def test_exact_mode_longer_batches(key, model_root):
    s = small_spec(key)
    d = synth.ensure_model(s, model_root)
    seqs = small_batch(key, n=5, max_len=260, seed=3)
    ref = of.OracleModel(d).encode_batch(seqs)
    m = model(d, "f32")
    assert m.precision == 3
    check(m.encode_batch(seqs), ref, True)


def test_qwen_long_and_ragged(model_root):
    s = small_spec("qwen3-2l")
    d = synth.ensure_model(s, model_root)
    rng = np.random.default_rng(5)
    lens = [1, 3, 64, 127, 128, 129, 255, 256, 300, 700]
    seqs = [rng.integers(0, s.vocab, size=L).astype(np.int32) for L in lens]
    ref = of.OracleModel(d).encode_batch(seqs)
    out = model(d, "bf16").encode_batch(seqs)
    check(out, ref, False)


def test_packed_equals_singleton_bitwise(model_root):
    s = small_spec("qwen3-2l")
    d = synth.ensure_model(s, model_root)
    m = model(d, "bf16")
    seqs = small_batch("qwen3-2l", n=4, max_len=200, seed=9)
    packed = m.encode_batch(seqs)
    single = np.stack([m.encode_into(q) for q in seqs])
    assert np.array_equal(packed, single)


def test_deterministic_repeats(model_root):
    s = small_spec("bge-bf16-2l")
    d = synth.ensure_model(s, model_root)
    m = model(d, "bf16")
    seqs = small_batch("bge-bf16-2l", n=8, max_len=300, seed=2)
    a = m.encode_batch(seqs)
    b = m.encode_batch(seqs)
    c = m.encode_batch(seqs)
    assert np.array_equal(a, b) and np.array_equal(b, c)


def test_invalid_inputs_rejected(model_root):
    s = small_spec("minilm-2l")
    d = synth.ensure_model(s, model_root)
    m = model(d, "f32")
    rc, _ = m.try_encode_batch([np.array([101, s.vocab, 102], np.int32)])
    assert rc == -1 and "invalid token id" in native.last_error()
    rc, _ = m.try_encode_batch([np.array([101, -1, 102], np.int32)])
    assert rc == -1
    rc, _ = m.try_encode_batch([np.zeros(0, np.int32)])
    assert rc == -1
    rc, _ = m.try_encode_batch([np.full(513, 1000, np.int32)])
    assert rc == -1 and "max_position_embeddings" in native.last_error()
    # the context stays usable after a rejected call
    seqs = small_batch("minilm-2l", n=2)
    ref = of.OracleModel(d).encode_batch(seqs)
    check(m.encode_batch(seqs), ref, True)


def test_xlmr_max_length_512(model_root):
    # position offset 2: 512 tokens fit max_position_embeddings 514 exactly
    s = small_spec("xlmr-2l")
    d = synth.ensure_model(s, model_root)
    seqs = synth.token_batch("xlmr-large", batch=2, vocab=s.vocab)
    ref = of.OracleModel(d).encode_batch(seqs)
    check(model(d, "bf16").encode_batch(seqs), ref, False)
    rc, _ = model(d, "bf16").try_encode_batch([np.full(513, 5, np.int32)])
    assert rc == -1


@pytest.mark.parametrize("name", span_fixtures())
@pytest.mark.parametrize("mode", ["f32", "bf16"])
def test_spans_golden(name, mode, model_root):
    """ffwd_b200_encode_spans_batch against the reference's own
    ffwd_model_encode_spans_batch (forward.c:528-589) rows.  Span rows are
    unnormalised means (the final RMSNorm applied, no L2), compared at the same
    gates as pooled rows."""
    spec, d, docs, spans, expected = load_spans(name, model_root)
    m = model(d, mode)
    out = m.encode_spans_batch(docs, spans)
    check(out, expected, m.precision >= 2)


@pytest.mark.parametrize("key", ["minilm-2l", "bge-bf16-2l"])
@pytest.mark.parametrize("mode", ["f32", "bf16"])
def test_bert_spans_match_checker(key, mode, model_root):
    """BERT-family spans: the reference's CPU spans path runs only the decoder
    forward, so these rows are checked against the numpy restatement (the BERT
    forward, then forward.c:492-526's span means)."""
    s = small_spec(key)
    d = synth.ensure_model(s, model_root)
    docs = small_batch(key, n=3, max_len=200, seed=6)
    spans = [[(1, len(docs[0]) - 2)], [(0, 1), (2, 9)],
             [(0, len(docs[2])), (4, 4), (len(docs[2]) - 1, 1)]]
    ref = of.OracleModel(d).encode_spans_batch(docs, spans)
    m = model(d, mode)
    check(m.encode_spans_batch(docs, spans), ref, m.precision >= 2)


def test_max_tokens_chunking_matches(model_root):
    s = small_spec("bge-bf16-2l")
    d = synth.ensure_model(s, model_root)
    seqs = small_batch("bge-bf16-2l", n=12, max_len=200, seed=6)
    whole = model(d, "bf16").encode_batch(seqs)
    native.lib().ffwd_b200_set_max_tokens(300)
    try:
        chunked = native.B200Model(d, gemm_mode="bf16").encode_batch(seqs)
    finally:
        native.lib().ffwd_b200_set_max_tokens(262144)
    # Sequences longer than one query tile have their own attention items, so
    # their rows do not depend on the rest of the forward; shorter ones share
    # items with their neighbours (windows), which a different chunking
    # regroups: equal to rounding.
    lens = np.array([len(q) for q in seqs])
    assert (lens > 128).any() and (lens <= 128).any()
    assert np.array_equal(whole[lens > 128], chunked[lens > 128])
    assert cos_rows(whole, chunked).min() >= 0.99999


def test_public_api_matches_abi(model_root):
    s = small_spec("bge-bf16-2l")
    d = synth.ensure_model(s, model_root)
    seqs = small_batch("bge-bf16-2l", n=3)
    a = native.FfwdApi(d, gemm_mode="bf16")
    out = a.encode_batch(seqs)
    a.close()
    assert np.array_equal(out, model(d, "bf16").encode_batch(seqs))


def test_deep_long_sequences_rescale_path(model_root):
    # Deeper random-init decoders grow the attention scores across key tiles,
    # which drives the online-softmax rescale of O in TMEM (lanes of one warp
    # disagree on whether to rescale).
    s = synth.spec("qwen3-0.6b", n_layers=6, vocab=4096)
    d = synth.ensure_model(s, model_root)
    rng = np.random.default_rng(21)
    lens = [2049, 1500, 900, 129, 33]
    seqs = [rng.integers(0, s.vocab, size=L).astype(np.int32) for L in lens]
    ref = of.OracleModel(d).encode_batch(seqs)
    check(model(d, "bf16").encode_batch(seqs), ref, False)


def test_multi_device_sharding_matches_single(model_root):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    s = small_spec("qwen3-2l")
    d = synth.ensure_model(s, model_root)
    seqs = small_batch("qwen3-2l", n=9, max_len=400, seed=13)
    single = native.B200Model(d, gemm_mode="bf16", devices=[0]).encode_batch(seqs)
    n = torch.cuda.device_count()
    multi = native.B200Model(d, gemm_mode="bf16", devices=list(range(n))).encode_batch(seqs)
    native.lib().ffwd_b200_set_devices((ctypes.c_int * 1)(0), 1)
    # Every sequence is computed identically on whichever device gets it.
    assert np.array_equal(single, multi)


@pytest.mark.parametrize("key,mode", [("qwen3-2l", "bf16"), ("minilm-2l", "f32")])
def test_output_encodings(key, mode, model_root):
    """ffwd_b200_encode_batch_as: the server's wire forms (tools/server/encode.c)
    made on the device from the same pooled embeddings."""
    s = small_spec(key)
    d = synth.ensure_model(s, model_root)
    m = model(d, mode)
    seqs = small_batch(key, n=5, max_len=200)
    H = m.hidden
    full = m.encode_batch(seqs)
    assert np.array_equal(m.encode_batch_as(seqs, H, False, "f32"), full)
    q = m.encode_batch_as(seqs, H, False, "int8").astype(np.int32)
    diff = np.abs(q - of.quantize_int8_tanh(full).astype(np.int32))
    assert diff.max() <= 1 and (diff != 0).mean() <= 1e-3  # tanhf ulp at rounding ties only
    assert np.array_equal(m.encode_batch_as(seqs, H, False, "binary"), of.binary_bits(full))
    dims = H // 4
    t = m.encode_batch_as(seqs, dims, True, "f32")
    assert np.abs(t - of.truncate_renormalize(full, dims)).max() <= 1e-6
    assert np.array_equal(m.encode_batch_as(seqs, dims, True, "binary"),
                          of.binary_bits(full[:, :dims]))
    assert np.array_equal(m.encode_batch_as(seqs, dims, False, "f32"), full[:, :dims])
    for bad in ((0, "f32"), (H + 1, "f32"), (12, "binary")):
        with pytest.raises(native.FfwdError):
            m.encode_batch_as(seqs, bad[0], True, bad[1])


def test_pipelined_forwards_errors_and_encodings(model_root):
    """Several forwards per call (tiny token budget): outputs in input order for
    every output form, an invalid id in a later forward fails the call, and the
    context stays usable."""
    s = small_spec("qwen3-2l")
    d = synth.ensure_model(s, model_root)
    seqs = small_batch("qwen3-2l", n=9, max_len=150, seed=7)
    whole = model(d, "bf16").encode_batch(seqs)
    native.lib().ffwd_b200_set_max_tokens(200)
    try:
        m = native.B200Model(d, gemm_mode="bf16")
        assert np.array_equal(m.encode_batch(seqs), whole)
        assert np.array_equal(m.encode_batch_as(seqs, m.hidden, False, "binary"),
                              of.binary_bits(whole))
        bad = [q.copy() for q in seqs]
        bad[-1][3] = s.vocab  # invalid id in the last forward
        with pytest.raises(native.FfwdError):
            m.encode_batch(bad)
        assert np.array_equal(m.encode_batch(seqs), whole)
        m.close()
    finally:
        native.lib().ffwd_b200_set_max_tokens(262144)


def test_qwen3_8b_shape_long_documents(model_root):
    """BASELINE config 5 shapes (hidden 4096, 32 / 8 heads x 128, SwiGLU 12288,
    8192-token documents, last-token pooling, Matryoshka truncation to 1024 then
    L2), one layer and a small vocabulary so the checker runs in seconds."""
    s = synth.spec("qwen3-8b", n_layers=1, vocab=4096)
    d = synth.ensure_model(s, model_root)
    rng = np.random.default_rng(31)
    seqs = [rng.integers(0, s.vocab - 1, size=L).astype(np.int32) for L in (8192, 1500)]
    for q in seqs:
        q[-1] = s.vocab - 1
    ref = of.OracleModel(d).encode_batch(seqs)
    m = model(d, "bf16")
    check(m.encode_batch(seqs), ref, False)
    trunc = m.encode_batch_as(seqs, 1024, True, "f32")
    check(trunc, of.truncate_renormalize(ref, 1024), False)


def test_dependent_launch_off_matches(model_root, tmp_path):
    """Programmatic dependent launch changes only when kernels start, not what
    they compute: the same batches with FFWD_B200_PDL=0 (ordinary launches, in
    a child process, since the switch is read once per process) give the same
    bits, for a decoder and an encoder."""
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    cases = [("qwen3-2l", "bf16", 300, 17), ("bge-bf16-2l", "bf16", 200, 5), ("minilm-2l", "f32", 128, 3)]
    want = []
    for key, mode, max_len, seed in cases:
        d = synth.ensure_model(small_spec(key), model_root)
        want.append(model(d, mode).encode_batch(small_batch(key, n=6, max_len=max_len, seed=seed)))
    code = (
        "import sys, numpy as np\n"
        f"sys.path[:0] = [{root!r}, {os.path.join(root, 'tests')!r}]\n"
        "from ffwd_b200 import native, synth\n"
        "from helpers import small_spec, small_batch\n"
        f"for i, (key, mode, max_len, seed) in enumerate({cases!r}):\n"
        f"    d = synth.ensure_model(small_spec(key), {model_root!r})\n"
        "    m = native.B200Model(d, gemm_mode=mode)\n"
        "    out = m.encode_batch(small_batch(key, n=6, max_len=max_len, seed=seed))\n"
        f"    np.save({str(tmp_path)!r} + f'/out{{i}}.npy', out)\n"
    )
    subprocess.run([sys.executable, "-c", code], env={**os.environ, "FFWD_B200_PDL": "0"},
                   check=True, cwd=root, timeout=600)
    for i, w in enumerate(want):
        assert np.array_equal(w, np.load(tmp_path / f"out{i}.npy"))
