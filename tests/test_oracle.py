"""The CPU checker against the reference: golden fixtures produced by the
reference's own CPU path, the compiled reference itself (when built), and the
reference's kernel known-answer values (tests/test_kernels.c:96-127)."""

import json
import os

import numpy as np
import pytest

from oracle import forward as of
from oracle import ref as oref

from golden_util import fixtures, load, span_fixtures, load_spans
from helpers import small_spec, small_batch, cos_rows
from ffwd_b200 import synth


@pytest.mark.parametrize("name", fixtures())
def test_oracle_matches_reference_golden(name, model_root):
    spec, d, seqs, expected = load(name, model_root)
    out = of.OracleModel(d).encode_batch(seqs)
    assert out.shape == expected.shape
    assert np.abs(out - expected).max() <= 2e-6, name
    assert cos_rows(out, expected).min() >= 0.999999


@pytest.mark.skipif(not oref.available(), reason="oracle/_ref not built")
@pytest.mark.parametrize("name", fixtures())
def test_compiled_reference_reproduces_golden(name, model_root):
    spec, d, seqs, expected = load(name, model_root)
    r = oref.RefModel(d, threads=2)
    out = r.encode_batch(seqs)
    r.close()
    assert np.abs(out - expected).max() <= 1e-6


@pytest.mark.parametrize("name", span_fixtures())
def test_oracle_spans_match_reference_golden(name, model_root):
    # ffwd_model_encode_spans_batch (forward.c:528-589) rows.  Span rows are
    # unnormalised means of final-norm outputs (|x| ~ 1, not the ~0.03 of an L2
    # row), so the f32 summation-order gate is 1e-5 here.
    spec, d, docs, spans, expected = load_spans(name, model_root)
    out = of.OracleModel(d).encode_spans_batch(docs, spans)
    assert out.shape == expected.shape
    assert np.abs(out - expected).max() <= 1e-5, name
    assert cos_rows(out, expected).min() >= 0.999999


@pytest.mark.skipif(not oref.available(), reason="oracle/_ref not built")
@pytest.mark.parametrize("name", span_fixtures())
def test_compiled_reference_reproduces_spans_golden(name, model_root):
    spec, d, docs, spans, expected = load_spans(name, model_root)
    r = oref.RefModel(d, threads=2)
    out = r.encode_spans(docs, spans)
    r.close()
    assert np.abs(out - expected).max() <= 1e-6


def test_gelu_known_values():
    # tests/test_kernels.c:106-126
    x = np.array([1.0], np.float32)
    assert abs(float(of.gelu(x, "erf")[0]) - 0.841344746) < 1e-6
    assert abs(float(of.gelu(x, "tanh")[0]) - 0.841191991) < 1e-6


def test_norms_known_values():
    x = np.array([[1.0, 2.0, 3.0, 4.0]], np.float32)
    w = np.ones(4, np.float32)
    r = of.rms_norm(x, w, np.float32(1e-6))
    assert np.allclose(r, x / np.sqrt(7.5 + 1e-6), atol=1e-6)
    ln = of.layer_norm(x, w, np.zeros(4, np.float32), np.float32(1e-12))
    assert np.allclose(ln, (x - 2.5) / np.sqrt(1.25), atol=1e-6)


def test_packed_equals_singleton_oracle(model_root):
    # test_qwen3.c:39-81: packed batch == per-sequence encode (<= 1e-5)
    s = small_spec("qwen3-2l")
    d = synth.ensure_model(s, model_root)
    m = of.OracleModel(d)
    seqs = small_batch("qwen3-2l", n=3, max_len=90)
    packed = m.encode_batch(seqs)
    single = np.stack([m.encode_batch([q])[0] for q in seqs])
    assert np.abs(packed - single).max() <= 1e-5
    assert np.allclose(np.linalg.norm(packed, axis=1), 1.0, atol=1e-5)


def test_oracle_rejects_bad_inputs(model_root):
    s = small_spec("minilm-2l")
    d = synth.ensure_model(s, model_root)
    m = of.OracleModel(d)
    with pytest.raises(ValueError):
        m.encode_batch([np.array([101, s.vocab + 5, 102], np.int32)])
    with pytest.raises(ValueError):
        m.encode_batch([np.zeros(0, np.int32)])
    with pytest.raises(ValueError):
        m.encode_batch([np.full(600, 1000, np.int32)])


LATE_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "late")


@pytest.mark.parametrize("name", sorted(os.path.splitext(f)[0] for f in os.listdir(LATE_DIR)
                                        if f.endswith(".npz")))
def test_late_oracle_matches_reference_golden(name, model_root):
    """The numpy late-interaction restatement against the reference's own CPU
    late path (ffwd_late_model_encode_tokens / _encode_docs / maxsim_batch)."""
    z = np.load(os.path.join(LATE_DIR, name + ".npz"))
    spec = synth.ModelSpec(**json.loads(str(z["spec"])))
    d = synth.ensure_model(spec, model_root)
    lo = np.concatenate([[0], np.cumsum(z["doc_lens"])])
    ko = np.concatenate([[0], np.cumsum(z["n_keep"])])
    docs = [z["doc_ids"][lo[i]:lo[i + 1]] for i in range(len(lo) - 1)]
    keeps = [z["keep"][ko[i]:ko[i + 1]] for i in range(len(ko) - 1)]
    o = of.OracleLate(d)
    assert np.abs(o.encode_tokens(z["query"], True) - z["q_vec"]).max() <= 1e-5
    assert np.abs(o.encode_tokens(z["query"], False) - z["q_raw"]).max() <= 1e-4
    dv, do = o.encode_docs(docs, keeps, True)
    assert np.array_equal(do, z["d_off"])
    assert np.abs(dv - z["d_vec"]).max() <= 1e-5
    sc = o.maxsim_batch(z["q_vec"][:int(z["query_n_keep"])], z["d_vec"], z["d_off"])
    assert np.abs(sc - z["scores"]).max() <= 1e-4


def test_output_encodings_known_values():
    """tools/server/encode.c:20-51 wire forms."""
    x = np.array([0.0, 10.0, -10.0, 0.5, -0.5, 1e-9, -1e-9], np.float32)
    q = of.quantize_int8_tanh(x)
    assert q.tolist() == [0, 127, -127, 59, -59, 0, 0]
    bits = of.binary_bits(np.array([1, -1, 0, -0.5, 2, 3, -4, 5, -1, 1, -1, -1, -1, -1, -1, -1],
                                   np.float32))
    assert bits.tolist() == [0b10110101, 0b00000010]
    e = of.truncate_renormalize(np.array([[3.0, 4.0, 12.0]], np.float32), 2)
    assert np.allclose(e, [[0.6, 0.8]])
