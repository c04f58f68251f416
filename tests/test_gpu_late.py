"""Late interaction (ColBERT-style MaxSim) on the B200 path, through the C ABI
and the public ffwd_rerank, against the reference's CPU late path (golden
fixtures in tests/golden/late/, made by its ffwd_late_model_encode_tokens /
_encode_docs / ffwd_late_maxsim_batch) and the numpy checker.

Gates: exact (f32 weights, f32 mode) vectors max-abs <= 1e-4, scores <= 1e-4
relative; bf16 decoder (16-bit compute) vectors cosine >= 0.999, scores within
2e-2 absolute (each score sums up to query_n_keep cosines)."""

import glob
import json
import os

import numpy as np
import pytest

from ffwd_b200 import native, synth
from oracle import forward as of

from helpers import small_spec, cos_rows

pytestmark = pytest.mark.gpu

LATE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "late")


def late_fixtures():
    return sorted(os.path.splitext(os.path.basename(p))[0]
                  for p in glob.glob(os.path.join(LATE, "*.npz")))


def load_late(name, model_root):
    z = np.load(os.path.join(LATE, name + ".npz"))
    spec = synth.ModelSpec(**json.loads(str(z["spec"])))
    d = synth.ensure_model(spec, model_root)
    lens, nk = z["doc_lens"], z["n_keep"]
    lo = np.concatenate([[0], np.cumsum(lens)])
    ko = np.concatenate([[0], np.cumsum(nk)])
    docs = [z["doc_ids"][lo[i]:lo[i + 1]] for i in range(len(lens))]
    keeps = [z["keep"][ko[i]:ko[i + 1]] for i in range(len(nk))]
    return spec, d, z, docs, keeps


def check_vecs(out, ref, exact):
    assert out.shape == ref.shape
    assert np.isfinite(out).all()
    if exact:
        assert np.abs(out - ref).max() <= 1e-4
    else:
        assert cos_rows(out, ref).min() >= 0.999


def check_scores(out, ref, exact):
    if exact:
        assert np.abs(out - ref).max() <= 1e-4 * max(1.0, np.abs(ref).max())
    else:
        assert np.abs(out - ref).max() <= 2e-2


@pytest.mark.parametrize("name", late_fixtures())
def test_late_golden(name, model_root):
    spec, d, z, docs, keeps = load_late(name, model_root)
    exact = spec.dtype == "f32"
    m = native.B200Late(d, gemm_mode="f32" if exact else "bf16")
    try:
        assert m.dim == spec.late_dim
        check_vecs(m.encode_tokens(z["query"], True), z["q_vec"], exact)
        check_vecs(m.encode_tokens(z["query"], False), z["q_raw"], exact)
        d_vec, d_off = m.encode_docs(docs, keeps, True)
        assert np.array_equal(d_off, z["d_off"])
        check_vecs(d_vec, z["d_vec"], exact)
        scores = m.rerank(z["query"], int(z["query_n_keep"]), docs, keeps)
        check_scores(scores, z["scores"], exact)
    finally:
        m.close()


def test_public_rerank_matches_abi(model_root):
    spec, d, z, docs, keeps = load_late("qwen3_late_bf16", model_root)
    qk = int(z["query_n_keep"])
    m = native.B200Late(d, gemm_mode="bf16")
    via_abi = m.rerank(z["query"], qk, docs, keeps)
    m.close()
    a = native.FfwdApi(d, gemm_mode="bf16", is_late=True)
    try:
        assert a.token_dim() == spec.late_dim
        assert np.array_equal(a.rerank(z["query"], qk, docs, keeps), via_abi)
    finally:
        a.close()


def test_bert_late_matches_checker(model_root):
    """BERT bases: the reference's CPU late path cannot run them
    (ffwd_model_forward_into is decoder-only), so the numpy checker restating
    the same steps over the BERT forward is the oracle."""
    s = small_spec("minilm-late-2l")
    d = synth.ensure_model(s, model_root)
    rng = np.random.default_rng(5)
    query = np.concatenate([[101], rng.integers(1000, 30000, 14), [102]]).astype(np.int32)
    docs = [np.concatenate([[101], rng.integers(1000, 30000, n), [102]]).astype(np.int32)
            for n in (30, 90, 3)]
    keeps = [np.arange(1, len(x) - 1, dtype=np.int32) for x in docs]
    ref = of.OracleLate(d)
    m = native.B200Late(d, gemm_mode="f32")
    try:
        check_vecs(m.encode_tokens(query, True), ref.encode_tokens(query, True), True)
        dv, do = m.encode_docs(docs, keeps, True)
        rv, ro = ref.encode_docs(docs, keeps, True)
        assert np.array_equal(do, ro)
        check_vecs(dv, rv, True)
        check_scores(m.rerank(query, 10, docs, keeps), ref.rerank(query, 10, docs, keeps), True)
    finally:
        m.close()


def test_late_model_kinds_are_kept_apart(model_root):
    late_dir = synth.ensure_model(small_spec("qwen3-late-f32-1l"), model_root)
    pooled_dir = synth.ensure_model(small_spec("qwen3-2l"), model_root)
    # A 1_Dense head makes the directory a late model only (libffwd/model.c:308-314).
    with pytest.raises(native.FfwdError):
        native.B200Model(late_dir)
    with pytest.raises(native.FfwdError):
        native.B200Late(pooled_dir)


def test_late_invalid_inputs(model_root):
    spec, d, z, docs, keeps = load_late("qwen3_late_f32", model_root)
    m = native.B200Late(d, gemm_mode="f32")
    try:
        q = z["query"]
        with pytest.raises(native.FfwdError):  # kept index outside the document
            m.encode_docs(docs, [keeps[0], np.array([len(docs[1])], np.int32), keeps[2]])
        with pytest.raises(native.FfwdError):  # nothing kept
            m.encode_docs(docs, [keeps[0], np.array([], np.int32), keeps[2]])
        with pytest.raises(native.FfwdError):  # query_n_keep beyond the query
            m.rerank(q, len(q) + 1, docs, keeps)
        with pytest.raises(native.FfwdError):  # token id outside the vocabulary
            m.encode_tokens(np.array([0, spec.vocab], np.int32))
        # the context stays usable after rejected calls
        check_vecs(m.encode_tokens(q, True), z["q_vec"], True)
    finally:
        m.close()
