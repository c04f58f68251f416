"""Generate the golden fixtures of this directory from the reference itself.

Each fixture holds a seeded synthetic model spec (the model is regenerated
bit-identically by ``ffwd_b200.synth.write_model``), a packed token batch and
the embeddings the reference's own CPU path (``oracle/_ref/libffwd_ref.so``,
built from the unmodified reference sources by ``oracle/Makefile``) returns
for it through ``ffwd_model_encode_batch``.  ``late/*.npz`` hold late-interaction
cases: a query, candidate documents and kept-token lists, with the reference's
``ffwd_late_model_encode_tokens`` / ``_encode_docs`` vectors and
``ffwd_late_maxsim_batch`` scores (the steps of ``ffwd_rerank``).
``spans/*.npz`` hold contextual-span cases: documents, (start, n_tokens) spans
and the reference's ``ffwd_model_encode_spans_batch`` rows.

    python tests/golden/make_golden.py [case ...]   (needs oracle/_ref: `make -C oracle`;
                                                     no names: every case;
                                                     "spans": the spans cases only)
"""

import dataclasses
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(HERE))

from ffwd_b200 import synth  # noqa: E402
from oracle.ref import RefLate, RefModel  # noqa: E402
from helpers import small_spec, small_batch  # noqa: E402

CASES = {
    # name: (small spec key, batch builder)
    "minilm_f32": ("minilm-2l", lambda: small_batch("minilm-2l", n=6)),
    "bge_bf16_cls": ("bge-bf16-2l", lambda: small_batch("bge-bf16-2l", n=5, max_len=160)),
    "xlmr_mean": ("xlmr-2l", lambda: small_batch("xlmr-2l", n=3, max_len=200)),
    "qwen3_last": ("qwen3-2l", lambda: small_batch("qwen3-2l", n=4, max_len=300)),
    "qwen3_edges": ("qwen3-2l", lambda: [np.arange(1, L + 1, dtype=np.int32) * 7 % 8000
                                         for L in (1, 2, 127, 128, 129, 257)]),
    "qwen2_mean": ("qwen2-1l", lambda: small_batch("qwen2-1l", n=3, max_len=150)),
    "bert_tanh_cls": ("bert-tanh-1l", lambda: small_batch("bert-tanh-1l", n=4)),
    "qwen3_bidir": ("qwen3-bidir-1l", lambda: small_batch("qwen3-bidir-1l", n=3, max_len=140)),
    "qwen3_f16": ("qwen3-f16-1l", lambda: small_batch("qwen3-f16-1l", n=3, max_len=200)),
    "minilm_f16": ("minilm-f16-2l", lambda: small_batch("minilm-f16-2l", n=4)),
}


LATE_CASES = {
    # name: (small spec key, query length, query_n_keep, doc lengths, seed)
    "qwen3_late_bf16": ("qwen3-late-2l", 24, 20, (60, 131, 9, 257), 3),
    "qwen3_late_f32": ("qwen3-late-f32-1l", 11, 11, (5, 40, 1), 4),
}


SPANS_CASES = {
    # name: (small spec key, documents builder, spans per document).  Decoder
    # models only: the reference CPU spans path runs the decoder forward
    # (forward_packed_inplace, forward.c:572) and refuses BERT-family models.
    "qwen3_spans": ("qwen3-2l", lambda: small_batch("qwen3-2l", n=2, max_len=180, seed=4),
                    lambda docs: [[(0, 10), (5, 50), (len(docs[0]) - 1, 1)],
                                  [(0, len(docs[1])), (3, 7)]]),
    "qwen3_f32_spans": ("qwen3-f32-2l",
                        lambda: small_batch("qwen3-f32-2l", n=3, max_len=150, seed=8),
                        lambda docs: [[(0, len(docs[0]))], [(1, 1), (0, 20), (20, 40)],
                                      [(len(docs[2]) - 5, 5)]]),
}


def main_spans(root):
    os.makedirs(os.path.join(HERE, "spans"), exist_ok=True)
    for name, (key, mk_docs, mk_spans) in SPANS_CASES.items():
        s = small_spec(key)
        d = synth.ensure_model(s, root)
        docs = [np.asarray(q, np.int32) for q in mk_docs()]
        spans = mk_spans(docs)
        ref = RefModel(d, threads=os.cpu_count() or 1)
        out = ref.encode_spans(docs, spans)
        ref.close()
        np.savez_compressed(
            os.path.join(HERE, "spans", f"{name}.npz"),
            spec=json.dumps(dataclasses.asdict(s)),
            ids=np.concatenate(docs), lens=np.array([len(q) for q in docs], np.int32),
            n_spans=np.array([len(sp) for sp in spans], np.int32),
            span_start=np.array([a for sp in spans for a, _ in sp], np.int32),
            span_len=np.array([n for sp in spans for _, n in sp], np.int32),
            expected=out.astype(np.float32))
        print(name, out.shape)


def late_case(spec, q_len, q_keep, doc_lens, seed):
    rng = np.random.default_rng(seed)
    hi = min(spec.vocab - 1, 151642)
    query = rng.integers(0, hi, q_len).astype(np.int32)
    docs = [rng.integers(0, hi, n).astype(np.int32) for n in doc_lens]
    keeps = [np.sort(rng.choice(n, size=max(1, (3 * n) // 4), replace=False)).astype(np.int32)
             for n in doc_lens]
    return query, q_keep, docs, keeps


def main_late(root):
    os.makedirs(os.path.join(HERE, "late"), exist_ok=True)
    for name, (key, q_len, q_keep, doc_lens, seed) in LATE_CASES.items():
        s = small_spec(key)
        d = synth.ensure_model(s, root)
        query, qk, docs, keeps = late_case(s, q_len, q_keep, doc_lens, seed)
        ref = RefLate(d, threads=os.cpu_count() or 1)
        q_vec = ref.encode_tokens(query, True)
        q_raw = ref.encode_tokens(query, False)
        d_vec, d_off = ref.encode_docs(docs, keeps, True)
        scores = ref.maxsim_batch(q_vec[:qk], d_vec, d_off)
        ref.close()
        np.savez_compressed(
            os.path.join(HERE, "late", f"{name}.npz"),
            spec=json.dumps(dataclasses.asdict(s)), query=query, query_n_keep=np.int32(qk),
            doc_ids=np.concatenate(docs), doc_lens=np.array(doc_lens, np.int32),
            keep=np.concatenate(keeps), n_keep=np.array([len(k) for k in keeps], np.int32),
            q_vec=q_vec, q_raw=q_raw, d_vec=d_vec, d_off=d_off, scores=scores)
        print(name, q_vec.shape, d_vec.shape, scores)


def main(only=()):
    root = tempfile.mkdtemp(prefix="ffwd_golden_")
    if only == ("spans",):
        main_spans(root)
        return
    for name, (key, mk) in CASES.items():
        if only and name not in only:
            continue
        s = small_spec(key)
        d = synth.ensure_model(s, root)
        seqs = [np.asarray(q, np.int32) for q in mk()]
        ref = RefModel(d, threads=os.cpu_count() or 1)
        out = ref.encode_batch(seqs)
        ref.close()
        np.savez_compressed(
            os.path.join(HERE, f"{name}.npz"),
            spec=json.dumps(dataclasses.asdict(s)),
            ids=np.concatenate(seqs).astype(np.int32),
            lens=np.array([len(q) for q in seqs], np.int32),
            expected=out.astype(np.float32),
        )
        print(name, out.shape)
    if not only:
        main_late(root)
        main_spans(root)


if __name__ == "__main__":
    main(tuple(sys.argv[1:]))
