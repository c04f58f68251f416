"""Parity at the benchmark configurations' real depth and vocabulary.

Every case runs the B200 forward through the C ABI and the reference's own CPU
path (oracle/_ref, ``ffwd_model_encode_batch``, libffwd/forward.c:628-652) on
the same seeded model directory and token ids, with all layers and the full
vocabulary of the configuration it names.  Gates (north star): f32 mode
max-abs <= 1e-4 and cosine >= 0.99999 per row; bf16 mode cosine >= 0.999 per
row.

The large models are written once under $FFWD_B200_MODEL_ROOT (default
/tmp/ffwd_b200_models), the same place bench.py writes its model.
"""

import os

import numpy as np
import pytest

from ffwd_b200 import native, synth
from oracle import ref as oref

from helpers import cos_rows

pytestmark = pytest.mark.gpu

F32_MAXABS = 1e-4
F32_COS = 0.99999
BF16_COS = 0.999


def _ref(d, seqs):
    assert oref.available(), "oracle/_ref/libffwd_ref.so is not built (make -C oracle)"
    r = oref.RefModel(d, threads=os.cpu_count() or 1)
    try:
        return r.encode_batch(seqs)
    finally:
        r.close()


def _check(out, ref, exact):
    assert out.shape == ref.shape
    assert np.isfinite(out).all()
    cos = cos_rows(out, ref)
    if exact:
        err = float(np.abs(out - ref).max())
        assert err <= F32_MAXABS, f"max-abs {err}"
        assert cos.min() >= F32_COS, f"cos {cos.min()}"
    else:
        assert cos.min() >= BF16_COS, f"cos {cos.min()}"
    return cos


def _gpu(d, seqs, mode, weight_dtype=None):
    m = native.B200Model(d, gemm_mode=mode, weight_dtype=weight_dtype)
    try:
        return m.encode_batch(seqs), m.precision
    finally:
        m.close()


def test_minilm_f32_whole_config():
    """Config 1 whole: 6 layers, vocab 30522, 32 sequences U[16,128], mean + L2."""
    d = synth.ensure_model(synth.spec("minilm"))
    seqs = synth.token_batch("minilm", seed=1)
    assert len(seqs) == 32
    out, prec = _gpu(d, seqs, "f32")
    assert prec in (2, 3)
    _check(out, _ref(d, seqs), True)


@pytest.mark.parametrize("cfg,mode,exact", [("bge-base", "f32", True),
                                             ("bge-base", "bf16", False),
                                             ("bge-base-bf16", "bf16", False),
                                             ("bge-base-bf16", "f32", True)])
def test_bge_base_12_layers(cfg, mode, exact):
    """Config 2 at full depth on its first 16 sequences (lognormal lengths), CLS + L2."""
    d = synth.ensure_model(synth.spec(cfg))
    seqs = synth.token_batch("bge-base", seed=1)[:16]
    out, _ = _gpu(d, seqs, mode)
    _check(out, _ref(d, seqs), exact)


def test_xlmr_large_24_layers_full_vocab():
    """Config 3: 24 layers, vocab 250002, position offset 2, 2 x 512 tokens, mean + L2."""
    d = synth.ensure_model(synth.spec("xlmr-large"))
    seqs = synth.token_batch("xlmr-large", seed=1, batch=2)
    out, prec = _gpu(d, seqs, "bf16")
    assert prec == 0
    _check(out, _ref(d, seqs), False)


def test_qwen3_0_6b_28_layers_full_vocab():
    """Config 4 (the benchmark model): 28 layers, vocab 151669, the first four
    sequences of the benchmark's seeded batch, last token + L2."""
    d = synth.ensure_model(synth.spec("qwen3-0.6b"))
    seqs = synth.token_batch("qwen3-0.6b", seed=1)[:4]
    out, prec = _gpu(d, seqs, "bf16")
    assert prec == 0
    _check(out, _ref(d, seqs), False)


def test_qwen3_8b_4_layers_8192_document_matryoshka():
    """Config 5 shapes (hidden 4096, 32 / 8 heads, FFN 12288, vocab 151665) at
    4 layers on one 8192-token document: last token, Matryoshka truncation to
    1024 dims, then L2 (tools/server/encode.c:107-122 semantics)."""
    d = synth.ensure_model(synth.spec("qwen3-8b", n_layers=4))
    seqs = synth.token_batch("qwen3-8b", seed=1, batch=1)
    m = native.B200Model(d, gemm_mode="bf16")
    try:
        out = m.encode_batch_as(seqs, 1024, True, "f32")
    finally:
        m.close()
    ref = _ref(d, seqs)[:, :1024].astype(np.float64)
    ref = (ref / np.linalg.norm(ref, axis=1, keepdims=True)).astype(np.float32)
    _check(out, ref, False)
    assert abs(float(np.linalg.norm(out[0])) - 1.0) < 1e-5
