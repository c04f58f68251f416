"""GEMM modes x weight storage on the B200 path (--gpu-gemm-mode f32 / tf32 /
bf16 / 16f and --gpu-weight-dtype; libffwd/cuda.cu:169-247, linear_ex
2905-2964, 4225-4237): the precision plan chosen at load, and parity with the
reference's CPU path on its golden fixtures.

F16 safetensors are widened to F32 by the reference at load (model.c:158-172),
so by default they run exactly like F32 files; an explicit f16 storage runs f16
tensor-core operands (kind::f16 with the f16 format) on the decoder in every
mode, and on BERT in the 16-bit modes.

Precision codes (ffwd_b200_precision): 0 single-pass bf16, 1 single-pass f16,
2 / 3 split-bf16 2- / 3-pass, 4 tf32 (kind::tf32 GEMMs, split-bf16 attention).
Gates: exact plans max-abs <= 1e-4 and cosine >= 0.99999 per row; the tf32 plan
cosine >= 0.9999 and max-abs <= 2e-3 (tf32 keeps 11 significant bits, as the
reference's CUBLAS_COMPUTE_32F_FAST_TF32 does); 16-bit plans cosine >= 0.999
per row."""

import numpy as np
import pytest

from ffwd_b200 import native

from golden_util import load
from helpers import cos_rows

pytestmark = pytest.mark.gpu

F32_MAXABS = 1e-4
F32_COS = 0.99999
TF32_MAXABS = 2e-3
TF32_COS = 0.9999
BF16_COS = 0.999


@pytest.fixture(autouse=True, scope="module")
def _restore_defaults():
    yield
    L = native.lib()
    L.ffwd_b200_set_weights_default()
    L.ffwd_b200_set_fast_gemm(b"f32")


def run(name, mode, wdt, model_root):
    spec, d, seqs, expected = load(name, model_root)
    m = native.B200Model(d, gemm_mode=mode, weight_dtype=wdt)
    try:
        return m.precision, m.encode_batch(seqs), expected
    finally:
        m.close()


CASES = [
    # fixture, gemm mode, weight storage, precision plan, exact
    # decoder, F16 file
    ("qwen3_f16", "f32", "file", 3, True),
    ("qwen3_f16", "tf32", "file", 4, True),
    ("qwen3_f16", "bf16", "file", 0, False),
    ("qwen3_f16", "16f", "file", 1, False),
    ("qwen3_f16", "f32", "f16", 1, False),
    ("qwen3_f16", "bf16", "f16", 1, False),
    ("qwen3_f16", "f32", "bf16", 0, False),
    # decoder, BF16 file: bf16 operands whatever the mode
    ("qwen3_last", "16f", "file", 0, False),
    ("qwen3_last", "tf32", "file", 0, False),
    # BERT, F16 file
    ("minilm_f16", "f32", "file", 3, True),
    ("minilm_f16", "tf32", "f16", 4, True),
    ("minilm_f16", "16f", "file", 1, False),
    ("minilm_f16", "bf16", "f16", 1, False),
    ("minilm_f16", "16f", "bf16", 0, False),
    ("minilm_f16", "f32", "bf16", 2, False),
    # BERT, F32 / BF16 files (head_dim 32 / 64)
    ("minilm_f32", "tf32", "file", 4, True),
    ("bge_bf16_cls", "tf32", "file", 4, True),
    ("xlmr_mean", "tf32", "file", 4, True),
    ("minilm_f32", "16f", "file", 1, False),
    ("bge_bf16_cls", "16f", "f16", 1, False),
    ("bge_bf16_cls", "16f", "file", 0, False),
]


@pytest.mark.parametrize("name,mode,wdt,prec,exact", CASES)
def test_mode_plan_and_parity(name, mode, wdt, prec, exact, model_root):
    got_prec, out, ref = run(name, mode, wdt, model_root)
    assert got_prec == prec
    assert np.isfinite(out).all()
    cos = cos_rows(out, ref)
    if exact:
        err = np.abs(out - ref).max()
        maxabs, mincos = (TF32_MAXABS, TF32_COS) if prec == 4 else (F32_MAXABS, F32_COS)
        assert err <= maxabs, f"max-abs {err}"
        assert cos.min() >= mincos, f"cos {cos.min()}"
    else:
        assert cos.min() >= BF16_COS, f"cos {cos.min()}"


@pytest.mark.parametrize("name,f16_args,bf16_args", [
    ("qwen3_f16", ("f32", "f16"), ("f32", "bf16")),
    ("minilm_f16", ("16f", "file"), ("bf16", "file")),
])
def test_f16_operands_beat_bf16(name, f16_args, bf16_args, model_root):
    """f16 operands keep 3 more significand bits than bf16: on the same F16
    weights the embeddings sit measurably closer to the reference."""
    p16, o16, ref = run(name, *f16_args, model_root)
    pb, ob, _ = run(name, *bf16_args, model_root)
    assert (p16, pb) == (1, 0)
    e16 = np.abs(o16 - ref).max()
    eb = np.abs(ob - ref).max()
    assert e16 < 0.5 * eb, f"f16 max-abs {e16} vs bf16 {eb}"


@pytest.mark.parametrize("name", ["qwen3_f16", "minilm_f32"])
def test_tf32_between_f32_and_bf16(name, model_root):
    """The tf32 plan sits between the exact plan and the bf16 plan."""
    p32, o32, ref = run(name, "f32", "file", model_root)
    ptf, otf, _ = run(name, "tf32", "file", model_root)
    pb, ob, _ = run(name, "bf16", "file", model_root)
    assert (p32, ptf, pb) == (3, 4, 0)
    e32, etf, eb = (np.abs(o - ref).max() for o in (o32, otf, ob))
    assert e32 < etf < eb, (e32, etf, eb)
