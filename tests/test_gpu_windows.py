"""Short sequences sharing attention work items (windows) in the 16-bit plans.

Neighbouring sequences of 1..128 tokens in the packed batch are cut into
windows of at most 128 rows (grouped-query models: the two blocks of an item
are two heads) or 256 rows (one key/value head per head: the blocks are the
window's two halves); each query row attends only to its own sequence.  These
batches mix runs of short sequences (lengths 1, 2, odd, 127, 128) with longer
ones, so windows of one and of several sequences, sequences straddling the
128-row boundary of a two-tile window, and rows past the window's end all
occur; each pooled row is checked against the CPU checker at the bf16 gate
(cosine >= 0.999), for mean / CLS / last-token pooling, causal and
bidirectional attention, head_dim 32 / 64 / 128, bf16 and f16 operands."""

import numpy as np
import pytest

from ffwd_b200 import native, synth
from oracle import forward as of

from helpers import small_spec, cos_rows

pytestmark = pytest.mark.gpu

LENS = [5, 1, 2, 60, 127, 128, 90, 33, 300, 17, 70, 71, 3, 128, 100, 200, 64, 64, 64, 64, 9]


def _batch(s, seed):
    rng = np.random.default_rng(seed)
    seqs = []
    for L in LENS:
        if s.family in ("qwen3", "qwen2"):
            q = rng.integers(0, s.vocab, size=L).astype(np.int32)
            q[-1] = min(151643, s.vocab - 1)
        else:
            q = rng.integers(1000, min(30521, s.vocab - 1) + 1, size=L).astype(np.int32)
            q[0] = 101
            if L > 1:
                q[-1] = 102
        seqs.append(q)
    return seqs


@pytest.mark.parametrize("key,mode", [
    ("minilm-2l", "bf16"),       # MHA, head_dim 32, mean pooling
    ("bge-bf16-2l", "bf16"),     # MHA, head_dim 64, CLS pooling
    ("qwen3-2l", "bf16"),        # GQA 16 / 8, head_dim 128, causal, last token
    ("qwen3-bidir-1l", "bf16"),  # GQA, bidirectional
    ("qwen3-f32-2l", "16f"),     # f16 operands
])
def test_short_sequence_windows_match_checker(key, mode, model_root):
    s = small_spec(key)
    d = synth.ensure_model(s, model_root)
    m = native.B200Model(d, gemm_mode=mode)
    assert m.precision in (0, 1)
    seqs = _batch(s, seed=21)
    lens = [len(q) for q in seqs]
    heads, kv = s.n_heads, s.n_kv_heads
    causal = s.family in ("qwen3", "qwen2") and s.is_causal is not False
    items = native.attention_items(lens, heads, kv, causal=causal, windows=True)
    assert (items[:, 6] > 1).any(), "the batch must form multi-sequence windows"
    out = m.encode_batch(seqs)
    ref = of.OracleModel(d).encode_batch(seqs)
    cos = cos_rows(out, ref)
    assert np.isfinite(out).all()
    assert cos.min() >= 0.999, f"min cosine {cos.min()} at {int(cos.argmin())}"
    # the same sequences in another order form other windows
    perm = np.random.default_rng(4).permutation(len(seqs))
    out2 = m.encode_batch([seqs[i] for i in perm])
    assert cos_rows(out2, out[perm]).min() >= 0.9999
    m.close()
