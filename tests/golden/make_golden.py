"""Generate the golden fixtures of this directory from the reference itself.

Each fixture holds a seeded synthetic model spec (the model is regenerated
bit-identically by ``ffwd_b200.synth.write_model``), a packed token batch and
the embeddings the reference's own CPU path (``oracle/_ref/libffwd_ref.so``,
built from the unmodified reference sources by ``oracle/Makefile``) returns
for it through ``ffwd_model_encode_batch``.

    python tests/golden/make_golden.py    (needs oracle/_ref, i.e. `make -C oracle`)
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
from oracle.ref import RefModel  # noqa: E402
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
}


def main():
    root = tempfile.mkdtemp(prefix="ffwd_golden_")
    for name, (key, mk) in CASES.items():
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


if __name__ == "__main__":
    main()
