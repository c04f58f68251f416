"""Shared helpers for the parity tests (test code only)."""

import numpy as np

from ffwd_b200 import synth

# Small variants of the BASELINE configs, sized so the CPU checker finishes in
# seconds: same hidden sizes / heads / head_dim / FFN ratios, fewer layers and
# (for the decoder / XLM-R) a smaller vocabulary.
SMALL = {
    "minilm-2l": ("minilm", dict(n_layers=2)),
    "bge-2l": ("bge-base", dict(n_layers=2)),
    "bge-bf16-2l": ("bge-base-bf16", dict(n_layers=2)),
    "xlmr-2l": ("xlmr-large", dict(n_layers=2, vocab=8192)),
    "qwen3-2l": ("qwen3-0.6b", dict(n_layers=2, vocab=8192)),
    "qwen3-f32-2l": ("qwen3-0.6b", dict(n_layers=2, vocab=8192, dtype="f32")),
    "qwen3-bidir-1l": ("qwen3-0.6b", dict(n_layers=1, vocab=4096, is_causal=False)),
    "qwen2-1l": ("qwen3-0.6b", dict(n_layers=1, vocab=4096, family="qwen2", pooling="mean")),
    "bert-tanh-1l": ("minilm", dict(n_layers=1, hidden_act="gelu_new", pooling="cls")),
    # F16 safetensors (the reference widens them to F32 at load)
    "qwen3-f16-1l": ("qwen3-0.6b", dict(n_layers=1, vocab=4096, dtype="f16")),
    "minilm-f16-2l": ("minilm", dict(n_layers=2, dtype="f16")),
    # late interaction (1_Dense head)
    "qwen3-late-2l": ("qwen3-0.6b", dict(n_layers=2, vocab=8192, late_dim=128)),
    "qwen3-late-f32-1l": ("qwen3-0.6b", dict(n_layers=1, vocab=4096, dtype="f32", late_dim=6)),
    "minilm-late-2l": ("minilm", dict(n_layers=2, late_dim=96)),
}


def small_spec(key):
    base, ov = SMALL[key]
    return synth.spec(base, **ov)


def small_batch(key, n=6, max_len=None, seed=1):
    base, ov = SMALL[key]
    s = small_spec(key)
    dist = base if base != "bge-base-bf16" else "bge-base"
    seqs = synth.token_batch(dist, seed=seed, batch=n, vocab=s.vocab)
    if max_len is not None:
        seqs = [q[:max_len] if len(q) > max_len else q for q in seqs]
        if s.family in ("qwen3", "qwen2"):
            for q in seqs:
                q[-1] = min(151643, s.vocab - 1)
    return seqs


def cos_rows(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return (a * b).sum(1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1))
