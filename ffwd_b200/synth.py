"""Seeded synthetic models and token batches for the five benchmark configs.

The reference has no public dataset on this path: its benchmark feeds token ids
straight into ``ffwd_encode_batch`` (libffwd/ffwd.h:187) for a model directory
that holds ``config.json``, sentence-transformers metadata and safetensors
weights.  This module writes such a directory with random-init weights and the
reference's tensor names, so both the reference CPU path and this backend load
the very same bytes:

* Qwen3 names follow libffwd/model.c:407-426 (``layers.N.self_attn.q_proj.weight``,
  ``layers.N.mlp.gate_proj.weight``, ``embed_tokens.weight``, ``norm.weight``).
* BERT / XLM-R names follow libffwd/model.c:218-305 (``embeddings.*``,
  ``encoder.layer.N.attention.self.query.weight`` ...).
* ``config.json`` keys are the ones libffwd/config.c:178-341 reads; pooling and
  normalisation come from ``1_Pooling/config.json`` and ``modules.json``
  (config.c:96-155).

Weights are N(0, 0.02^2); norm gains are 1 + N(0, 0.02^2) and norm biases
N(0, 0.02^2).  Token batches follow each config's length and id distribution
(seed 1 by default).
"""

from __future__ import annotations

import hashlib
import json
import os
import struct
from dataclasses import dataclass, field, asdict, replace

import numpy as np

__all__ = [
    "ModelSpec", "CONFIGS", "spec", "write_model", "ensure_model", "token_batch",
    "f32_to_bf16_bits", "bf16_bits_to_f32",
]


@dataclass(frozen=True)
class ModelSpec:
    name: str
    family: str               # "qwen3" | "bert" | "xlm-roberta" | "qwen2"
    n_layers: int
    hidden: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    dtype: str                # "f32" | "bf16" | "f16" (safetensors storage dtype)
    pooling: str              # "mean" | "cls" | "last"
    normalize: bool = True
    max_pos: int = 512
    pad_token_id: int = 1
    type_vocab: int = 2
    eps: float = 1e-12        # layer_norm_eps (BERT) or rms_norm_eps (Qwen)
    rope_theta: float = 1e6
    hidden_act: str = "gelu"
    is_causal: bool | None = None
    seed: int = 0
    late_dim: int = 0         # > 0: late-interaction model with a 1_Dense head [late_dim, hidden]


# The five BASELINE configurations (shapes exactly as stated there).
CONFIGS = {
    "minilm": ModelSpec("minilm", "bert", 6, 384, 12, 12, 32, 1536, 30522, "f32", "mean",
                        max_pos=512, type_vocab=2, eps=1e-12),
    "bge-base": ModelSpec("bge-base", "bert", 12, 768, 12, 12, 64, 3072, 30522, "f32", "cls",
                          max_pos=512, type_vocab=2, eps=1e-12),
    "bge-base-bf16": ModelSpec("bge-base-bf16", "bert", 12, 768, 12, 12, 64, 3072, 30522, "bf16",
                               "cls", max_pos=512, type_vocab=2, eps=1e-12),
    "xlmr-large": ModelSpec("xlmr-large", "xlm-roberta", 24, 1024, 16, 16, 64, 4096, 250002, "bf16",
                            "mean", max_pos=514, pad_token_id=1, type_vocab=1, eps=1e-5),
    "qwen3-0.6b": ModelSpec("qwen3-0.6b", "qwen3", 28, 1024, 16, 8, 128, 3072, 151669, "bf16",
                            "last", eps=1e-6, rope_theta=1e6),
    "qwen3-8b": ModelSpec("qwen3-8b", "qwen3", 36, 4096, 32, 8, 128, 12288, 151665, "bf16", "last",
                          eps=1e-6, rope_theta=1e6),
}


def spec(name: str, **overrides) -> ModelSpec:
    """A named config, optionally with fields replaced (e.g. fewer layers)."""
    s = CONFIGS[name]
    if overrides:
        s = replace(s, **overrides)
        if "name" not in overrides:
            tag = ",".join(f"{k}={overrides[k]}" for k in sorted(overrides))
            s = replace(s, name=f"{name}[{tag}]")
    return s


# --------------------------------------------------------------------------- bf16


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bit patterns (uint16)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    lsb = (u >> np.uint32(16)) & np.uint32(1)
    r = (u + np.uint32(0x7FFF) + lsb) >> np.uint32(16)
    nan = np.isnan(x)
    if nan.any():
        r = np.where(nan, np.uint32(0x7FC0), r)
    return r.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


# --------------------------------------------------------------------------- tensors


def _tensor_list(s: ModelSpec):
    """(name, shape, kind) for every tensor; kind in {w, gain, bias}."""
    H, I, L = s.hidden, s.intermediate, s.n_layers
    out = []
    if s.family in ("qwen3", "qwen2"):
        q_dim, kv_dim = s.n_heads * s.head_dim, s.n_kv_heads * s.head_dim
        out.append(("embed_tokens.weight", (s.vocab, H), "w"))
        for i in range(L):
            p = f"layers.{i}."
            out += [
                (p + "self_attn.q_proj.weight", (q_dim, H), "w"),
                (p + "self_attn.k_proj.weight", (kv_dim, H), "w"),
                (p + "self_attn.v_proj.weight", (kv_dim, H), "w"),
                (p + "self_attn.o_proj.weight", (H, q_dim), "w"),
            ]
            if s.family == "qwen2":
                out += [
                    (p + "self_attn.q_proj.bias", (q_dim,), "bias"),
                    (p + "self_attn.k_proj.bias", (kv_dim,), "bias"),
                    (p + "self_attn.v_proj.bias", (kv_dim,), "bias"),
                ]
            else:
                out += [
                    (p + "self_attn.q_norm.weight", (s.head_dim,), "gain"),
                    (p + "self_attn.k_norm.weight", (s.head_dim,), "gain"),
                ]
            out += [
                (p + "input_layernorm.weight", (H,), "gain"),
                (p + "post_attention_layernorm.weight", (H,), "gain"),
                (p + "mlp.gate_proj.weight", (I, H), "w"),
                (p + "mlp.up_proj.weight", (I, H), "w"),
                (p + "mlp.down_proj.weight", (H, I), "w"),
            ]
        out.append(("norm.weight", (H,), "gain"))
    else:
        out += [
            ("embeddings.word_embeddings.weight", (s.vocab, H), "w"),
            ("embeddings.position_embeddings.weight", (s.max_pos, H), "w"),
            ("embeddings.token_type_embeddings.weight", (s.type_vocab, H), "w"),
            ("embeddings.LayerNorm.weight", (H,), "gain"),
            ("embeddings.LayerNorm.bias", (H,), "bias"),
        ]
        for i in range(L):
            p = f"encoder.layer.{i}."
            out += [
                (p + "attention.self.query.weight", (H, H), "w"),
                (p + "attention.self.query.bias", (H,), "bias"),
                (p + "attention.self.key.weight", (H, H), "w"),
                (p + "attention.self.key.bias", (H,), "bias"),
                (p + "attention.self.value.weight", (H, H), "w"),
                (p + "attention.self.value.bias", (H,), "bias"),
                (p + "attention.output.dense.weight", (H, H), "w"),
                (p + "attention.output.dense.bias", (H,), "bias"),
                (p + "attention.output.LayerNorm.weight", (H,), "gain"),
                (p + "attention.output.LayerNorm.bias", (H,), "bias"),
                (p + "intermediate.dense.weight", (I, H), "w"),
                (p + "intermediate.dense.bias", (I,), "bias"),
                (p + "output.dense.weight", (H, I), "w"),
                (p + "output.dense.bias", (H,), "bias"),
                (p + "output.LayerNorm.weight", (H,), "gain"),
                (p + "output.LayerNorm.bias", (H,), "bias"),
            ]
    return out


def _config_json(s: ModelSpec) -> dict:
    if s.family in ("qwen3", "qwen2"):
        c = {
            "model_type": s.family,
            "hidden_size": s.hidden,
            "num_hidden_layers": s.n_layers,
            "num_attention_heads": s.n_heads,
            "num_key_value_heads": s.n_kv_heads,
            "head_dim": s.head_dim,
            "intermediate_size": s.intermediate,
            "vocab_size": s.vocab,
            "rms_norm_eps": s.eps,
            "rope_theta": s.rope_theta,
            "max_position_embeddings": 32768,
            "torch_dtype": _TORCH_DTYPE[s.dtype],
        }
    else:
        c = {
            "model_type": s.family,
            "hidden_size": s.hidden,
            "num_hidden_layers": s.n_layers,
            "num_attention_heads": s.n_heads,
            "intermediate_size": s.intermediate,
            "vocab_size": s.vocab,
            "layer_norm_eps": s.eps,
            "max_position_embeddings": s.max_pos,
            "type_vocab_size": s.type_vocab,
            "hidden_act": s.hidden_act,
            "pad_token_id": s.pad_token_id,
            "torch_dtype": _TORCH_DTYPE[s.dtype],
        }
    if s.is_causal is not None:
        c["is_causal"] = bool(s.is_causal)
    return c


_TORCH_DTYPE = {"f32": "float32", "bf16": "bfloat16", "f16": "float16"}
_ST_DTYPE = {"f32": "F32", "bf16": "BF16", "f16": "F16"}


def _encode(v: np.ndarray, dtype: str) -> bytes:
    """Tensor bytes in the storage dtype (bf16 / f16 round to nearest even)."""
    if dtype == "bf16":
        return f32_to_bf16_bits(v).tobytes()
    if dtype == "f16":
        return v.astype(np.float16).tobytes()
    return v.astype(np.float32).tobytes()


def _safetensors_header(entries) -> bytes:
    hdr = {"__metadata__": {"format": "pt"}}
    for name, dt, shape, off, nbytes in entries:
        hdr[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [off, off + nbytes]}
    raw = json.dumps(hdr, separators=(",", ":")).encode()
    raw += b" " * ((8 - len(raw) % 8) % 8)
    return raw


def _gen(rng: np.random.Generator, shape, kind: str) -> np.ndarray:
    n = int(np.prod(shape))
    v = rng.standard_normal(n, dtype=np.float32)
    v *= np.float32(0.02)
    if kind == "gain":
        v += np.float32(1.0)
    return v.reshape(shape)


def write_model(s: ModelSpec, out_dir: str, max_shard_bytes: int = 4 << 30) -> str:
    """Write config + metadata + safetensors shards for spec ``s`` into out_dir."""
    os.makedirs(os.path.join(out_dir, "1_Pooling"), exist_ok=True)
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(_config_json(s), f, indent=1)
    with open(os.path.join(out_dir, "1_Pooling", "config.json"), "w") as f:
        json.dump({
            "word_embedding_dimension": s.hidden,
            "pooling_mode_cls_token": s.pooling == "cls",
            "pooling_mode_mean_tokens": s.pooling == "mean",
            "pooling_mode_max_tokens": False,
            "pooling_mode_mean_sqrt_len_tokens": False,
            "pooling_mode_weightedmean_tokens": False,
            "pooling_mode_lasttoken": s.pooling == "last",
        }, f, indent=1)
    mods = [
        {"idx": 0, "name": "0", "path": "", "type": "sentence_transformers.models.Transformer"},
        {"idx": 1, "name": "1", "path": "1_Pooling", "type": "sentence_transformers.models.Pooling"},
    ]
    if s.normalize:
        mods.append({"idx": 2, "name": "2", "path": "2_Normalize",
                     "type": "sentence_transformers.models.Normalize"})
    with open(os.path.join(out_dir, "modules.json"), "w") as f:
        json.dump(mods, f, indent=1)

    rng = np.random.default_rng(s.seed)
    tensors = _tensor_list(s)
    # Matrices follow the storage dtype; the reference reads 1-D norms/biases
    # and BERT position/type tables as F32 or BF16 alike (load_norm_f32).
    st_dt = _ST_DTYPE[s.dtype]
    esz = 4 if s.dtype == "f32" else 2
    shards, cur, cur_bytes = [], [], 0
    for name, shape, kind in tensors:
        nb = int(np.prod(shape)) * esz
        if cur and cur_bytes + nb > max_shard_bytes:
            shards.append(cur)
            cur, cur_bytes = [], 0
        cur.append((name, shape, kind))
        cur_bytes += nb
    if cur:
        shards.append(cur)
    n_sh = len(shards)
    for si, group in enumerate(shards):
        fname = "model.safetensors" if n_sh == 1 else f"model-{si + 1:05d}-of-{n_sh:05d}.safetensors"
        entries, off = [], 0
        for name, shape, kind in group:
            nb = int(np.prod(shape)) * esz
            entries.append((name, st_dt, shape, off, nb))
            off += nb
        hdr = _safetensors_header(entries)
        with open(os.path.join(out_dir, fname), "wb") as f:
            f.write(struct.pack("<Q", len(hdr)))
            f.write(hdr)
            for name, shape, kind in group:
                f.write(_encode(_gen(rng, shape, kind), s.dtype))
    if s.late_dim > 0:
        write_late_projection(s, out_dir)
    return out_dir


def write_late_projection(s: ModelSpec, out_dir: str) -> None:
    """1_Dense head of a late-interaction model: ``1_Dense/config.json`` and
    ``1_Dense/model.safetensors`` holding ``linear.weight`` [late_dim, hidden]
    (no bias) in the model's storage dtype, the files libffwd/late.c:41-86
    loads.  Weights N(0, 0.02^2) from their own seeded stream."""
    dd = os.path.join(out_dir, "1_Dense")
    os.makedirs(dd, exist_ok=True)
    with open(os.path.join(dd, "config.json"), "w") as f:
        json.dump({"in_features": s.hidden, "out_features": s.late_dim, "bias": False,
                   "activation_function": "torch.nn.modules.linear.Identity"}, f, indent=1)
    v = _gen(np.random.default_rng(s.seed + 7919), (s.late_dim, s.hidden), "w")
    st_dt, data = _ST_DTYPE[s.dtype], _encode(v, s.dtype)
    hdr = _safetensors_header([("linear.weight", st_dt, (s.late_dim, s.hidden), 0, len(data))])
    with open(os.path.join(dd, "model.safetensors"), "wb") as f:
        f.write(struct.pack("<Q", len(hdr)))
        f.write(hdr)
        f.write(data)


def _spec_key(s: ModelSpec) -> str:
    d = asdict(s)
    if not d.get("late_dim"):
        d.pop("late_dim", None)  # keys of pooled models predate the field
    return hashlib.sha1(json.dumps(d, sort_keys=True).encode()).hexdigest()[:12]


def ensure_model(s: ModelSpec, root: str | None = None) -> str:
    """Write the model once under root (default $FFWD_B200_MODEL_ROOT or /tmp)."""
    root = root or os.environ.get("FFWD_B200_MODEL_ROOT", "/tmp/ffwd_b200_models")
    d = os.path.join(root, f"{s.name.replace('[', '_').replace(']', '').replace(',', '_').replace('=', '')}-{_spec_key(s)}")
    done = os.path.join(d, ".complete")
    if not os.path.exists(done):
        write_model(s, d)
        open(done, "w").close()
    return d


# --------------------------------------------------------------------------- token batches


def token_batch(config: str, seed: int = 1, batch: int | None = None, vocab: int | None = None):
    """Seeded token id lists following a BASELINE config's distribution.

    Returns a list of int32 numpy arrays, one per sequence.
    """
    rng = np.random.default_rng(seed)
    seqs = []
    if config == "minilm":
        B = batch or 32
        V = vocab or 30522
        for _ in range(B):
            L = int(rng.integers(16, 129))
            ids = rng.integers(1000, min(30521, V - 1) + 1, size=L).astype(np.int32)
            ids[0], ids[-1] = 101, 102
            seqs.append(ids)
    elif config in ("bge-base", "bge-base-bf16"):
        B = batch or 256
        V = vocab or 30522
        for _ in range(B):
            L = int(np.clip(np.round(np.exp(np.log(64.0) + 0.8 * rng.standard_normal())), 8, 512))
            ids = rng.integers(1000, min(30521, V - 1) + 1, size=L).astype(np.int32)
            ids[0], ids[-1] = 101, 102
            seqs.append(ids)
    elif config == "xlmr-large":
        B = batch or 64
        V = vocab or 250002
        for _ in range(B):
            ids = rng.integers(3, min(250001, V - 1) + 1, size=512).astype(np.int32)
            ids[0], ids[-1] = 0, 2
            seqs.append(ids)
    elif config == "qwen3-0.6b":
        B = batch or 128
        V = vocab or 151669
        for _ in range(B):
            L = int(rng.integers(32, 2049))
            ids = rng.integers(0, min(151642, V - 1) + 1, size=L + 1).astype(np.int32)
            ids[-1] = min(151643, V - 1)
            seqs.append(ids)
    elif config == "qwen3-8b":
        B = batch or 64
        V = vocab or 151665
        for _ in range(B):
            ids = rng.integers(0, min(151642, V - 1) + 1, size=8192).astype(np.int32)
            ids[-1] = min(151643, V - 1)
            seqs.append(ids)
    else:
        raise KeyError(config)
    return seqs
