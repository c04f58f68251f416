"""CPU restatement (numpy, f32) of the reference's packed embedding forward.

TEST INFRASTRUCTURE ONLY.  This module is the checker: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it.
The product path (``ffwd_b200``) never calls it and has no CPU fallback.

Parity pin: the restatement is checked against the reference's own compiled
CPU path (``oracle/_ref/libffwd_ref.so``, built from the unmodified reference
sources by ``oracle/Makefile``) in ``tests/test_oracle.py``, and against
fixtures produced by that library (``tests/golden/``).

Each function names the reference code it restates (paths are relative to the
reference project root).
"""

from __future__ import annotations

import json
import os
import struct

import numpy as np

F32 = np.float32


# --------------------------------------------------------------------------- loading


def _read_json(path, default=None):
    if not os.path.exists(path):
        return default
    with open(path) as f:
        return json.load(f)


def parse_config(model_dir: str) -> dict:
    """libffwd/config.c:178-341 (defaults, family detection, metadata files)."""
    root = _read_json(os.path.join(model_dir, "config.json"))
    c = {
        "hidden": int(root.get("hidden_size", 0)),
        "n_layers": int(root.get("num_hidden_layers", 0)),
        "n_heads": int(root.get("num_attention_heads", 0)),
        "n_kv_heads": int(root.get("num_key_value_heads", 0)),
        "head_dim": int(root.get("head_dim", 128)),
        "inter": int(root.get("intermediate_size", 0)),
        "vocab": int(root.get("vocab_size", 151936)),
        "rms_eps": F32(root.get("rms_norm_eps", 1e-6)),
        "ln_eps": F32(root.get("layer_norm_eps", 1e-12)),
        "rope_theta": F32(root.get("rope_theta", 1e6)),
        "max_pos": int(root.get("max_position_embeddings", 0)),
        "pos_offset": 0,
        "type_vocab": int(root.get("type_vocab_size", 2)),
        "family": "qwen",
        "qk_norm": True,
        "qkv_bias": False,
        "causal": False,
        "pooling": "mean",
        "normalize": False,
        "act": "erf",
    }
    mt = root.get("model_type")
    if mt == "qwen3":
        c.update(causal=True, pooling="last", normalize=True)
    elif mt == "qwen2":
        c.update(qk_norm=False, qkv_bias=True, causal=True)
    elif mt in ("bert", "roberta", "xlm-roberta"):
        c.update(family="bert", qk_norm=False, qkv_bias=True, causal=False)
        c["n_kv_heads"] = c["n_heads"]
        c["head_dim"] = c["hidden"] // c["n_heads"]
        if mt in ("roberta", "xlm-roberta"):
            c["pos_offset"] = int(root.get("pad_token_id", 1)) + 1
        if root.get("hidden_act") in ("gelu_new", "gelu_pytorch_tanh"):
            c["act"] = "tanh"
    if "is_causal" in root:
        c["causal"] = bool(root["is_causal"])
    pool = _read_json(os.path.join(model_dir, "1_Pooling", "config.json"))
    if pool is not None:
        if pool.get("pooling_mode_cls_token"):
            c["pooling"] = "cls"
        elif pool.get("pooling_mode_lasttoken"):
            c["pooling"] = "last"
        else:
            c["pooling"] = "mean"
    mods = _read_json(os.path.join(model_dir, "modules.json"))
    if mods is not None:
        c["normalize"] = any(m.get("type") == "sentence_transformers.models.Normalize" for m in mods)
    c["q_dim"] = c["n_heads"] * c["head_dim"]
    c["kv_dim"] = c["n_kv_heads"] * c["head_dim"]
    return c


def load_tensors(model_dir: str) -> dict:
    """Safetensors reader (libffwd/safetensors.c); every tensor widened to f32."""
    out = {}
    files = sorted(f for f in os.listdir(model_dir) if f.endswith(".safetensors"))
    for fn in files:
        with open(os.path.join(model_dir, fn), "rb") as f:
            n = struct.unpack("<Q", f.read(8))[0]
            hdr = json.loads(f.read(n))
            base = 8 + n
        mm = np.memmap(os.path.join(model_dir, fn), dtype=np.uint8, mode="r")
        for name, meta in hdr.items():
            if name == "__metadata__":
                continue
            a, b = meta["data_offsets"]
            raw = mm[base + a: base + b]
            if meta["dtype"] == "F32":
                v = raw.view(np.float32)
            elif meta["dtype"] == "BF16":
                v = (raw.view(np.uint16).astype(np.uint32) << 16).view(np.float32)
            elif meta["dtype"] == "F16":  # widened exactly at load (model.c:158-172)
                v = raw.view(np.float16).astype(np.float32)
            else:
                raise ValueError(meta["dtype"])
            out[name] = np.array(v, dtype=F32).reshape(meta["shape"])
    return out


# --------------------------------------------------------------------------- kernels


def rms_norm(x, w, eps):
    """libffwd/norm.c:34-46: out = x * 1/sqrt(mean(x^2) + eps) * w."""
    ss = np.sum(x * x, axis=-1, dtype=F32, keepdims=True)
    inv = F32(1.0) / np.sqrt(ss / F32(x.shape[-1]) + eps)
    return (x * inv * w).astype(F32)


def layer_norm(x, g, b, eps):
    """libffwd/norm.c:107-138 (two-pass mean / variance)."""
    h = F32(1.0 / x.shape[-1])
    mean = np.sum(x, axis=-1, dtype=F32, keepdims=True) * h
    d = x - mean
    var = np.sum(d * d, axis=-1, dtype=F32, keepdims=True) * h
    inv = F32(1.0) / np.sqrt(var + eps)
    return (g * d * inv + b).astype(F32)


def rope_tables(n_pos, head_dim, theta):
    """libffwd/model_blas.c:85-123: f32 cos/sin cache, halves duplicated."""
    half = head_dim // 2
    d = np.arange(half, dtype=F32)
    inv = F32(1.0) / np.power(F32(theta), (F32(2.0) * d) / F32(head_dim)).astype(F32)
    pos = np.arange(n_pos, dtype=F32)[:, None]
    ang = (pos * inv[None, :]).astype(F32)
    c, s = np.cos(ang).astype(F32), np.sin(ang).astype(F32)
    return np.concatenate([c, c], 1), np.concatenate([s, s], 1)


def apply_rope_neox(x, cos, sin, n_heads, head_dim):
    """libffwd/rope.c:54-137: x*cos + cat(-x2, x1)*sin per head, positions 0..L-1."""
    L = x.shape[0]
    half = head_dim // 2
    v = x.reshape(L, n_heads, head_dim)
    x1, x2 = v[..., :half], v[..., half:]
    c, s = cos[:L, None, :half], sin[:L, None, :half]
    o1 = x1 * c - x2 * s
    o2 = x2 * c + x1 * s
    return np.concatenate([o1, o2], -1).reshape(L, n_heads * head_dim).astype(F32)


def attention(q, k, v, n_heads, n_kv_heads, head_dim, causal):
    """libffwd/attn.c:50-458: softmax(q k^T * 1/sqrt(d)) v, kv head = h / (nh/nkv)."""
    L = q.shape[0]
    scale = F32(1.0) / np.sqrt(F32(head_dim))
    rep = n_heads // n_kv_heads
    qh = q.reshape(L, n_heads, head_dim).transpose(1, 0, 2)
    kh = k.reshape(L, n_kv_heads, head_dim).transpose(1, 0, 2)
    vh = v.reshape(L, n_kv_heads, head_dim).transpose(1, 0, 2)
    kh = np.repeat(kh, rep, axis=0)
    vh = np.repeat(vh, rep, axis=0)
    s = np.matmul(qh, kh.transpose(0, 2, 1)) * scale
    if causal:
        s = np.where(np.tril(np.ones((L, L), dtype=bool))[None], s, F32(-np.inf))
    m = s.max(-1, keepdims=True)
    p = np.exp(s - m)
    p = p / p.sum(-1, keepdims=True, dtype=F32)
    o = np.matmul(p.astype(F32), vh)
    return o.transpose(1, 0, 2).reshape(L, n_heads * head_dim).astype(F32)


def silu_mul(g, u):
    """libffwd/act.c:30-52: (g / (1 + exp(-g))) * u."""
    return ((g / (F32(1.0) + np.exp(-g))) * u).astype(F32)


def gelu(x, act):
    """libffwd/act.c:54-70: erf GeLU or the tanh approximation."""
    if act == "tanh":
        inner = F32(0.79788456080286536) * (x + F32(0.044715) * x * x * x)
        return (F32(0.5) * x * (F32(1.0) + np.tanh(inner))).astype(F32)
    from scipy.special import erf
    return (F32(0.5) * x * (F32(1.0) + erf(x * F32(0.70710678118654752)).astype(F32))).astype(F32)


def l2_normalize(v):
    """libffwd/vec.c:7-22."""
    n = np.sum(v * v, dtype=F32)
    if not (n > 0) or not np.isfinite(n):
        raise ValueError("zero or non-finite embedding norm")
    return (v * (F32(1.0) / np.sqrt(n))).astype(F32)


# --------------------------------------------------------------------------- model


class OracleModel:
    """Numpy model over a reference-format model directory."""

    def __init__(self, model_dir: str):
        self.cfg = parse_config(model_dir)
        self.t = load_tensors(model_dir)
        if self.cfg["family"] == "bert":
            self.p = next(p for p in ("", "bert.", "roberta.")
                          if p + "embeddings.word_embeddings.weight" in self.t)
        else:
            self.p = "model." if "model.embed_tokens.weight" in self.t else ""

    # forward.c:166-285
    def _forward_qwen(self, seqs):
        c, t, p = self.cfg, self.t, self.p
        ids = np.concatenate(seqs)
        if ids.min() < 0 or ids.max() >= c["vocab"]:
            raise ValueError("invalid token id")
        x = t[p + "embed_tokens.weight"][ids].astype(F32)
        lens = [len(s) for s in seqs]
        offs = np.concatenate([[0], np.cumsum(lens)])
        cos, sin = rope_tables(max(lens), c["head_dim"], c["rope_theta"])
        H, hd, nh, nkv = c["hidden"], c["head_dim"], c["n_heads"], c["n_kv_heads"]
        for i in range(c["n_layers"]):
            lp = f"{p}layers.{i}."
            xn = rms_norm(x, t[lp + "input_layernorm.weight"], c["rms_eps"])
            q = xn @ t[lp + "self_attn.q_proj.weight"].T
            k = xn @ t[lp + "self_attn.k_proj.weight"].T
            v = xn @ t[lp + "self_attn.v_proj.weight"].T
            if c["qkv_bias"]:
                q = q + t[lp + "self_attn.q_proj.bias"]
                k = k + t[lp + "self_attn.k_proj.bias"]
                v = v + t[lp + "self_attn.v_proj.bias"]
            if c["qk_norm"]:
                L = q.shape[0]
                q = rms_norm(q.reshape(L, nh, hd), t[lp + "self_attn.q_norm.weight"],
                             c["rms_eps"]).reshape(L, nh * hd)
                k = rms_norm(k.reshape(L, nkv, hd), t[lp + "self_attn.k_norm.weight"],
                             c["rms_eps"]).reshape(L, nkv * hd)
            att = np.empty((x.shape[0], nh * hd), dtype=F32)
            for b in range(len(seqs)):
                s, e = offs[b], offs[b + 1]
                qb = apply_rope_neox(q[s:e], cos, sin, nh, hd)
                kb = apply_rope_neox(k[s:e], cos, sin, nkv, hd)
                att[s:e] = attention(qb, kb, v[s:e], nh, nkv, hd, c["causal"])
            x = (x + att @ t[lp + "self_attn.o_proj.weight"].T).astype(F32)
            xn = rms_norm(x, t[lp + "post_attention_layernorm.weight"], c["rms_eps"])
            g = xn @ t[lp + "mlp.gate_proj.weight"].T
            u = xn @ t[lp + "mlp.up_proj.weight"].T
            x = (x + silu_mul(g, u) @ t[lp + "mlp.down_proj.weight"].T).astype(F32)
        return x, offs

    # forward.c:314-404
    def _forward_bert(self, seqs):
        c, t, p = self.cfg, self.t, self.p
        lens = [len(s) for s in seqs]
        if max(lens) > c["max_pos"] - c["pos_offset"]:
            raise ValueError("sequence exceeds max_position_embeddings")
        ids = np.concatenate(seqs)
        if ids.min() < 0 or ids.max() >= c["vocab"]:
            raise ValueError("invalid token id")
        offs = np.concatenate([[0], np.cumsum(lens)])
        pos = np.concatenate([np.arange(n) + c["pos_offset"] for n in lens])
        x = (t[p + "embeddings.word_embeddings.weight"][ids]
             + t[p + "embeddings.position_embeddings.weight"][pos]
             + t[p + "embeddings.token_type_embeddings.weight"][0]).astype(F32)
        eps = c["ln_eps"]
        x = layer_norm(x, t[p + "embeddings.LayerNorm.weight"], t[p + "embeddings.LayerNorm.bias"], eps)
        nh, hd = c["n_heads"], c["head_dim"]
        for i in range(c["n_layers"]):
            lp = f"{p}encoder.layer.{i}."
            q = x @ t[lp + "attention.self.query.weight"].T + t[lp + "attention.self.query.bias"]
            k = x @ t[lp + "attention.self.key.weight"].T + t[lp + "attention.self.key.bias"]
            v = x @ t[lp + "attention.self.value.weight"].T + t[lp + "attention.self.value.bias"]
            att = np.empty_like(q)
            for b in range(len(seqs)):
                s, e = offs[b], offs[b + 1]
                att[s:e] = attention(q[s:e], k[s:e], v[s:e], nh, nh, hd, c["causal"])
            proj = att @ t[lp + "attention.output.dense.weight"].T + t[lp + "attention.output.dense.bias"]
            x = layer_norm(x + proj, t[lp + "attention.output.LayerNorm.weight"],
                           t[lp + "attention.output.LayerNorm.bias"], eps)
            up = gelu(x @ t[lp + "intermediate.dense.weight"].T + t[lp + "intermediate.dense.bias"],
                      c["act"])
            dn = up @ t[lp + "output.dense.weight"].T + t[lp + "output.dense.bias"]
            x = layer_norm(x + dn, t[lp + "output.LayerNorm.weight"], t[lp + "output.LayerNorm.bias"], eps)
        return x, offs

    def hidden_states(self, seqs):
        seqs = [np.asarray(s, dtype=np.int64) for s in seqs]
        if self.cfg["family"] == "bert":
            return self._forward_bert(seqs)
        return self._forward_qwen(seqs)

    # forward.c:406-466
    def encode_batch(self, seqs) -> np.ndarray:
        if not seqs or any(len(s) <= 0 for s in seqs):
            raise ValueError("empty input")
        c, t = self.cfg, self.t
        x, offs = self.hidden_states(seqs)
        norm_w = t.get(self.p + "norm.weight") if c["family"] != "bert" else None
        out = np.empty((len(seqs), c["hidden"]), dtype=F32)
        for b in range(len(seqs)):
            s, e = offs[b], offs[b + 1]
            if c["pooling"] in ("last", "cls"):
                row = x[s if c["pooling"] == "cls" else e - 1]
                emb = rms_norm(row, norm_w, c["rms_eps"]) if norm_w is not None else row.copy()
            else:
                rows = x[s:e]
                if norm_w is not None:
                    rows = rms_norm(rows, norm_w, c["rms_eps"])
                emb = (np.sum(rows, 0, dtype=F32) * (F32(1.0) / F32(e - s))).astype(F32)
            out[b] = l2_normalize(emb) if c["normalize"] else emb
        return out

    # forward.c:492-589 (ffwd_pool_spans, ffwd_model_encode_spans_batch): the
    # packed forward with the decoder's final RMSNorm applied to every row
    # (apply_final_norm = 1), then per span the f32 mean of its rows, in span
    # order; no L2 normalisation.
    def encode_spans_batch(self, docs, spans) -> np.ndarray:
        c, t = self.cfg, self.t
        for doc, sp in zip(docs, spans):
            if len(doc) <= 0 or not sp:
                raise ValueError("empty document or span list")
            for a, n in sp:
                if a < 0 or n <= 0 or a > len(doc) or n > len(doc) - a:
                    raise ValueError("span outside its document")
        x, offs = self.hidden_states(docs)
        if c["family"] != "bert":
            x = rms_norm(x, t[self.p + "norm.weight"], c["rms_eps"])
        out = []
        for b, sp in enumerate(spans):
            for a, n in sp:
                rows = x[offs[b] + a:offs[b] + a + n]
                out.append((np.sum(rows, 0, dtype=F32) * (F32(1.0) / F32(n))).astype(F32))
        return np.stack(out)


# --------------------------------------------------------------------------- late interaction


class OracleLate:
    """Numpy late-interaction model: the base model's final hidden states (the
    decoder's after its final RMSNorm, forward.c:470-490 with
    apply_final_norm = 1), the 1_Dense projection (late.c:41-86, no bias), L2 per
    vector (late_blas.c:57-85) and MaxSim (late.c:126-219).  The reference's CPU
    path only runs decoder base models (ffwd_model_forward_into); for BERT
    bases this restates the same steps over the BERT forward."""

    def __init__(self, model_dir: str):
        self.base = OracleModel(model_dir)
        self.w = load_tensors(os.path.join(model_dir, "1_Dense"))["linear.weight"]
        self.dim = int(self.w.shape[0])

    def _vectors(self, seqs, rows, normalize):
        x, _ = self.base.hidden_states(seqs)
        c, t = self.base.cfg, self.base.t
        if c["family"] != "bert":
            x = rms_norm(x, t[self.base.p + "norm.weight"], c["rms_eps"])
        v = (x[np.asarray(rows, np.int64)] @ self.w.T).astype(F32)
        if normalize:
            v = np.stack([l2_normalize(r) for r in v]) if len(v) else v
        return v

    def encode_tokens(self, ids, normalize=True):
        return self._vectors([ids], np.arange(len(ids)), normalize)

    def encode_docs(self, docs, keeps, normalize=True):
        starts = np.concatenate([[0], np.cumsum([len(d) for d in docs])])
        rows = np.concatenate([starts[i] + np.asarray(k, np.int64) for i, k in enumerate(keeps)])
        offs = np.concatenate([[0], np.cumsum([len(k) for k in keeps])]).astype(np.int32)
        return self._vectors(docs, rows, normalize), offs

    @staticmethod
    def maxsim_batch(q, docs, offs):
        out = np.zeros(len(offs) - 1, dtype=F32)
        for i in range(len(offs) - 1):
            sim = q @ docs[offs[i]:offs[i + 1]].T
            out[i] = np.sum(sim.max(axis=1), dtype=F32)
        return out

    def rerank(self, query, query_n_keep, docs, keeps):
        """ffwd_rerank (backend_cuda.c:132-156)."""
        qv = self.encode_tokens(query, True)[:query_n_keep]
        dv, offs = self.encode_docs(docs, keeps, True)
        return self.maxsim_batch(qv, dv, offs)



# --------------------------------------------------------------------------- output encodings


def quantize_int8_tanh(x):
    """tools/server/encode.c:20-27: lrintf(tanhf(x) * 127) clamped to [-128, 127]."""
    v = np.rint(np.tanh(np.asarray(x, F32)).astype(F32) * F32(127.0))
    return np.clip(v, -128, 127).astype(np.int8)


def binary_bits(x):
    """tools/server/encode.c:42-51: bit i = (x[i] >= 0), bits[i >> 3] |= 1 << (i & 7)."""
    return np.packbits(np.asarray(x) >= 0, axis=-1, bitorder="little")


def truncate_renormalize(emb, dims):
    """tools/server/encode.c:107-122: first dims values, then ffwd_l2_normalize."""
    return np.stack([l2_normalize(r[:dims].astype(F32)) for r in np.atleast_2d(emb)])
