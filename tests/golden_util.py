"""Loading the golden fixtures (test code only)."""

import glob
import json
import os

import numpy as np

from ffwd_b200 import synth

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def fixtures():
    return sorted(os.path.splitext(os.path.basename(p))[0]
                  for p in glob.glob(os.path.join(GOLDEN, "*.npz")))


def load(name, model_root):
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    spec = synth.ModelSpec(**json.loads(str(z["spec"])))
    d = synth.ensure_model(spec, model_root)
    lens = z["lens"]
    offs = np.concatenate([[0], np.cumsum(lens)])
    ids = z["ids"]
    seqs = [ids[offs[i]:offs[i + 1]] for i in range(len(lens))]
    return spec, d, seqs, z["expected"]


def span_fixtures():
    return sorted(os.path.splitext(os.path.basename(p))[0]
                  for p in glob.glob(os.path.join(GOLDEN, "spans", "*.npz")))


def load_spans(name, model_root):
    """(spec, model dir, documents, spans per document, expected rows) of a
    contextual-span fixture made by the reference's ffwd_model_encode_spans_batch."""
    z = np.load(os.path.join(GOLDEN, "spans", name + ".npz"))
    spec = synth.ModelSpec(**json.loads(str(z["spec"])))
    d = synth.ensure_model(spec, model_root)
    lens, ns = z["lens"], z["n_spans"]
    offs = np.concatenate([[0], np.cumsum(lens)])
    soffs = np.concatenate([[0], np.cumsum(ns)])
    docs = [z["ids"][offs[i]:offs[i + 1]] for i in range(len(lens))]
    spans = [[(int(a), int(n)) for a, n in zip(z["span_start"][soffs[i]:soffs[i + 1]],
                                               z["span_len"][soffs[i]:soffs[i + 1]])]
             for i in range(len(lens))]
    return spec, d, docs, spans, z["expected"]
