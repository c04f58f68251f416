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
