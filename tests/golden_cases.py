"""Loads a golden fixture and regenerates its .rbin from the recorded recipe (checked by sha256)."""
import hashlib
import os

import numpy as np

from redukt_b200 import rbin

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")
NAMES = ("reftest", "gauss_small", "gauss_ln_untied")


def sha256(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def load(name, model_dir):
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    dims = rbin.MambaDims(vocab=int(z["vocab"]), d_model=int(z["d_model"]), n_layer=int(z["n_layer"]))
    path = os.path.join(model_dir, "golden_" + name + ".rbin")
    kind = str(z["kind"])
    if kind == "reference_test":
        rbin.ensure_model(path, dims, kind="reference_test")
    else:
        rbin.ensure_model(path, dims, kind="gaussian", seed=int(z["seed"]), flags=int(z["flags"]))
    assert sha256(path) == str(z["sha256"]), f"{name}: regenerated model differs from the fixture's"
    return path, z["tokens"], z["logits"]
