"""Generates the golden fixtures in this directory from the reference's own NumPy Mamba.

`RefMamba` is the float32 NumPy Mamba-1 step of the reference's GPU validation script
(notebooks/redukt-gpu-cuda-test.py:150-207 in the redukt tree); it is imported from the mounted
reference tree, so this script runs only where that tree exists.  Each fixture holds the model
recipe and sha256 (the .rbin is regenerated from its seed by redukt_b200.rbin), the token
sequence and RefMamba's logits; tests compare the C oracle and the GPU engine against them.

    python tests/golden/make_golden.py [/path/to/redukt]
"""
import hashlib
import importlib.util
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from redukt_b200 import rbin  # noqa: E402

CASES = {
    # name: (dims, kind, seed, flags, steps)
    "reftest": (rbin.REFERENCE_TEST_DIMS, "reference_test", 0, 0, 10),
    "gauss_small": (rbin.MambaDims(vocab=2000, d_model=128, n_layer=3), "gaussian", 12345, 0, 10),
    "gauss_ln_untied": (rbin.MambaDims(vocab=512, d_model=64, n_layer=2), "gaussian", 777,
                        rbin.FLAG_NORM_BIAS | rbin.FLAG_UNTIED_HEAD, 8),
}


def load_refmamba(ref_root):
    path = os.path.join(ref_root, "notebooks", "redukt-gpu-cuda-test.py")
    spec = importlib.util.spec_from_file_location("redukt_gpu_cuda_test", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)  # the script's main() is behind `if __name__ == "__main__"`
    return mod.RefMamba


def build_case(name, d, tmp):
    dims, kind, seed, flags, steps = CASES[name]
    path = os.path.join(tmp, name + ".rbin")
    if kind == "reference_test":
        rbin.ensure_model(path, dims, kind="reference_test")
    else:
        rbin.ensure_model(path, dims, kind="gaussian", seed=seed, flags=flags)
    return path


def sha256(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def main(ref_root=None):
    """ref_root: the redukt source tree (default: $REDUKT_REF_ROOT, else `reference` beside the repo)."""
    if ref_root is None:
        sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
        from oracle.oracle import reference_root
        ref_root = reference_root()
        if ref_root is None:
            raise SystemExit("the redukt source tree was not found: set REDUKT_REF_ROOT")
    RefMamba = load_refmamba(ref_root)
    tmp = tempfile.mkdtemp()
    for name, (dims, kind, seed, flags, steps) in CASES.items():
        path = build_case(name, dims, tmp)
        ref = RefMamba(path)
        toks = np.array([(t * 977 + 7) % dims.vocab for t in range(steps)], np.uint32)
        logits = np.stack([ref.step(int(t)).astype(np.float32) for t in toks])
        np.savez_compressed(os.path.join(HERE, name + ".npz"), tokens=toks, logits=logits,
                            sha256=np.array(sha256(path)), kind=np.array(kind), seed=np.array(seed),
                            flags=np.array(flags), vocab=np.array(dims.vocab), d_model=np.array(dims.d_model),
                            n_layer=np.array(dims.n_layer))
        print(name, logits.shape, sha256(path)[:16])


if __name__ == "__main__":
    main(*sys.argv[1:])
