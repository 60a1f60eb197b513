"""Seeded synthetic token streams standing in for the reference's benchmark inputs.

The reference measures on real text through the GPT-NeoX tokenizer, which is not available here;
the benchmark configurations instead draw token ids from a seeded Zipf(s) law over the vocabulary
ranks (rank r -> id r - 1), one seed per stream (seed_base + stream index).
"""
from __future__ import annotations

import numpy as np

ZIPF_SEED_BASE = 0x70C3E500


def zipf_cdf(vocab: int, s: float = 1.1) -> np.ndarray:
    w = np.arange(1, vocab + 1, dtype=np.float64) ** (-s)
    c = np.cumsum(w)
    return c / c[-1]


def zipf_tokens(n_streams: int, length: int, vocab: int = 50280, s: float = 1.1,
                seed_base: int = ZIPF_SEED_BASE) -> np.ndarray:
    """[n_streams, length] uint32 token ids, stream i drawn with seed seed_base + i."""
    cdf = zipf_cdf(vocab, s)
    out = np.empty((n_streams, length), np.uint32)
    for i in range(n_streams):
        u = np.random.Generator(np.random.PCG64(seed_base + i)).random(length)
        out[i] = np.minimum(np.searchsorted(cdf, u, side="right"), vocab - 1)
    return out


def uniform_tokens(n_streams: int, length: int, vocab: int, seed_base: int = ZIPF_SEED_BASE) -> np.ndarray:
    out = np.empty((n_streams, length), np.uint32)
    for i in range(n_streams):
        out[i] = np.random.Generator(np.random.PCG64(seed_base + i)).integers(0, vocab, length)
    return out
