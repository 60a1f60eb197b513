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


# ---- archive workload: windows of synthetic order-3 Markov text -------------------

ARCHIVE_SEED_BASE = 0x0A4C0000  # window i is sample ARCHIVE_SEED_BASE + i of the Markov source
ARCHIVE_WINDOW = 10240          # bytes per window
VOCAB_TRAIN_SEED = 12345        # the sample the archive vocabulary is learned from
VOCAB_TRAIN_BYTES = 1_000_000
VOCAB_MAX_LEN = 5               # bytes per vocabulary entry: about 3.6 bytes per token on this source


def archive_windows(n: int, first: int = 0, size: int = ARCHIVE_WINDOW):
    """Windows first .. first + n - 1 of the archive workload (bytes each)."""
    from redukt_b200.archive import markov_text
    return [markov_text(ARCHIVE_SEED_BASE + first + i, size) for i in range(n)]


def archive_tokenizer(vocab: int, cache_dir: str = None):
    """The workload's byte-level vocabulary (learned once from a fixed sample; cached as .npz)."""
    import os
    from redukt_b200.archive import Tokenizer, markov_text
    path = os.path.join(cache_dir, f"archive_vocab_{vocab}.npz") if cache_dir else None
    if path and os.path.exists(path):
        z = np.load(path)
        blob, offs = z["blob"].tobytes(), z["offs"]
        return Tokenizer([blob[offs[i]:offs[i + 1]] for i in range(vocab)])
    tok = Tokenizer.learn(markov_text(VOCAB_TRAIN_SEED, VOCAB_TRAIN_BYTES), vocab, per_round=2048,
                          max_len=VOCAB_MAX_LEN)
    if path:
        os.makedirs(cache_dir, exist_ok=True)
        offs = np.zeros(vocab + 1, np.uint64)
        offs[1:] = np.cumsum([len(t) for t in tok.tokens])
        np.savez(path, blob=np.frombuffer(b"".join(tok.tokens), np.uint8), offs=offs)
    return tok
