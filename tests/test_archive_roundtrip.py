"""Archive round trips: engine logits -> device CDF -> the reference's range coder -> bytes -> back.

An archive is decodable only if the decoder rebuilds, token by token, exactly the frequency table
the encoder coded with.  The reference codes each stream with Cdf::uniform at position 0 and then
with the CDF of the previous forward's logits (src/application/lockstep.rs:297-337; the CM
ensemble that the reference mixes into those logits stays on the host and is not part of this
engine).  These tests run that loop with the engine's lockstep step and the device CDF
(redukt_b200_cdf, symbol queries when encoding, cumulative-frequency lookups when decoding) and the
reference's range coder restated in oracle/range_coder.py.

CPU tests pin the range-coder restatement with the reference's own coder tests
(src/domain/coder.rs:301-450).  GPU tests:
- Mamba-1: encode and decode on the engine give back every token;
- RWKV-7 (W8A8, whose logits are bit-identical to the oracle's): the archive bytes equal those of a
  pure-CPU pipeline (oracle forward, oracle CDF, same coder), and decode gives back every token.
"""
import os

import numpy as np
import pytest

from oracle import oracle as O
from oracle import range_coder as RC

TOTAL = 1 << 24


def _from_probs(probs):
    return [int(v) for v in O.cdf_from_probs(np.asarray(probs, dtype=np.float32))]


def _encode(symbols, cdfs):
    enc = RC.RangeEncoder()
    for s, (c, total) in zip(symbols, cdfs):
        enc.encode(c[s], c[s + 1], total)
    return enc.finish()


def _decode(data, cdfs):
    dec = RC.RangeDecoder(data)
    out = []
    for c, total in cdfs:
        s = RC.lookup(c, dec.get_freq(total))
        dec.update(c[s], c[s + 1], total)
        out.append(s)
    return out


# ----------------------------------------------------------------------------------------------
# CPU: the reference's coder tests (coder.rs:301-450) on the restatement
# ----------------------------------------------------------------------------------------------

def test_coder_roundtrip_uniform():
    c = RC.uniform(256)
    syms = [i % 256 for i in range(1000)]
    assert _decode(_encode(syms, [c] * 1000), [c] * 1000) == syms


def _normalised(p):
    p = np.asarray(p, dtype=np.float32)
    s = np.float32(0)
    for v in p:            # f32 sequential sum, as `probs.iter().sum()` on f32
        s = np.float32(s + v)
    return p / s


def test_coder_roundtrip_skewed():
    p = np.full(100, 0.001, np.float32)
    p[0] = 0.90
    c = (_from_probs(_normalised(p)), TOTAL)
    syms = [0, 0, 0, 1, 0, 0, 50, 0, 99, 0, 0, 0, 42, 0]
    assert _decode(_encode(syms, [c] * len(syms)), [c] * len(syms)) == syms


def test_coder_roundtrip_large_alphabet():
    p = np.full(65536, 1e-8, np.float32)
    p[0], p[1], p[2] = 0.3, 0.2, 0.1
    p[3:100] = 0.004
    c = (_from_probs(_normalised(p)), TOTAL)
    syms = [0, 1, 2, 50, 1000, 65535, 0, 0, 32768, 2]
    assert _decode(_encode(syms, [c] * len(syms)), [c] * len(syms)) == syms


def test_coder_roundtrip_varying_distributions():
    syms = [10, 200, 50, 100, 0, 255, 128]
    cdfs = []
    for s in syms:
        p = np.full(256, 0.001, np.float32)
        p[s], p[(s + 1) % 256] = 0.5, 0.2
        cdfs.append((_from_probs(_normalised(p)), TOTAL))
    assert _decode(_encode(syms, cdfs), cdfs) == syms


def test_coder_compression_efficiency():
    p = np.full(256, 0.0001, np.float32)
    p[0], p[1], p[2] = 0.5, 0.3, 0.1
    c = (_from_probs(_normalised(p)), TOTAL)
    data = _encode([0] * 10000, [c] * 10000)
    ratio = len(data) * 8.0 / (10000 * 1.0)   # -log2(0.5) bits per symbol
    assert 0.95 < ratio < 1.05


def test_coder_empty_stream_decodes_without_error():
    c, total = RC.uniform(256)
    dec = RC.RangeDecoder(b"")
    s = RC.lookup(c, dec.get_freq(total))
    assert 0 <= s < 256


# ----------------------------------------------------------------------------------------------
# GPU: archive round trips through the engine and the device CDF
# ----------------------------------------------------------------------------------------------

def _engine_encode(b, lib, windows):
    """Lockstep encode of n windows: position 0 uniform, then the CDF of the previous step's logits
    (symbol queries on the device)."""
    n, T = windows.shape
    V = b.vocab_size
    cu = RC.uniform(V)
    encs = [RC.RangeEncoder() for _ in range(n)]
    for r in range(n):
        s = int(windows[r, 0])
        encs[r].encode(cu[0][s], cu[0][s + 1], cu[1])
    slots = list(range(n))
    b.batch_reset(slots)
    for t in range(1, T):
        logits = b.forward_batch(slots, windows[:, t - 1].tolist())
        _, q = lib.cdf(logits, symbols=windows[:, t].astype(np.uint32), want_cdf=False)
        for r in range(n):
            assert q[r, 0] == windows[r, t]
            encs[r].encode(int(q[r, 1]), int(q[r, 2]), TOTAL)
    return [e.finish() for e in encs]


def _engine_decode(b, lib, archives, T):
    n = len(archives)
    V = b.vocab_size
    cu = RC.uniform(V)
    decs = [RC.RangeDecoder(a) for a in archives]
    out = np.zeros((n, T), dtype=np.int64)
    for r in range(n):
        s = RC.lookup(cu[0], decs[r].get_freq(cu[1]))
        decs[r].update(cu[0][s], cu[0][s + 1], cu[1])
        out[r, 0] = s
    slots = list(range(n))
    b.batch_reset(slots)
    for t in range(1, T):
        logits = b.forward_batch(slots, out[:, t - 1].tolist())
        cum = np.array([d.get_freq(TOTAL) for d in decs], dtype=np.uint32)
        _, q = lib.cdf(logits, cum_freqs=cum, want_cdf=False)
        for r in range(n):
            assert q[r, 0] < V, f"stream {r} step {t}: cum {cum[r]} found no symbol"
            decs[r].update(int(q[r, 1]), int(q[r, 2]), TOTAL)
            out[r, t] = q[r, 0]
    return out


def _fused_encode(b, windows):
    """_engine_encode through redukt_b200_forward_batch_cdf: the step and the CDF on the device,
    12 bytes per stream back."""
    n, T = windows.shape
    cu = RC.uniform(b.vocab_size)
    encs = [RC.RangeEncoder() for _ in range(n)]
    for r in range(n):
        s = int(windows[r, 0])
        encs[r].encode(cu[0][s], cu[0][s + 1], cu[1])
    slots = list(range(n))
    b.batch_reset(slots)
    for t in range(1, T):
        q, _ = b.forward_batch_cdf(slots, windows[:, t - 1], symbols=windows[:, t])
        for r in range(n):
            encs[r].encode(int(q[r, 1]), int(q[r, 2]), TOTAL)
    return [e.finish() for e in encs]


def _fused_decode(b, archives, T):
    n = len(archives)
    cu = RC.uniform(b.vocab_size)
    decs = [RC.RangeDecoder(a) for a in archives]
    out = np.zeros((n, T), dtype=np.int64)
    for r in range(n):
        s = RC.lookup(cu[0], decs[r].get_freq(cu[1]))
        decs[r].update(cu[0][s], cu[0][s + 1], cu[1])
        out[r, 0] = s
    slots = list(range(n))
    b.batch_reset(slots)
    for t in range(1, T):
        cum = [d.get_freq(TOTAL) for d in decs]
        q, _ = b.forward_batch_cdf(slots, out[:, t - 1], cum_freqs=cum)
        for r in range(n):
            decs[r].update(int(q[r, 1]), int(q[r, 2]), TOTAL)
            out[r, t] = q[r, 0]
    return out


def _zipf_windows(n, T, vocab, seed):
    rng = np.random.default_rng(seed)
    ranks = rng.zipf(1.1, size=(n, T))
    return ((ranks - 1) % vocab).astype(np.int64)


@pytest.mark.gpu
def test_mamba_archive_roundtrip(small_gauss_rbin):
    from conftest import shared_backend
    from redukt_b200.plugin import PluginLibrary

    b = shared_backend(small_gauss_rbin)
    lib = PluginLibrary()
    n, T = 4, 40
    b.batch_init(n)
    w = _zipf_windows(n, T, b.vocab_size, 11)
    archives = _engine_encode(b, lib, w)
    assert all(len(a) > 0 for a in archives)
    back = _engine_decode(b, lib, archives, T)
    np.testing.assert_array_equal(back, w)
    # the same loop through the one-call step + CDF entry point: same bytes, same tokens back
    assert _fused_encode(b, w) == archives
    np.testing.assert_array_equal(_fused_decode(b, archives, T), w)


@pytest.mark.gpu
def test_forward_batch_cdf_matches_step_then_cdf(small_gauss_rbin):
    from conftest import shared_backend
    from redukt_b200.plugin import PluginError, PluginLibrary

    b = shared_backend(small_gauss_rbin)
    lib = PluginLibrary()
    n = 5
    b.batch_init(n)
    w = _zipf_windows(n, 3, b.vocab_size, 5)
    slots = [4, 0, 3, 1, 2]
    b.batch_reset()
    logits = b.forward_batch(slots, w[:, 0].tolist())
    want, wq = lib.cdf(logits, symbols=w[:, 1].astype(np.uint32))
    b.batch_reset()
    q, c = b.forward_batch_cdf(slots, w[:, 0], symbols=w[:, 1], want_cdf=True)
    np.testing.assert_array_equal(c, want)
    np.testing.assert_array_equal(q, wq)
    with pytest.raises(PluginError):      # duplicate slot: rejected before any launch
        b.forward_batch_cdf([0, 0], [1, 2], symbols=[1, 2])
    with pytest.raises(PluginError):      # token outside the vocabulary
        b.forward_batch_cdf([0], [b.vocab_size], symbols=[1])


@pytest.mark.gpu
def test_rwkv7_archive_bytes_match_cpu_pipeline(tmp_path):
    from oracle import rwkv7 as W
    from redukt_b200 import rwkv7_rbin as R
    from conftest import shared_backend
    from redukt_b200.plugin import PluginLibrary

    path = R.ensure_model(os.path.join(str(tmp_path), "rwkv7_small.rbin"), R.RWKV7_TEST_DIMS)
    n, T = 3, 24
    w = R.byte_tokens(n, T).astype(np.int64)
    # CPU pipeline: oracle forward, oracle CDF, the same coder
    m = W.Model(path)
    states = [W.State(m) for _ in range(n)]
    cpu = [RC.RangeEncoder() for _ in range(n)]
    for t in range(1, T):
        logits = W.forward_multi(m, states, w[:, t - 1])
        c = O.cdf_from_logits(logits)
        if t == 1:   # position 0 is coded with the uniform CDF before any forward
            cu, ctot = RC.uniform(logits.shape[1])
            for r in range(n):
                s0 = int(w[r, 0])
                cpu[r].encode(cu[s0], cu[s0 + 1], ctot)
        for r in range(n):
            s = int(w[r, t])
            cpu[r].encode(int(c[r, s]), int(c[r, s + 1]), TOTAL)
    cpu_bytes = [e.finish() for e in cpu]

    b = shared_backend(path)
    lib = PluginLibrary()
    b.batch_init(n)
    gpu_bytes = _engine_encode(b, lib, w)
    assert gpu_bytes == cpu_bytes
    back = _engine_decode(b, lib, gpu_bytes, T)
    np.testing.assert_array_equal(back, w)
    assert _fused_encode(b, w) == cpu_bytes


# ----------------------------------------------------------------------------------------------
# GPU: the configs[4] workload through the native host side (libredukt_archive.so)
# ----------------------------------------------------------------------------------------------

@pytest.mark.gpu
def test_markov_windows_round_trip_with_crc(mamba130m_rbin, model_dir):
    """16 windows of 10 KB of the synthetic order-3 Markov text, Mamba-130M Q8 with the reset every
    4096 forwards: compressed in lockstep (device step + CDF, native range coder, RDKT v5 with
    CRC-32), decompressed in lockstep on the GPU, byte-equal.  A byte flipped inside one window's
    coded stream is caught: that window fails its size or CRC-32 check, the other windows of the
    batch still decode exactly."""
    from conftest import q8, shared_backend
    from redukt_b200 import archive as A
    from redukt_b200.workload import archive_tokenizer, archive_windows

    b = shared_backend(q8(mamba130m_rbin))
    tok = archive_tokenizer(b.vocab_size, model_dir)
    wins = archive_windows(16)
    b.batch_init(16)
    arcs = A.compress_windows(b, wins, tok)
    assert all(a[:8] == b"RDKT\x05\x00\x00\x00" for a in arcs)
    for a, w in zip(arcs, wins):
        h, stream, crc = A.unpack(a)
        assert h.total_bytes == len(w) and crc == A.crc32(w) and h.reset_log2 == 12
    back = A.decompress_windows(b, arcs, tok)
    assert back == wins
    # the same windows again: the archive is deterministic
    assert A.compress_windows(b, wins, tok) == arcs
    # corrupt one byte in the middle of window 5's coded stream
    bad = bytearray(arcs[5])
    bad[16 + len(bad) // 3] ^= 0x5A
    arcs2 = list(arcs)
    arcs2[5] = bytes(bad)
    back2 = A.decompress_windows(b, arcs2, tok)
    assert isinstance(back2[5], A.ArchiveError)
    assert "CRC-32 mismatch" in str(back2[5]) or "size mismatch" in str(back2[5]) or "corrupt" in str(back2[5])
    assert [x for i, x in enumerate(back2) if i != 5] == [w for i, w in enumerate(wins) if i != 5]
