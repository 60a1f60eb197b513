"""The native host side of an archive (libredukt_archive.so) on the CPU.

- CRC-32: the reference's known vectors (src/domain/crc32.rs tests: "123456789" -> 0xCBF43926,
  the empty string -> 0) and incremental updates.
- Range coder: byte for byte the same output as the Python restatement in oracle/range_coder.py,
  which is pinned by the reference's own coder tests (tests/test_archive_roundtrip.py), on random
  interval sequences, and decodes back.
- Container: the RDKT v5 layout of a plugin archive (FORMAT-SPEC.md:182-226), round trip and the
  rejection of anything else.
- Workload: the Markov source is printable ASCII and seeded; the learned vocabulary tokenises it
  at a few bytes per token and detokenises it exactly.
"""
import numpy as np
import pytest

from oracle import range_coder as RC
from redukt_b200 import archive as A

TOTAL = 1 << 24


def test_crc32_known_vectors():
    assert A.crc32(b"123456789") == 0xCBF43926
    assert A.crc32(b"") == 0
    assert A.crc32(b"The quick brown fox jumps over the lazy dog") == 0x414FA339
    data = np.random.default_rng(0).integers(0, 256, 100003).astype(np.uint8).tobytes()
    import zlib
    assert A.crc32(data) == zlib.crc32(data)
    L = A.lib()
    st = 0xFFFFFFFF
    for i in range(0, len(data), 777):
        chunk = np.frombuffer(data[i:i + 777], np.uint8)
        st = L.rk_crc32_update(st, chunk.ctypes.data, len(chunk))
    assert st ^ 0xFFFFFFFF == zlib.crc32(data)


def _random_cdfs(rng, steps, alphabet):
    out = []
    for _ in range(steps):
        f = rng.integers(1, 2000, alphabet).astype(np.int64)
        f = np.maximum(1, (f * (TOTAL - alphabet) // f.sum())) + 1
        f[-1] += TOTAL - f.sum()
        c = np.concatenate([[0], np.cumsum(f)])
        assert c[-1] == TOTAL
        out.append(c)
    return out


@pytest.mark.parametrize("seed", range(4))
def test_native_coder_matches_restated_reference_coder(seed):
    rng = np.random.default_rng(seed)
    n, steps, alphabet = 5, 400, 300
    cdfs = [_random_cdfs(rng, steps, alphabet) for _ in range(n)]
    syms = rng.integers(0, alphabet, (n, steps))
    syms[:, ::7] = alphabet - 1  # the last symbol: the encoder's hi == total branch
    first = rng.integers(0, alphabet, n).astype(np.uint32)
    L = A.lib()
    cod = A.Coders(n)
    assert L.rk_enc_uniform(cod.h, n, None, first.ctypes.data, alphabet) == A.OK
    for t in range(steps):
        q = np.array([[syms[s, t], cdfs[s][t][syms[s, t]], cdfs[s][t][syms[s, t] + 1]] for s in range(n)], np.uint32)
        assert L.rk_enc_batch(cod.h, n, None, q.ctypes.data, TOTAL) == A.OK
    streams = []
    for s in range(n):
        size = L.rk_enc_finish(cod.h, s, None, 0)
        buf = np.empty(size, np.uint8)
        assert L.rk_enc_finish(cod.h, s, buf.ctypes.data, size) == size
        streams.append(buf.tobytes())
        # the restated reference coder on the same intervals
        enc = RC.RangeEncoder()
        uc, ut = RC.uniform(alphabet)
        enc.encode(uc[first[s]], uc[first[s] + 1], ut)
        for t in range(steps):
            enc.encode(int(cdfs[s][t][syms[s, t]]), int(cdfs[s][t][syms[s, t] + 1]), TOTAL)
        assert streams[-1] == enc.finish(), s
    # and back
    dec = A.Coders(n)
    for s in range(n):
        st = np.frombuffer(streams[s], np.uint8)
        assert L.rk_dec_start(dec.h, s, st.ctypes.data, len(st)) == A.OK
    got0 = np.empty(n, np.uint32)
    assert L.rk_dec_uniform(dec.h, n, None, alphabet, got0.ctypes.data) == A.OK
    assert np.array_equal(got0, first)
    for t in range(steps):
        cum = np.empty(n, np.uint32)
        assert L.rk_dec_freq_batch(dec.h, n, None, TOTAL, cum.ctypes.data) == A.OK
        q = np.empty((n, 3), np.uint32)
        for s in range(n):
            y = RC.lookup(cdfs[s][t], int(cum[s]))
            q[s] = (y, cdfs[s][t][y], cdfs[s][t][y + 1])
            assert y == syms[s, t]
        assert L.rk_dec_update_batch(dec.h, n, None, q.ctypes.data, TOTAL) == A.OK


def test_coder_rejects_impossible_intervals():
    L = A.lib()
    cod = A.Coders(1)
    q = np.array([[0, 5, 5]], np.uint32)  # empty interval
    assert L.rk_enc_batch(cod.h, 1, None, q.ctypes.data, TOTAL) == A.CORRUPT
    q = np.array([[0, 0, TOTAL + 1]], np.uint32)
    assert L.rk_enc_batch(cod.h, 1, None, q.ctypes.data, TOTAL) == A.CORRUPT
    s = np.array([7], np.uint32)
    assert L.rk_enc_batch(cod.h, 1, s.ctypes.data, q.ctypes.data, TOTAL) == A.INVALID


def test_container_layout_and_round_trip():
    hdr = A.Header(total_bytes=10240)
    buf = A.pack(hdr, b"\x01\x02\x03", 0xDEADBEEF)
    # MAGIC v5, TOTAL_BYTES, FLAGS (backbone byte follows), PROFILE (reset flag), RESET_LOG2, BACKBONE
    assert buf[:8] == b"RDKT\x05\x00\x00\x00"
    assert buf[8:12] == (10240).to_bytes(4, "little")
    assert buf[12] == 0x40 and buf[13] == 0x50 and buf[14] == 12 and buf[15] == 0x03
    assert len(buf) == 16 + 3 + 4 and buf[-4:] == (0xDEADBEEF).to_bytes(4, "little")
    h2, stream, crc = A.unpack(buf)
    assert (h2.total_bytes, h2.profile, h2.reset_log2, h2.backbone) == (10240, 0x10, 12, 3)
    assert stream == b"\x01\x02\x03" and crc == 0xDEADBEEF
    for bad in (b"RDKT\x04\x00\x00\x00" + buf[8:], buf[:12] + b"\x00" + buf[13:], buf[:10]):
        with pytest.raises(A.ArchiveError):
            A.unpack(bad)
    assert A.pack(A.Header(5, reset_log2=0), b"", 1)[13] == 0x10  # no RESET_LOG2 byte


def test_markov_text_is_seeded_printable_ascii():
    a, b = A.markov_text(7, 20000), A.markov_text(7, 20000)
    assert a == b and a != A.markov_text(8, 20000)
    arr = np.frombuffer(a, np.uint8)
    assert arr.min() >= 0x20 and arr.max() <= 0x7E
    assert len(set(a)) > 40  # letters of both cases, space, comma, full stop


def test_learned_vocabulary_tokenises_and_round_trips():
    train = A.markov_text(12345, 400_000)
    tok = A.Tokenizer.learn(train, vocab=4096, per_round=512, max_len=5)
    assert tok.vocab == 4096 and all(tok.tokens[i] == bytes([i]) for i in range(256))
    assert len(set(tok.tokens)) == 4096
    text = A.markov_text(99, 50_000)
    ids = tok.encode(text)
    assert tok.decode(ids) == text
    assert len(text) / len(ids) > 2.5  # multi-byte tokens are used
