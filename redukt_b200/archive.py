"""Lockstep window archives through the device CDF and the native range coder.

The reference compresses each window in lockstep with other windows
(src/application/lockstep.rs:297-442): a stream's first token is coded with Cdf::uniform, every
later token with the CDF of the backbone's previous step, and the window becomes one RDKT v5 file
(header, coded stream, CRC-32 of the window's bytes).  Here the backbone step and the CDF run on
the device (redukt_b200_forward_batch_cdf returns only the coder's {symbol, low, high} per
stream), and the range coder, CRC-32 and container run natively (libredukt_archive.so).  The
reference's context-mixing ensemble is not part of this engine, so these archives code the
backbone's own distribution; they are decodable by this engine (the same plugin build) only,
like the reference's plugin archives (docs/api/PLUGIN-FFI-V2.md:102-108).

Decompression replays the same steps: the decoder's cumulative frequency goes to the device, which
looks the symbol up in the step's CDF; the window is complete when its tokens give back TOTAL_BYTES
bytes, and it is accepted only if their CRC-32 equals the stored one.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from typing import List, Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libredukt_archive.so")
TOTAL = 1 << 24          # CDF total of the device coder queries (coder.rs TOP)
PLUGIN_BACKBONE = 0x03   # BACKBONE_ID of the GPU plugin (FORMAT-SPEC.md, backbone table)
PLUGIN_PROFILE = 0x10    # quant F32 (the reference records F32 for plugin archives), numeric contract 1
RESET_LOG2 = 12          # 4096 forwards between state resets (the reference's default)

OK, INVALID, CORRUPT, FORMAT = 0, 1, 2, 3


class ArchiveError(RuntimeError):
    pass


class _Header(ctypes.Structure):
    _fields_ = [("total_bytes", ctypes.c_uint32), ("profile", ctypes.c_uint8), ("reset_log2", ctypes.c_uint8),
                ("backbone", ctypes.c_uint8)]


_lib: Optional[ctypes.CDLL] = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            raise ArchiveError(f"{LIB} is missing: run `python -m redukt_b200.build`")
        L = ctypes.CDLL(LIB)
        u8p, u32p, vp, sz = ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t
        u32, i32, i64 = ctypes.c_uint32, ctypes.c_int32, ctypes.c_int64
        L.rk_crc32.argtypes, L.rk_crc32.restype = [u8p, sz], u32
        L.rk_crc32_update.argtypes, L.rk_crc32_update.restype = [u32, u8p, sz], u32
        L.rk_coders_new.argtypes, L.rk_coders_new.restype = [u32], vp
        L.rk_coders_free.argtypes = [vp]
        L.rk_enc_uniform.argtypes, L.rk_enc_uniform.restype = [vp, u32, u32p, u32p, u32], i32
        L.rk_enc_batch.argtypes, L.rk_enc_batch.restype = [vp, u32, u32p, u32p, u32], i32
        L.rk_enc_finish.argtypes, L.rk_enc_finish.restype = [vp, u32, u8p, sz], i64
        L.rk_dec_start.argtypes, L.rk_dec_start.restype = [vp, u32, u8p, sz], i32
        L.rk_dec_uniform.argtypes, L.rk_dec_uniform.restype = [vp, u32, u32p, u32, u32p], i32
        L.rk_dec_freq_batch.argtypes, L.rk_dec_freq_batch.restype = [vp, u32, u32p, u32, u32p], i32
        L.rk_dec_update_batch.argtypes, L.rk_dec_update_batch.restype = [vp, u32, u32p, u32p, u32], i32
        L.rk_arc_pack.argtypes, L.rk_arc_pack.restype = [ctypes.POINTER(_Header), u8p, sz, u32, u8p, sz], i64
        L.rk_arc_unpack.argtypes = [u8p, sz, ctypes.POINTER(_Header), ctypes.POINTER(sz), ctypes.POINTER(sz),
                                    ctypes.POINTER(u32)]
        L.rk_arc_unpack.restype = i32
        L.rk_markov_text.argtypes, L.rk_markov_text.restype = [ctypes.c_uint64, ctypes.c_uint64, u8p, sz], sz
        L.rk_vocab_learn.argtypes = [u8p, sz, u32, u32, u32, u8p, sz, u32p]
        L.rk_vocab_learn.restype = i64
        L.rk_tok_new.argtypes, L.rk_tok_new.restype = [u8p, u32p, u32], vp
        L.rk_tok_free.argtypes = [vp]
        L.rk_tok_encode.argtypes, L.rk_tok_encode.restype = [vp, u8p, sz, u32p, sz], i64
        L.rk_tok_decode.argtypes, L.rk_tok_decode.restype = [vp, u32p, sz, u8p, sz], i64
        _lib = L
    return _lib


def _ptr(a) -> Optional[int]:
    if a is None:
        return None
    if isinstance(a, (bytes, bytearray)):
        return ctypes.cast(ctypes.c_char_p(bytes(a)), ctypes.c_void_p).value
    return a.ctypes.data


def crc32(data: bytes) -> int:
    b = np.frombuffer(data, np.uint8)
    return int(lib().rk_crc32(b.ctypes.data if len(b) else None, len(b)))


# ---- container ---------------------------------------------------------------------------------

@dataclass
class Header:
    total_bytes: int
    profile: int = PLUGIN_PROFILE
    reset_log2: int = RESET_LOG2
    backbone: int = PLUGIN_BACKBONE


def pack(hdr: Header, stream: bytes, crc: int) -> bytes:
    h = _Header(hdr.total_bytes, hdr.profile, hdr.reset_log2, hdr.backbone)
    s = np.frombuffer(stream, np.uint8)
    sp = s.ctypes.data if len(s) else None
    need = lib().rk_arc_pack(ctypes.byref(h), sp, len(s), crc, None, 0)
    out = np.empty(need, np.uint8)
    if lib().rk_arc_pack(ctypes.byref(h), sp, len(s), crc, out.ctypes.data, need) != need:
        raise ArchiveError("pack failed")
    return out.tobytes()


def unpack(buf: bytes):
    """(Header, stream bytes, crc); ArchiveError(FORMAT) for anything that is not this container."""
    b = np.frombuffer(buf, np.uint8)
    h = _Header()
    off, ln, crc = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_uint32()
    rc = lib().rk_arc_unpack(b.ctypes.data if len(b) else None, len(b), ctypes.byref(h), ctypes.byref(off),
                             ctypes.byref(ln), ctypes.byref(crc))
    if rc != OK:
        raise ArchiveError(f"not an RDKT v5 plugin archive (code {rc})")
    return (Header(h.total_bytes, h.profile & 0xBF, h.reset_log2, h.backbone), bytes(buf[off.value:off.value + ln.value]),
            int(crc.value))


# ---- synthetic text workload ---------------------------------------------------------------------

MARKOV_MODEL_SEED = 0x0DE7E3  # the order-3 source of the archive workload


def markov_text(seed: int, n: int, model_seed: int = MARKOV_MODEL_SEED) -> bytes:
    """n bytes of the synthetic order-3 Markov source (printable ASCII), sample `seed`."""
    out = np.empty(n, np.uint8)
    lib().rk_markov_text(model_seed, seed, out.ctypes.data, n)
    return out.tobytes()


class Tokenizer:
    """Greedy longest-match tokenizer over a byte-level vocabulary (token i = its byte string)."""

    def __init__(self, tokens: Sequence[bytes]):
        self.tokens = list(tokens)
        self.vocab = len(self.tokens)
        blob = b"".join(self.tokens)
        offs = np.zeros(self.vocab + 1, np.uint32)
        offs[1:] = np.cumsum([len(t) for t in self.tokens])
        self._blob = np.frombuffer(blob, np.uint8).copy()
        self._offs = offs
        self._h = lib().rk_tok_new(self._blob.ctypes.data, offs.ctypes.data, self.vocab)
        if not self._h:
            raise ArchiveError("tokenizer: bad vocabulary")

    @classmethod
    def learn(cls, text: bytes, vocab: int, per_round: int = 2048, max_len: int = 24) -> "Tokenizer":
        """The 256 byte tokens, then rounds of the most frequent adjacent pairs of `text`."""
        t = np.frombuffer(text, np.uint8)
        offs = np.zeros(vocab + 1, np.uint32)
        size = lib().rk_vocab_learn(t.ctypes.data, len(t), vocab, per_round, max_len, None, 0, offs.ctypes.data)
        if size < 0:
            raise ArchiveError("vocabulary learning failed")
        blob = np.empty(max(1, size), np.uint8)
        lib().rk_vocab_learn(t.ctypes.data, len(t), vocab, per_round, max_len, blob.ctypes.data, size, offs.ctypes.data)
        b = blob.tobytes()
        return cls([b[offs[i]:offs[i + 1]] for i in range(vocab)])

    def close(self) -> None:
        if self._h:
            lib().rk_tok_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def encode(self, text: bytes) -> np.ndarray:
        t = np.frombuffer(text, np.uint8)
        tp = t.ctypes.data if len(t) else None
        n = lib().rk_tok_encode(self._h, tp, len(t), None, 0)
        ids = np.empty(max(1, n), np.uint32)
        if n < 0 or lib().rk_tok_encode(self._h, tp, len(t), ids.ctypes.data, n) != n:
            raise ArchiveError("tokenize failed")
        return ids[:n]

    def decode(self, ids: np.ndarray) -> bytes:
        ids = np.ascontiguousarray(ids, np.uint32)
        n = lib().rk_tok_decode(self._h, ids.ctypes.data if len(ids) else None, len(ids), None, 0)
        if n < 0:
            raise ArchiveError("detokenize: token out of range")
        out = np.empty(max(1, n), np.uint8)
        lib().rk_tok_decode(self._h, ids.ctypes.data if len(ids) else None, len(ids), out.ctypes.data, n)
        return out[:n].tobytes()

    def lengths(self) -> np.ndarray:
        return np.diff(self._offs).astype(np.int64)


# ---- lockstep compression through the plugin ------------------------------------------------------

class Coders:
    def __init__(self, n: int):
        self.n = n
        self.h = lib().rk_coders_new(n)
        if not self.h:
            raise MemoryError("rk_coders_new")

    def close(self):
        if self.h:
            lib().rk_coders_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _check(rc: int, what: str) -> None:
    if rc != OK:
        raise ArchiveError(f"{what}: {'corrupt stream' if rc == CORRUPT else 'invalid argument'} (code {rc})")


def compress_windows(backend, windows: Sequence[bytes], tok: Tokenizer, reset_log2: int = RESET_LOG2) -> List[bytes]:
    """One RDKT v5 archive per window, all windows in lockstep on the plugin's batch slots
    0..len(windows)-1 (the pool must hold that many).  The backbone's periodic reset is set to
    2^reset_log2 forwards and recorded in the header."""
    n = len(windows)
    ids = [tok.encode(w) for w in windows]
    lens = np.array([len(x) for x in ids], np.int64)
    V = backend.vocab_size
    backend.set_reset_every(1 << reset_log2 if reset_log2 else 0)
    backend.batch_reset(list(range(n)))
    cod = Coders(n)
    L = lib()
    try:
        live = np.nonzero(lens > 0)[0].astype(np.uint32)
        first = np.array([ids[s][0] for s in live], np.uint32)
        _check(L.rk_enc_uniform(cod.h, len(live), live.ctypes.data, first.ctypes.data, V), "encode first tokens")
        T = int(lens.max()) if n else 0
        for t in range(T - 1):
            act = np.nonzero(lens > t + 1)[0].astype(np.uint32)  # streams with a token t + 1 to code
            if len(act) == 0:
                break
            cur = np.array([ids[s][t] for s in act], np.uint32)
            nxt = np.array([ids[s][t + 1] for s in act], np.uint32)
            q, _ = backend.forward_batch_cdf(act.tolist(), cur, symbols=nxt)
            q = np.ascontiguousarray(q, np.uint32)
            _check(L.rk_enc_batch(cod.h, len(act), act.ctypes.data, q.ctypes.data, TOTAL), f"encode step {t}")
        out = []
        for s in range(n):
            size = L.rk_enc_finish(cod.h, s, None, 0)
            buf = np.empty(max(1, size), np.uint8)
            if L.rk_enc_finish(cod.h, s, buf.ctypes.data, size) != size:
                raise ArchiveError("encoder finish failed")
            hdr = Header(len(windows[s]), PLUGIN_PROFILE, reset_log2, PLUGIN_BACKBONE)
            out.append(pack(hdr, buf[:size].tobytes(), crc32(windows[s])))
        return out
    finally:
        cod.close()
        backend.set_reset_every(0)


def decompress_windows(backend, archives: Sequence[bytes], tok: Tokenizer) -> List[object]:
    """Each archive back to its window's bytes, all in lockstep on slots 0..len(archives)-1.
    A window whose decoded bytes do not match the stored size or CRC-32 (or whose stream cannot be
    decoded) comes back as an ArchiveError instead of bytes."""
    n = len(archives)
    V = backend.vocab_size
    hdrs, crcs = [], []
    cod = Coders(n)
    L = lib()
    lengths = tok.lengths()
    result: List[object] = [None] * n
    try:
        for s, a in enumerate(archives):
            h, stream, crc = unpack(a)
            hdrs.append(h)
            crcs.append(crc)
            st = np.frombuffer(stream, np.uint8)
            _check(L.rk_dec_start(cod.h, s, st.ctypes.data if len(st) else None, len(st)), "decoder start")
        logs = {h.reset_log2 for h in hdrs}
        if len(logs) > 1:
            raise ArchiveError("windows of one lockstep batch must share RESET_LOG2")
        rl = logs.pop() if logs else 0
        backend.set_reset_every(1 << rl if rl else 0)
        backend.batch_reset(list(range(n)))
        total = np.array([h.total_bytes for h in hdrs], np.int64)
        got = np.zeros(n, np.int64)
        toks: List[List[int]] = [[] for _ in range(n)]
        live = np.nonzero(total > 0)[0].astype(np.uint32)
        if len(live):
            first = np.empty(len(live), np.uint32)
            rc = L.rk_dec_uniform(cod.h, len(live), live.ctypes.data, V, first.ctypes.data)
            _check(rc, "decode first tokens")
            for s, y in zip(live, first):
                toks[s].append(int(y))
                got[s] += lengths[y]
        failed = np.zeros(n, bool)
        while True:
            act = np.nonzero((got < total) & ~failed)[0].astype(np.uint32)
            if len(act) == 0:
                break
            cur = np.array([toks[s][-1] for s in act], np.uint32)
            cum = np.empty(len(act), np.uint32)
            if L.rk_dec_freq_batch(cod.h, len(act), act.ctypes.data, TOTAL, cum.ctypes.data) != OK:
                raise ArchiveError("decoder range underflow")
            q, _ = backend.forward_batch_cdf(act.tolist(), cur, cum_freqs=cum)
            q = np.ascontiguousarray(q, np.uint32)
            bad = q[:, 1] == 0xFFFFFFFF
            if bad.any():
                failed[act[bad]] = True
            ok_s = np.ascontiguousarray(act[~bad])  # kept alive across the native call
            ok_q = np.ascontiguousarray(q[~bad])
            _check(L.rk_dec_update_batch(cod.h, len(ok_s), ok_s.ctypes.data, ok_q.ctypes.data, TOTAL), "decode step")
            for s, y in zip(ok_s, ok_q[:, 0]):
                toks[s].append(int(y))
                got[s] += lengths[y]
        for s in range(n):
            if failed[s]:
                result[s] = ArchiveError("window stream is corrupt (symbol lookup failed)")
                continue
            data = tok.decode(np.array(toks[s], np.uint32)) if total[s] else b""
            if len(data) != total[s]:
                result[s] = ArchiveError(f"size mismatch: decoded {len(data)} bytes, expected {total[s]}")
            elif crc32(data) != crcs[s]:
                result[s] = ArchiveError(f"CRC-32 mismatch: expected {crcs[s]:08X}, got {crc32(data):08X}")
            else:
                result[s] = data
        return result
    finally:
        cod.close()
        backend.set_reset_every(0)
