"""`.rbin` weight files and the seeded synthetic models the engine is measured on.

The `.rbin` container is redukt's GPU-plugin weight format (reference
`plugins/redukt-gpu-cuda/README.md:38-70`, reader `plugins/redukt-gpu-cuda/mamba_cuda.cu:95-120,
466-544`, host parser `src/infrastructure/plugin_backend/model.rs:157-232`): a 44-byte
little-endian header of eleven u32 words followed by f32 arrays in a fixed order.  The
layout has to stay byte-compatible so one file serves the reference plugin, this engine and
the reference's Rust host.

Flag bits 0 (LayerNorm bias) and 1 (untied head) are the reference's.  Bits 2 and 3 are this
engine's additive selectors for the Q8 weight-only profile (quantised at load with the
reference recipe, `src/domain/gemv.rs:251-273`): bit 2 = Q8 with one scale per 64 columns
(`Q8_GROUP`, `src/infrastructure/mamba/model.rs:50-56`), bit 3 (with bit 2) = one scale per row.
The reference plugin ignores both bits and runs F32.  Bit 6 (with bit 2, group scales) marks a
native Q8 payload: the Q8 matrices (embedding, in_proj, out_proj, untied head) are stored as int8
[rows][cols] followed by their f32 scales [rows][cols/64], already quantised with the same recipe,
so loading skips the f32 read and the quantisation (`to_q8_payload` converts an F32 file).  Such a
file is this engine's only; the reference plugin cannot read it.

No real checkpoint is available, so every model here is generated from a seed.
"""
from __future__ import annotations

import dataclasses
import hashlib
import os
import struct
from typing import Dict, Iterator, List, Optional, Tuple

import numpy as np

RBIN_MAGIC = 0x55504752  # "RGPU" little-endian
RBIN_HEADER = struct.Struct("<11I")
FLAG_NORM_BIAS = 1 << 0
FLAG_UNTIED_HEAD = 1 << 1
FLAG_Q8 = 1 << 2
FLAG_Q8_PER_ROW = 1 << 3
FLAG_Q8_PAYLOAD = 1 << 6
Q8_GROUP = 64
TOK_BYTE, TOK_BPE = 0, 1

MAMBA130M_SEED = 0x5EED0130


@dataclasses.dataclass(frozen=True)
class MambaDims:
    vocab: int
    d_model: int
    n_layer: int
    d_state: int = 16
    d_conv: int = 4

    @property
    def d_inner(self) -> int:  # MambaConfig::from_d_model (model.rs:34-46)
        return 2 * self.d_model

    @property
    def dt_rank(self) -> int:
        return (self.d_model + 15) // 16

    @property
    def xr(self) -> int:
        return self.dt_rank + 2 * self.d_state

    def state_bytes(self) -> int:  # model.rs:757-760
        return self.n_layer * self.d_inner * (self.d_conv - 1 + self.d_state) * 4


MAMBA_130M = MambaDims(vocab=50280, d_model=768, n_layer=24)


def header_bytes(dims: MambaDims, flags: int = 0, version: int = 2, tokenizer: Optional[int] = None) -> bytes:
    if tokenizer is None:
        tokenizer = TOK_BYTE if dims.vocab == 256 else TOK_BPE
    return RBIN_HEADER.pack(RBIN_MAGIC, version, dims.vocab, dims.d_model, dims.d_inner, dims.d_state,
                            dims.d_conv, dims.dt_rank, dims.n_layer, flags, tokenizer if version == 2 else 0)


def read_header(path: str) -> Tuple[MambaDims, int, int]:
    with open(path, "rb") as f:
        w = RBIN_HEADER.unpack(f.read(RBIN_HEADER.size))
    if w[0] != RBIN_MAGIC or w[1] not in (1, 2):
        raise ValueError(f"{path}: not an .rbin v1/v2 file")
    dims = MambaDims(vocab=w[2], d_model=w[3], n_layer=w[8], d_state=w[5], d_conv=w[6])
    if dims.d_inner != w[4] or dims.dt_rank != w[7]:
        raise ValueError(f"{path}: d_inner/dt_rank do not follow the Mamba config rule")
    return dims, w[9], w[10]


def array_order(dims: MambaDims, flags: int) -> List[Tuple[str, Tuple[int, ...]]]:
    """Names and shapes of the body arrays in file order."""
    d, di, ds, dc, dr = dims.d_model, dims.d_inner, dims.d_state, dims.d_conv, dims.dt_rank
    out: List[Tuple[str, Tuple[int, ...]]] = [("embeddings", (dims.vocab, d))]
    for i in range(dims.n_layer):
        p = f"layers.{i}."
        out.append((p + "norm_w", (d,)))
        if flags & FLAG_NORM_BIAS:
            out.append((p + "norm_b", (d,)))
        out += [(p + "in_proj_w", (2 * di, d)), (p + "conv1d_w", (di, dc)), (p + "conv1d_b", (di,)),
                (p + "x_proj_w", (dr + 2 * ds, di)), (p + "dt_proj_w", (di, dr)), (p + "dt_proj_b", (di,)),
                (p + "A_log", (di, ds)), (p + "D", (di,)), (p + "out_proj_w", (d, di))]
    out.append(("norm_f_w", (d,)))
    if flags & FLAG_NORM_BIAS:
        out.append(("norm_f_b", (d,)))
    if flags & FLAG_UNTIED_HEAD:
        out.append(("lm_head_w", (dims.vocab, d)))
    return out


def write_rbin(path: str, dims: MambaDims, arrays: Iterator[Tuple[str, np.ndarray]], flags: int = 0,
               version: int = 2) -> str:
    """Write a header and the arrays (yielded in file order); returns the sha256 of the file."""
    expect = array_order(dims, flags)
    h = hashlib.sha256()
    tmp = path + ".part"
    with open(tmp, "wb") as f:
        hb = header_bytes(dims, flags, version)
        f.write(hb)
        h.update(hb)
        for (name, shape), (got_name, arr) in zip(expect, arrays):
            a = np.ascontiguousarray(arr, dtype="<f4")
            if got_name != name or a.shape != shape:
                raise ValueError(f"array {got_name}{a.shape} where {name}{shape} was expected")
            b = a.tobytes()
            f.write(b)
            h.update(b)
    os.replace(tmp, path)
    return h.hexdigest()


def is_q8_matrix(name: str) -> bool:
    """The matrices the Q8 profile quantises (src/infrastructure/mamba/model.rs:375-376)."""
    return name in ("embeddings", "lm_head_w") or name.endswith(("in_proj_w", "out_proj_w"))


def q8_quantize(w: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """Q8wMatrix::quantize (src/domain/gemv.rs:256-273) with one scale per 64 columns, in f32:
    scale = max|w| / 127 (1 for an all-zero group), q = clamp(round(w * (1 / scale)), -127, 127),
    round half away from zero.  Returns (int8 [rows][cols], f32 [rows][cols / 64])."""
    rows, cols = w.shape
    g = np.ascontiguousarray(w, dtype=np.float32).reshape(rows, cols // Q8_GROUP, Q8_GROUP)
    amax = np.abs(g).max(axis=2)
    scale = np.where(amax > 0, amax / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    inv = (np.float32(1.0) / scale).astype(np.float32)
    prod = (g * inv[:, :, None]).astype(np.float32)
    t = np.trunc(prod)
    r = t + np.where(np.abs(prod - t) >= np.float32(0.5), np.sign(prod), np.float32(0.0))
    q = np.clip(r, -127, 127).astype(np.int8).reshape(rows, cols)
    return q, scale


def to_q8_payload(src: str, dst: str) -> str:
    """Rewrite an F32 Mamba .rbin as a native Q8 payload file (flags |= FLAG_Q8 | FLAG_Q8_PAYLOAD):
    each Q8 matrix becomes its int8 values followed by its group scales; the rest is copied."""
    dims, flags, tok = read_header(src)
    if flags & (FLAG_Q8_PAYLOAD | FLAG_Q8_PER_ROW):
        raise ValueError(f"{src}: already a payload file, or per-row scales (the payload has group scales)")
    _, _, arrays = read_arrays(src)
    with open(src, "rb") as f:
        w = list(RBIN_HEADER.unpack(f.read(RBIN_HEADER.size)))
    w[9] = flags | FLAG_Q8 | FLAG_Q8_PAYLOAD
    with open(dst + ".part", "wb") as g:
        g.write(RBIN_HEADER.pack(*w))
        for name, _shape in array_order(dims, flags):
            a = arrays[name]
            if is_q8_matrix(name):
                q, sc = q8_quantize(a)
                g.write(q.tobytes())
                g.write(np.ascontiguousarray(sc, dtype="<f4").tobytes())
            else:
                g.write(np.ascontiguousarray(a, dtype="<f4").tobytes())
    os.replace(dst + ".part", dst)
    return dst


def read_q8_payload(path: str) -> Tuple[MambaDims, int, Dict[str, object]]:
    """Arrays of a payload file: f32 arrays as they are, Q8 matrices as (int8 q, f32 scales)."""
    dims, flags, _ = read_header(path)
    if not flags & FLAG_Q8_PAYLOAD:
        raise ValueError(f"{path}: not a Q8 payload file")
    raw = np.fromfile(path, dtype=np.uint8, offset=RBIN_HEADER.size)
    out: Dict[str, object] = {}
    off = 0
    for name, shape in array_order(dims, flags & ~(FLAG_Q8 | FLAG_Q8_PAYLOAD)):
        n = int(np.prod(shape))
        if is_q8_matrix(name):
            q = raw[off:off + n].view(np.int8).reshape(shape)
            off += n
            ns = shape[0] * (shape[1] // Q8_GROUP)
            sc = raw[off:off + 4 * ns].view("<f4").reshape(shape[0], shape[1] // Q8_GROUP)
            off += 4 * ns
            out[name] = (q, sc)
        else:
            out[name] = raw[off:off + 4 * n].view("<f4").reshape(shape)
            off += 4 * n
    if off != raw.size:
        raise ValueError(f"{path}: {raw.size - off} trailing bytes")
    return dims, flags, out


def read_arrays(path: str) -> Tuple[MambaDims, int, Dict[str, np.ndarray]]:
    dims, flags, _ = read_header(path)
    if flags & FLAG_Q8_PAYLOAD:
        raise ValueError(f"{path}: a Q8 payload file (read_q8_payload)")
    mm = np.memmap(path, dtype="<f4", mode="r", offset=RBIN_HEADER.size)
    out, off = {}, 0
    for name, shape in array_order(dims, flags):
        n = int(np.prod(shape))
        out[name] = np.asarray(mm[off:off + n]).reshape(shape)
        off += n
    if off != mm.shape[0]:
        raise ValueError(f"{path}: {mm.shape[0] - off} trailing floats")
    return dims, flags, out


# ---------------------------------------------------------------------------------------------
# Seeded models
# ---------------------------------------------------------------------------------------------

def _softplus_inv(u: np.ndarray) -> np.ndarray:
    return u + np.log(-np.expm1(-u))


def gaussian_arrays(dims: MambaDims, seed: int = MAMBA130M_SEED, flags: int = 0,
                    std: float = 0.02) -> Iterator[Tuple[str, np.ndarray]]:
    """The benchmark model: matrices and conv weights/bias N(0, std); A_log[j, k] = ln(k + 1);
    D = 1; dt bias = softplus^-1(u), u log-uniform in [1e-3, 0.1]; norm weights 1 (biases 0)."""
    rng = np.random.Generator(np.random.PCG64(seed))

    def normal(*shape):
        return (rng.standard_normal(size=shape, dtype=np.float32) * np.float32(std)).astype(np.float32)

    a_log = np.log(np.arange(1, dims.d_state + 1, dtype=np.float64)).astype(np.float32)
    for name, shape in array_order(dims, flags):
        base = name.rsplit(".", 1)[-1]
        if base in ("norm_w", "norm_f_w"):
            yield name, np.ones(shape, np.float32)
        elif base in ("norm_b", "norm_f_b"):
            yield name, np.zeros(shape, np.float32)
        elif base == "A_log":
            yield name, np.broadcast_to(a_log, shape).astype(np.float32)
        elif base == "D":
            yield name, np.ones(shape, np.float32)
        elif base == "dt_proj_b":
            u = np.exp(rng.uniform(np.log(1e-3), np.log(0.1), size=shape))
            yield name, _softplus_inv(u).astype(np.float32)
        else:
            yield name, normal(*shape)


def _xorshift_vec(n: int, seed: int, amp: float) -> np.ndarray:
    """`rand_vec` of the reference's Mamba tests (src/infrastructure/mamba/model.rs:1035-1044):
    xorshift32 mapped to f32 in [-amp, amp) with f32 arithmetic."""
    st = max(seed, 1) & 0xFFFFFFFF
    raw = np.empty(n, np.uint32)
    for i in range(n):
        st ^= (st << 13) & 0xFFFFFFFF
        st ^= st >> 17
        st ^= (st << 5) & 0xFFFFFFFF
        raw[i] = st
    f = raw.astype(np.float32)  # `st as f32` rounds to nearest
    umax = np.float32(4294967295.0)
    return ((f / umax) * np.float32(2.0) - np.float32(1.0)) * np.float32(amp)


def reference_test_arrays(dims: MambaDims) -> Iterator[Tuple[str, np.ndarray]]:
    """`synthetic_model` of the reference's unit tests (src/infrastructure/mamba/model.rs:1050-1082),
    the model its `forward_multi_bit_identical_to_single_stream` test runs (d=64, 2 layers, vocab 1200).
    Seeds advance by 17 from 1000 in struct-field order: every layer, then the embedding, then norm_f."""
    d, di, ds, dc, dr = dims.d_model, dims.d_inner, dims.d_state, dims.d_conv, dims.dt_rank
    seed = [1000]

    def nxt() -> int:
        seed[0] += 17
        return seed[0]

    layers = []
    for _ in range(dims.n_layer):
        L = {}
        L["norm_w"] = np.float32(1.0) + _xorshift_vec(d, nxt(), 0.5)
        L["in_proj_w"] = _xorshift_vec(2 * di * d, nxt(), 0.3).reshape(2 * di, d)
        L["conv1d_w"] = _xorshift_vec(di * dc, nxt(), 0.5).reshape(di, dc)
        L["conv1d_b"] = _xorshift_vec(di, nxt(), 0.1)
        L["x_proj_w"] = _xorshift_vec((dr + 2 * ds) * di, nxt(), 0.2).reshape(dr + 2 * ds, di)
        L["dt_proj_w"] = _xorshift_vec(di * dr, nxt(), 0.5).reshape(di, dr)
        L["dt_proj_b"] = _xorshift_vec(di, nxt(), 1.0) - np.float32(2.0)
        L["A_log"] = np.abs(_xorshift_vec(di * ds, nxt(), 1.0)).reshape(di, ds)
        L["D"] = _xorshift_vec(di, nxt(), 1.0)
        L["out_proj_w"] = _xorshift_vec(d * di, nxt(), 0.2).reshape(d, di)
        layers.append(L)
    emb = _xorshift_vec(dims.vocab * d, nxt(), 1.0).reshape(dims.vocab, d)
    norm_f = np.float32(1.0) + _xorshift_vec(d, nxt(), 0.5)
    yield "embeddings", emb
    for i, L in enumerate(layers):
        for k in ("norm_w", "in_proj_w", "conv1d_w", "conv1d_b", "x_proj_w", "dt_proj_w", "dt_proj_b",
                  "A_log", "D", "out_proj_w"):
            yield f"layers.{i}.{k}", L[k]
    yield "norm_f_w", norm_f


REFERENCE_TEST_DIMS = MambaDims(vocab=1200, d_model=64, n_layer=2)


def ensure_model(path: str, dims: MambaDims, kind: str = "gaussian", seed: int = MAMBA130M_SEED,
                 flags: int = 0) -> str:
    """Write the seeded model to `path` unless an identical one (same header) already exists."""
    if os.path.exists(path):
        try:
            d2, f2, _ = read_header(path)
            nbytes = RBIN_HEADER.size + 4 * sum(int(np.prod(s)) for _, s in array_order(dims, flags))
            if d2 == dims and f2 == flags and os.path.getsize(path) == nbytes:
                return path
        except ValueError:
            pass
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    if kind == "gaussian":
        arrays = gaussian_arrays(dims, seed, flags & (FLAG_NORM_BIAS | FLAG_UNTIED_HEAD))
    elif kind == "reference_test":
        if flags & (FLAG_NORM_BIAS | FLAG_UNTIED_HEAD):
            raise ValueError("the reference's synthetic model is RMSNorm with a tied head")
        arrays = reference_test_arrays(dims)
    else:
        raise ValueError(kind)
    write_rbin(path, dims, arrays, flags)
    return path


def with_flags(src: str, dst: str, set_flags: int, clear_flags: int = 0) -> str:
    """Copy an .rbin with header flag bits changed (the body is unchanged)."""
    dims, flags, tok = read_header(src)
    new = (flags | set_flags) & ~clear_flags
    if (new ^ flags) & (FLAG_NORM_BIAS | FLAG_UNTIED_HEAD | FLAG_Q8_PAYLOAD):
        raise ValueError("layout bits cannot be changed without rewriting the body")
    if os.path.exists(dst):
        try:
            d2, f2, _ = read_header(dst)
            if d2 == dims and f2 == new and os.path.getsize(dst) == os.path.getsize(src):
                return dst
        except ValueError:
            pass
    with open(src, "rb") as f, open(dst + ".part", "wb") as g:
        w = list(RBIN_HEADER.unpack(f.read(RBIN_HEADER.size)))
        w[9] = new
        g.write(RBIN_HEADER.pack(*w))
        while True:
            chunk = f.read(1 << 24)
            if not chunk:
                break
            g.write(chunk)
    os.replace(dst + ".part", dst)
    return dst
