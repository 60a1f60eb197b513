"""RWKV-7 weight files (`.rbin` version 3, model kind RWKV-7) and the seeded RWKV-7 models the engine is measured on.

The reference loads RWKV-7 from HF SafeTensors and quantises it W8A8 at load
(`src/infrastructure/rwkv7/model.rs:249-329`, `load_layer_hf` `:929-995`).  The GPU plugin's
`.rbin` container has no RWKV form (it carries Mamba only), so this engine extends it with a
model kind: header version 3 and flag bit 4 select RWKV-7, which the reference plugin rejects
cleanly because it accepts versions 1 and 2 only (`plugins/redukt-gpu-cuda/mamba_cuda.cu:472`).

Header: nineteen little-endian u32 words
    0 magic 0x55504752   1 version 3      2 vocab      3 d_model    4 d_ffn      5 head_size
    6 n_head             7 0              8 n_layer    9 flags      10 tokenizer (2 = World)
    11 lora_w  12 lora_a  13 lora_v  14 lora_g       15..18 0
flags: bit 4 = RWKV-7 (required), bit 5 = G1k bonus variant (`Rwkv7Config::g1k`, model.rs:14-21).

Body: f32 arrays in `array_order`, every matrix row-major [out][in] like the HF tensors.  The
embedding is stored raw and pre-normalised with ln0 at load, like `Rwkv7Model::load`.  Every
matrix the reference quantises (r/k/v/o projections, FFN key/value, head) is stored f32 and
quantised per row at load (`Q8Tensor::from_f32`, `src/domain/tensor.rs:113-135`).
"""
from __future__ import annotations

import dataclasses
import hashlib
import os
import struct
from typing import Dict, Iterator, List, Tuple

import numpy as np

RBIN_MAGIC = 0x55504752
RWKV7_VERSION = 3
RWKV7_HEADER = struct.Struct("<19I")
FLAG_RWKV7 = 1 << 4
FLAG_G1K = 1 << 5
TOK_WORLD = 2

RWKV7_SEED = 0x5EED0701


@dataclasses.dataclass(frozen=True)
class Rwkv7Dims:
    vocab: int
    d_model: int
    n_layer: int
    d_ffn: int
    head_size: int = 64
    lora_w: int = 64
    lora_a: int = 64
    lora_v: int = 32
    lora_g: int = 128
    g1k: bool = False

    @property
    def n_head(self) -> int:
        return self.d_model // self.head_size

    def state_floats(self) -> int:
        """Per stream: x_prev_att, WKV matrices and x_prev_ffn of every layer, plus v_first
        (`Rwkv7State`, model.rs:113-120)."""
        d, n = self.d_model, self.head_size
        return self.n_layer * (2 * d + self.n_head * n * n) + d


# The 0.1B shape of `Rwkv7Config::default_0_1b` (model.rs:24-26).  d_ffn = 4 d; the LoRA ranks are
# those of the public RWKV-7 0.1B checkpoint (decay 64, a 64, v 32, gate 128).
RWKV7_0_1B = Rwkv7Dims(vocab=65536, d_model=768, n_layer=12, d_ffn=3072)
# A small model the CPU oracle runs in milliseconds per token (two heads, ragged LoRA ranks
# so the portable tail of the lane functions is exercised).
RWKV7_TEST_DIMS = Rwkv7Dims(vocab=300, d_model=128, n_layer=2, d_ffn=512, lora_w=20, lora_a=16, lora_v=12, lora_g=36)


def header_bytes(dims: Rwkv7Dims) -> bytes:
    flags = FLAG_RWKV7 | (FLAG_G1K if dims.g1k else 0)
    return RWKV7_HEADER.pack(RBIN_MAGIC, RWKV7_VERSION, dims.vocab, dims.d_model, dims.d_ffn, dims.head_size,
                             dims.n_head, 0, dims.n_layer, flags, TOK_WORLD, dims.lora_w, dims.lora_a,
                             dims.lora_v, dims.lora_g, 0, 0, 0, 0)


def read_header(path: str) -> Rwkv7Dims:
    with open(path, "rb") as f:
        w = RWKV7_HEADER.unpack(f.read(RWKV7_HEADER.size))
    if w[0] != RBIN_MAGIC or w[1] != RWKV7_VERSION or not (w[9] & FLAG_RWKV7):
        raise ValueError(f"{path}: not an RWKV-7 .rbin file")
    dims = Rwkv7Dims(vocab=w[2], d_model=w[3], n_layer=w[8], d_ffn=w[4], head_size=w[5], lora_w=w[11],
                     lora_a=w[12], lora_v=w[13], lora_g=w[14], g1k=bool(w[9] & FLAG_G1K))
    if dims.n_head != w[6] or dims.n_head * dims.head_size != dims.d_model:
        raise ValueError(f"{path}: n_head * head_size != d_model")
    return dims


def array_order(dims: Rwkv7Dims) -> List[Tuple[str, Tuple[int, ...]]]:
    d, f, v = dims.d_model, dims.d_ffn, dims.vocab
    out: List[Tuple[str, Tuple[int, ...]]] = [("emb", (v, d)), ("ln0_w", (d,)), ("ln0_b", (d,))]
    for i in range(dims.n_layer):
        p = f"layers.{i}."
        out += [(p + n, (d,)) for n in ("ln1_w", "ln1_b", "ln2_w", "ln2_b", "x_r", "x_w", "x_k", "x_v", "x_a", "x_g")]
        out += [(p + "w0", (d,)), (p + "w1", (dims.lora_w, d)), (p + "w2", (d, dims.lora_w)),
                (p + "a0", (d,)), (p + "a1", (dims.lora_a, d)), (p + "a2", (d, dims.lora_a)),
                (p + "v0", (d,)), (p + "v1", (dims.lora_v, d)), (p + "v2", (d, dims.lora_v)),
                (p + "g1", (dims.lora_g, d)), (p + "g2", (d, dims.lora_g)),
                (p + "k_k", (d,)), (p + "k_a", (d,)), (p + "r_k", (d,)),
                (p + "receptance", (d, d)), (p + "key", (d, d)), (p + "value", (d, d)), (p + "output", (d, d)),
                (p + "ln_x_w", (d,)), (p + "ln_x_b", (d,)),
                (p + "ffn_x_k", (d,)), (p + "ffn_key", (f, d)), (p + "ffn_value", (d, f))]
    out += [("ln_out_w", (d,)), ("ln_out_b", (d,)), ("head", (v, d))]
    return out


def file_bytes(dims: Rwkv7Dims) -> int:
    return RWKV7_HEADER.size + 4 * sum(int(np.prod(s)) for _, s in array_order(dims))


def seeded_arrays(dims: Rwkv7Dims, seed: int = RWKV7_SEED, std: float = 0.02) -> Iterator[Tuple[str, np.ndarray]]:
    """The benchmark/test model.  Big matrices (r/k/v/o, FFN, head, embedding) and the LoRA
    down-projections N(0, std); the a/v/g LoRA up-projections N(0, 0.1); the decay LoRA
    up-projection N(0, std).  Decay bias w0 = logit(u), u uniform in [0.00165, 0.1737], so the
    decay exp(-0.606531 * sigmoid(w0)) lies in [0.9, 0.999] before the LoRA term.  Token-shift
    mixes and k_a uniform in [0, 1), k_k uniform in [0.5, 1), r_k N(0, 0.1), a0/v0 N(0, 0.5).
    LayerNorm/GroupNorm weights 1 + N(0, 0.1), biases N(0, 0.1), so a swapped norm shows."""
    rng = np.random.Generator(np.random.PCG64(seed))

    def normal(shape, s):
        return (rng.standard_normal(size=shape, dtype=np.float32) * np.float32(s)).astype(np.float32)

    for name, shape in array_order(dims):
        base = name.rsplit(".", 1)[-1]
        if base.endswith("_w") and base.startswith("ln"):
            yield name, (np.float32(1.0) + normal(shape, 0.1)).astype(np.float32)
        elif base.endswith("_b") and base.startswith("ln"):
            yield name, normal(shape, 0.1)
        elif base in ("x_r", "x_w", "x_k", "x_v", "x_a", "x_g", "ffn_x_k", "k_a"):
            yield name, rng.uniform(0.0, 1.0, size=shape).astype(np.float32)
        elif base == "k_k":
            yield name, rng.uniform(0.5, 1.0, size=shape).astype(np.float32)
        elif base == "w0":
            u = rng.uniform(0.00165, 0.1737, size=shape)
            yield name, np.log(u / (1.0 - u)).astype(np.float32)
        elif base in ("a0", "v0"):
            yield name, normal(shape, 0.5)
        elif base == "r_k":
            yield name, normal(shape, 0.1)
        elif base in ("a2", "v2", "g2"):
            yield name, normal(shape, 0.1)
        else:
            yield name, normal(shape, std)


def write_rbin(path: str, dims: Rwkv7Dims, arrays: Iterator[Tuple[str, np.ndarray]]) -> str:
    """Write the header and the arrays (yielded in file order); returns the file's sha256."""
    expect = array_order(dims)
    h = hashlib.sha256()
    tmp = path + ".part"
    with open(tmp, "wb") as f:
        hb = header_bytes(dims)
        f.write(hb)
        h.update(hb)
        n = 0
        for (name, shape), (got_name, arr) in zip(expect, arrays):
            a = np.ascontiguousarray(arr, dtype="<f4")
            if got_name != name or a.shape != shape:
                raise ValueError(f"array {got_name}{a.shape} where {name}{shape} was expected")
            b = a.tobytes()
            f.write(b)
            h.update(b)
            n += 1
        if n != len(expect):
            raise ValueError(f"{len(expect) - n} arrays missing")
    os.replace(tmp, path)
    return h.hexdigest()


def read_arrays(path: str) -> Tuple[Rwkv7Dims, Dict[str, np.ndarray]]:
    dims = read_header(path)
    mm = np.memmap(path, dtype="<f4", mode="r", offset=RWKV7_HEADER.size)
    out, off = {}, 0
    for name, shape in array_order(dims):
        n = int(np.prod(shape))
        out[name] = np.asarray(mm[off:off + n]).reshape(shape)
        off += n
    if off != mm.shape[0]:
        raise ValueError(f"{path}: {mm.shape[0] - off} trailing floats")
    return dims, out


def ensure_model(path: str, dims: Rwkv7Dims, seed: int = RWKV7_SEED) -> str:
    """Write the seeded model to `path` unless a file with the same header and size exists."""
    if os.path.exists(path):
        try:
            if read_header(path) == dims and os.path.getsize(path) == file_bytes(dims):
                return path
        except ValueError:
            pass
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    write_rbin(path, dims, seeded_arrays(dims, seed))
    return path


def byte_tokens(n_streams: int, n_tokens: int, seed: int = 0x70C3E700) -> np.ndarray:
    """Uniform byte ids 0..255, one seeded generator per stream (seed + stream index): the
    RWKV-7 workload's token stream.  Returns [n_streams, n_tokens] uint32."""
    out = np.empty((n_streams, n_tokens), np.uint32)
    for b in range(n_streams):
        out[b] = np.random.Generator(np.random.PCG64(seed + b)).integers(0, 256, size=n_tokens, dtype=np.uint32)
    return out
