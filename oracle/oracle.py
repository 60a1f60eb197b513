"""ctypes view of the CPU oracle (mamba_oracle.c, cdf_oracle.c; RWKV-7 in rwkv7.py) -- TEST INFRASTRUCTURE ONLY.

Only tests/, `__graft_entry__.smoke()` and bench.py's CPU-baseline leg import this module, and
only as the checker or the timed CPU baseline.  The product path (redukt_b200) never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import List, Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmamba_oracle.so")
REF_PLUGIN_PATH = os.path.join(HERE, "_ref", "libredukt_gpu_ref.so")

_lib: Optional[ctypes.CDLL] = None

PROFILE_F32, PROFILE_Q8 = 0, 1


def reference_root() -> Optional[str]:
    """The redukt source tree used to build and pin the test infrastructure: $REDUKT_REF_ROOT, else a
    directory named `reference` beside this repository's own directory; None when neither exists
    (as on a GPU box, which uses the prebuilt files)."""
    cand = os.environ.get("REDUKT_REF_ROOT") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
    return cand if os.path.isdir(cand) else None


def build(ref: bool = False) -> None:
    target = "all" if ref else "oracle"
    cmd = ["make", "-s", "-C", HERE, target]
    root = reference_root()
    if ref and root:
        cmd.append(f"REF_ROOT={root}")
    subprocess.run(cmd, check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        srcs = [os.path.join(HERE, f) for f in ("mamba_oracle.c", "rwkv7_oracle.c", "cdf_oracle.c", "oracle_internal.h")]
        if not os.path.exists(LIB_PATH) or any(
                os.path.exists(s) and os.path.getmtime(s) > os.path.getmtime(LIB_PATH) for s in srcs):
            build(ref=False)
        L = ctypes.CDLL(LIB_PATH)
        f32, u32, i32, vp = ctypes.c_float, ctypes.c_uint32, ctypes.c_int, ctypes.c_void_p
        L.orc_expf.argtypes, L.orc_expf.restype = [f32], f32
        L.orc_lnf.argtypes, L.orc_lnf.restype = [f32], f32
        L.orc_softplus.argtypes, L.orc_softplus.restype = [f32], f32
        L.orc_lane_sigmoidf.argtypes, L.orc_lane_sigmoidf.restype = [f32], f32
        L.orc_model_load.argtypes, L.orc_model_load.restype = [ctypes.c_char_p, i32, u32], vp
        L.orc_model_free.argtypes = [vp]
        L.orc_model_dims.argtypes = [vp, vp]
        L.orc_model_q8.argtypes, L.orc_model_q8.restype = [vp, i32, u32, vp, vp], i32
        L.orc_state_new.argtypes, L.orc_state_new.restype = [vp], vp
        L.orc_state_free.argtypes = [vp]
        L.orc_state_reset.argtypes = [vp]
        L.orc_state_set_reset_every.argtypes = [vp, ctypes.c_uint64]
        L.orc_state_export.argtypes = [vp, vp, vp]
        L.orc_forward.argtypes = [vp, u32, vp, vp]
        L.orc_forward_multi.argtypes = [vp, u32, vp, vp, vp]
        L.orc_softmax.argtypes = [vp, u32, vp]
        L.orc_q8_quantize.argtypes = [vp, u32, u32, u32, vp, vp]
        L.orc_q8_effective_group.argtypes, L.orc_q8_effective_group.restype = [u32, u32], u32
        L.orc_gemv_f32.argtypes = [vp, vp, u32, u32, vp]
        L.orc_gemv_q8.argtypes = [vp, vp, u32, u32, u32, vp, vp]
        L.orc_set_threads.argtypes = [i32]
        L.orc_get_threads.restype = i32
        L.orc_set_simd.argtypes = [i32]
        L.orc_exp_f64.argtypes, L.orc_exp_f64.restype = [ctypes.c_double], ctypes.c_double
        L.orc_cdf_from_logits.argtypes, L.orc_cdf_from_logits.restype = [vp, u32, u32, u32, vp, u32, i32], i32
        L.orc_cdf_lookup.argtypes, L.orc_cdf_lookup.restype = [vp, u32, u32], u32
        L.orc_cdf_from_probs.argtypes, L.orc_cdf_from_probs.restype = [vp, u32, vp], i32
        _lib = L
    return _lib


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


def expf(x: float) -> float:
    return lib().orc_expf(x)


def lnf(x: float) -> float:
    return lib().orc_lnf(x)


def softplus(x: float) -> float:
    return lib().orc_softplus(x)


def exp_f64(x: float) -> float:
    """The reference's portable binary64 exp (fmath-v1, src/domain/fmath.rs:383-429)."""
    return lib().orc_exp_f64(x)


def cdf_from_logits(logits: np.ndarray, threads: int = 1) -> np.ndarray:
    """Rows of f32 logits -> rows of vocab+1 uint32 CDF entries (total 2^24), the reference's
    `cdf_from_logits_with(.., FmathV1)` + `Cdf::from_probs` (codec.rs:785-798, coder.rs:43-82)."""
    x = np.ascontiguousarray(np.atleast_2d(logits), dtype=np.float32)
    n, v = x.shape
    out = np.empty((n, v + 1), dtype=np.uint32)
    if lib().orc_cdf_from_logits(_p(x), n, v, v, _p(out), v + 1, int(threads)) != 0:
        raise ValueError(f"cdf_from_logits: invalid shape {x.shape}")
    return out


def cdf_from_probs(probs: np.ndarray) -> np.ndarray:
    """`Cdf::from_probs` (coder.rs:43-82) of one row of f32 probabilities -> vocab+1 uint32 entries."""
    p = np.ascontiguousarray(probs, dtype=np.float32).reshape(-1)
    out = np.empty(p.shape[0] + 1, dtype=np.uint32)
    if lib().orc_cdf_from_probs(_p(p), p.shape[0], _p(out)) != 0:
        raise ValueError(f"cdf_from_probs: invalid length {p.shape[0]}")
    return out


def cdf_lookup(cdf_row: np.ndarray, cum_freq: int) -> int:
    """`Cdf::lookup` (coder.rs:100-114): the symbol whose interval holds cum_freq."""
    c = np.ascontiguousarray(cdf_row, dtype=np.uint32)
    return int(lib().orc_cdf_lookup(_p(c), c.shape[0] - 1, int(cum_freq)))


def set_threads(n: int) -> None:
    lib().orc_set_threads(n)


def get_threads() -> int:
    return lib().orc_get_threads()


def set_simd(on: bool) -> None:
    lib().orc_set_simd(1 if on else 0)


def softmax(logits: np.ndarray) -> np.ndarray:
    lg = np.ascontiguousarray(logits, np.float32)
    out = np.empty_like(lg)
    lib().orc_softmax(_p(lg), lg.size, _p(out))
    return out


def q8_quantize(w: np.ndarray, group: int):
    w = np.ascontiguousarray(w, np.float32)
    rows, cols = w.shape
    g = lib().orc_q8_effective_group(cols, group)
    q = np.empty((rows, cols), np.int8)
    s = np.empty((rows, cols // g), np.float32)
    lib().orc_q8_quantize(_p(w), rows, cols, group, _p(q), _p(s))
    return q, s


def gemv_f32(m: np.ndarray, v: np.ndarray) -> np.ndarray:
    m = np.ascontiguousarray(m, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    out = np.empty(m.shape[0], np.float32)
    lib().orc_gemv_f32(_p(m), _p(v), m.shape[0], m.shape[1], _p(out))
    return out


def gemv_q8(q: np.ndarray, s: np.ndarray, v: np.ndarray, group: int) -> np.ndarray:
    q = np.ascontiguousarray(q, np.int8)
    s = np.ascontiguousarray(s, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    out = np.empty(q.shape[0], np.float32)
    lib().orc_gemv_q8(_p(q), _p(s), q.shape[0], q.shape[1], group, _p(v), _p(out))
    return out


class Model:
    """The reference CPU Mamba model loaded from an .rbin (profile F32 or Q8, group 64 or per-row)."""

    def __init__(self, rbin: str, profile: int = PROFILE_F32, group: int = 64):
        self._h = lib().orc_model_load(rbin.encode(), profile, group)
        if not self._h:
            raise RuntimeError(f"oracle could not load {rbin}")
        dims = (ctypes.c_uint32 * 10)()
        lib().orc_model_dims(self._h, ctypes.addressof(dims))
        (self.vocab, self.d, self.di, self.ds, self.dc, self.dr, self.nl, self.flags, self.profile,
         _) = list(dims)
        self.group = group

    def close(self) -> None:
        if self._h:
            lib().orc_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def q8(self, which: str, layer: int = 0):
        """Quantized matrix as the oracle holds it: which in emb|head|in_proj|out_proj."""
        code = {"emb": 0, "head": 1, "in_proj": 2, "out_proj": 3}[which]
        rows, cols = {"emb": (self.vocab, self.d), "head": (self.vocab, self.d),
                      "in_proj": (2 * self.di, self.d), "out_proj": (self.d, self.di)}[which]
        g = lib().orc_q8_effective_group(cols, self.group)
        q = np.empty((rows, cols), np.int8)
        s = np.empty((rows, cols // g), np.float32)
        if lib().orc_model_q8(self._h, code, layer, _p(q), _p(s)) != 0:
            raise ValueError("not a Q8 model")
        return q, s

    def new_state(self, reset_every: int = 0) -> "State":
        return State(self, reset_every)

    def forward(self, token: int, state: "State") -> np.ndarray:
        out = np.empty(self.vocab, np.float32)
        lib().orc_forward(self._h, token, state._h, _p(out))
        return out

    def forward_multi(self, tokens: Sequence[int], states: Sequence["State"]) -> np.ndarray:
        n = len(tokens)
        toks = np.asarray(tokens, np.uint32)
        arr = (ctypes.c_void_p * n)(*[s._h for s in states])
        out = np.empty((n, self.vocab), np.float32)
        lib().orc_forward_multi(self._h, n, _p(toks), ctypes.addressof(arr), _p(out))
        return out


class State:
    def __init__(self, model: Model, reset_every: int = 0):
        self.model = model
        self._h = lib().orc_state_new(model._h)
        if reset_every:
            lib().orc_state_set_reset_every(self._h, reset_every)

    def __del__(self):
        try:
            if self._h:
                lib().orc_state_free(self._h)
                self._h = None
        except Exception:
            pass

    def reset(self) -> None:
        lib().orc_state_reset(self._h)

    def export(self):
        """(conv [L, di, dc-1], ssm [L, di, ds]) in the reference layout."""
        m = self.model
        conv = np.empty((m.nl, m.di, m.dc - 1), np.float32)
        ssm = np.empty((m.nl, m.di, m.ds), np.float32)
        lib().orc_state_export(self._h, _p(conv), _p(ssm))
        return conv, ssm


def run_streams(model: Model, token_rows: np.ndarray, reset_every: int = 0) -> np.ndarray:
    """Lockstep run: token_rows [n, T] -> logits [T, n, V] (all streams advance together)."""
    n, T = token_rows.shape
    states: List[State] = [model.new_state(reset_every) for _ in range(n)]
    out = np.empty((T, n, model.vocab), np.float32)
    for t in range(T):
        out[t] = model.forward_multi(token_rows[:, t].tolist(), states)
    return out
