"""ctypes view of the RWKV-7 CPU oracle (rwkv7_oracle.c) -- TEST INFRASTRUCTURE ONLY.

Only tests/, `__graft_entry__.smoke()` and bench.py's CPU-baseline leg import this module.
"""
from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence

import numpy as np

from oracle.oracle import lib as _base_lib, _p

_ready = False


def lib() -> ctypes.CDLL:
    global _ready
    L = _base_lib()
    if not _ready:
        f32, u32, i32, vp, sz = ctypes.c_float, ctypes.c_uint32, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t
        L.rw_model_load.argtypes, L.rw_model_load.restype = [ctypes.c_char_p], vp
        L.rw_model_free.argtypes = [vp]
        L.rw_model_dims.argtypes = [vp, vp]
        L.rw_model_q8.argtypes, L.rw_model_q8.restype = [vp, i32, u32, vp, vp], sz
        L.rw_model_embedding.argtypes, L.rw_model_embedding.restype = [vp], vp
        L.rw_state_new.argtypes, L.rw_state_new.restype = [vp], vp
        L.rw_state_free.argtypes = [vp]
        L.rw_state_reset.argtypes = [vp, vp]
        L.rw_state_set_reset_every.argtypes = [vp, ctypes.c_uint64]
        L.rw_state_export.argtypes = [vp, vp, vp, vp, vp, vp]
        L.rw_forward.argtypes = [vp, u32, vp, vp]
        L.rw_forward_multi.argtypes = [vp, u32, vp, vp, vp]
        L.rw_run_streams.argtypes = [vp, u32, u32, vp, vp, vp, i32]
        for name in ("rw_tanh_inplace", "rw_sigmoid_inplace"):
            getattr(L, name).argtypes = [vp, sz]
        for name in ("rw_sigmoid_add_into", "rw_decay_sigmoid_into"):
            getattr(L, name).argtypes = [vp, vp, vp, sz]
        L.rw_sigmoid_mix_inplace.argtypes = [vp, vp, vp, vp, sz]
        L.rw_q8_quantize_rows.argtypes = [vp, u32, u32, vp, vp]
        L.rw_quantize_vec.argtypes, L.rw_quantize_vec.restype = [vp, u32, vp], f32
        L.rw_gemv_w8a8.argtypes = [vp, vp, u32, u32, vp, vp]
        _ready = True
    return L


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, np.float32)


def tanh(x) -> np.ndarray:
    y = _f32(x).copy()
    lib().rw_tanh_inplace(_p(y), y.size)
    return y


def sigmoid(x) -> np.ndarray:
    y = _f32(x).copy()
    lib().rw_sigmoid_inplace(_p(y), y.size)
    return y


def sigmoid_add(base, off) -> np.ndarray:
    b, o = _f32(base), _f32(off)
    out = np.empty_like(b)
    lib().rw_sigmoid_add_into(_p(out), _p(b), _p(o), b.size)
    return out


def decay_sigmoid(base, off) -> np.ndarray:
    b, o = _f32(base), _f32(off)
    out = np.empty_like(b)
    lib().rw_decay_sigmoid_into(_p(out), _p(b), _p(o), b.size)
    return out


def sigmoid_mix(v_out, v_first, base, off) -> np.ndarray:
    v, f, b, o = _f32(v_out).copy(), _f32(v_first), _f32(base), _f32(off)
    lib().rw_sigmoid_mix_inplace(_p(v), _p(f), _p(b), _p(o), v.size)
    return v


def q8_quantize_rows(w):
    w = _f32(w)
    rows, cols = w.shape
    q = np.empty((rows, cols), np.int8)
    s = np.empty(rows, np.float32)
    lib().rw_q8_quantize_rows(_p(w), rows, cols, _p(q), _p(s))
    return q, s


def quantize_vec(v):
    v = _f32(v)
    q = np.empty(v.size, np.int8)
    s = lib().rw_quantize_vec(_p(v), v.size, _p(q))
    return q, np.float32(s)


def gemv_w8a8(q, s, v) -> np.ndarray:
    q = np.ascontiguousarray(q, np.int8)
    s, v = _f32(s), _f32(v)
    out = np.empty(q.shape[0], np.float32)
    lib().rw_gemv_w8a8(_p(q), _p(s), q.shape[0], q.shape[1], _p(v), _p(out))
    return out


class Model:
    """The reference's RWKV-7 model (W8A8) loaded from an RWKV-7 .rbin."""

    def __init__(self, rbin: str):
        self._h = lib().rw_model_load(rbin.encode())
        if not self._h:
            raise RuntimeError(f"oracle could not load {rbin}")
        d = (ctypes.c_uint32 * 11)()
        lib().rw_model_dims(self._h, ctypes.addressof(d))
        (self.vocab, self.d, self.n_head, self.head_size, self.d_ffn, self.n_layer, self.lora_w, self.lora_a,
         self.lora_v, self.lora_g, self.g1k) = list(d)

    def close(self) -> None:
        if self._h:
            lib().rw_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def q8(self, which: int, layer: int = 0):
        """which: 0 r, 1 k, 2 v, 3 o, 4 FFN key, 5 FFN value, 6 head -> (int8 [rows, cols], scales [rows])."""
        shapes = {0: (self.d, self.d), 1: (self.d, self.d), 2: (self.d, self.d), 3: (self.d, self.d),
                  4: (self.d_ffn, self.d), 5: (self.d, self.d_ffn), 6: (self.vocab, self.d)}
        rows, cols = shapes[which]
        q = np.empty((rows, cols), np.int8)
        s = np.empty(rows, np.float32)
        if lib().rw_model_q8(self._h, which, layer, _p(q), _p(s)) != rows * cols:
            raise ValueError("bad matrix selector")
        return q, s

    def embedding(self) -> np.ndarray:
        ptr = lib().rw_model_embedding(self._h)
        arr = np.ctypeslib.as_array(ctypes.cast(ptr, ctypes.POINTER(ctypes.c_float)), shape=(self.vocab, self.d))
        return arr.copy()


class State:
    def __init__(self, model: Model):
        self.model = model
        self._h = lib().rw_state_new(model._h)

    def close(self) -> None:
        if self._h:
            lib().rw_state_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self) -> None:
        lib().rw_state_reset(self.model._h, self._h)

    def set_reset_every(self, every: int) -> None:
        lib().rw_state_set_reset_every(self._h, every)

    def forward(self, token: int) -> np.ndarray:
        out = np.empty(self.model.vocab, np.float32)
        lib().rw_forward(self.model._h, token, self._h, _p(out))
        return out

    def export(self):
        """(x_prev_att [L, D], wkv [L, H, N, N], x_prev_ffn [L, D], v_first [D])"""
        m = self.model
        xa = np.empty((m.n_layer, m.d), np.float32)
        wkv = np.empty((m.n_layer, m.n_head, m.head_size, m.head_size), np.float32)
        xf = np.empty((m.n_layer, m.d), np.float32)
        vf = np.empty(m.d, np.float32)
        lib().rw_state_export(m._h, self._h, _p(xa), _p(wkv), _p(xf), _p(vf))
        return xa, wkv, xf, vf


def forward_multi(model: Model, states: Sequence[State], tokens: Sequence[int]) -> np.ndarray:
    n = len(states)
    toks = np.ascontiguousarray(tokens, np.uint32)
    hs = (ctypes.c_void_p * n)(*[s._h for s in states])
    out = np.empty((n, model.vocab), np.float32)
    lib().rw_forward_multi(model._h, n, _p(toks), ctypes.addressof(hs), _p(out))
    return out


def run_streams(model: Model, states: Sequence[State], tokens: np.ndarray, last_only: bool = True) -> np.ndarray:
    """Advance each stream over its row of `tokens` ([n, steps]); returns the last step's logits
    ([n, V]) or every step's ([n, steps, V])."""
    toks = np.ascontiguousarray(tokens, np.uint32)
    n, steps = toks.shape
    hs = (ctypes.c_void_p * n)(*[s._h for s in states])
    out = np.empty((n, model.vocab) if last_only else (n, steps, model.vocab), np.float32)
    lib().rw_run_streams(model._h, n, steps, _p(toks), ctypes.addressof(hs), _p(out), 1 if last_only else 0)
    return out
