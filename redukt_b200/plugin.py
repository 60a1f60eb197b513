"""Host-side binding of libredukt_gpu.so, mirroring redukt's plugin host.

The reference host is Rust: `PluginLibrary` (src/infrastructure/plugin_backend/loader.rs:157-245)
resolves the v1 symbols and, when all four v2 symbols exist and `abi_version() >= 2`, the v2
table (loader.rs:196-216); `PluginBackend` (src/infrastructure/plugin_backend/model.rs:362-452)
validates batch arguments on the host before crossing the boundary (`validate_batch_args`,
src/domain/backend_ffi.rs:182-202) and maps raw codes with `BackendResult::from_code`
(backend_ffi.rs:48-57).  This module restates that host in Python over ctypes, with the same
names, argument meaning and error behaviour, plus the engine's additive symbols.

There is no CPU fallback: if the library or a CUDA device is missing, calls fail loudly.
"""
from __future__ import annotations

import ctypes
import enum
import os
from typing import Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
DEFAULT_LIB = os.path.join(HERE, "libredukt_gpu.so")

BACKEND_FFI_VERSION = 1
BACKEND_ABI_V2 = 2
BACKEND_NAME_MAX = 64
MAX_STREAMS = 4096

V1_SYMBOLS = ("redukt_backend_init", "redukt_backend_forward", "redukt_backend_reset_state", "redukt_backend_free")
V2_SYMBOLS = ("redukt_backend_abi_version", "redukt_backend_batch_init", "redukt_backend_batch_reset",
              "redukt_backend_forward_batch")
EXT_SYMBOLS = ("redukt_backend_set_reset_every", "redukt_backend_forward_batch_probs",
               "redukt_b200_forward_batch_device", "redukt_b200_device_error", "redukt_b200_get_state",
               "redukt_b200_get_q8", "redukt_b200_info", "redukt_b200_set_option", "redukt_b200_kernel_times",
               "redukt_b200_time_kernel", "redukt_b200_softmax_noalloc", "redukt_b200_rwkv_get_state",
               "redukt_b200_cdf_device", "redukt_b200_cdf", "redukt_b200_forward_batch_cdf",
               "redukt_b200_last_error")
KERNEL_CLASSES = ("embed", "norm", "in_proj", "x_proj", "scan", "out_proj", "head", "softmax", "step")


class BackendResult(enum.IntEnum):
    OK = 0
    INIT_FAILED = 1
    FORWARD_FAILED = 2
    VERSION_MISMATCH = 3
    WEIGHTS_NOT_FOUND = 4
    INVALID_ARGUMENT = 5

    @classmethod
    def from_code(cls, code: int) -> "BackendResult":
        """Unknown codes map to FORWARD_FAILED (backend_ffi.rs:48-57)."""
        try:
            return cls(code)
        except ValueError:
            return cls.FORWARD_FAILED


class BackendInfo(ctypes.Structure):
    _fields_ = [("ffi_version", ctypes.c_uint32), ("vocab_size", ctypes.c_uint32),
                ("hidden_dim", ctypes.c_uint32), ("name", ctypes.c_uint8 * BACKEND_NAME_MAX)]

    def name_str(self) -> str:
        raw = bytes(self.name)
        return raw.split(b"\0", 1)[0].decode("utf-8", "replace")


class PluginError(RuntimeError):
    def __init__(self, what: str, code: BackendResult, detail: str = ""):
        super().__init__(f"{what}: {code.name}" + (f" ({detail})" if detail else ""))
        self.code = code


def validate_batch_args(slots: Sequence[int], tokens: Sequence[int], out_len: int, vocab_size: int,
                        max_streams: int) -> BackendResult:
    """Host-side check of forward_batch arguments (backend_ffi.rs:182-202)."""
    n = len(slots)
    if len(tokens) != n or n > max_streams or out_len != n * vocab_size:
        return BackendResult.INVALID_ARGUMENT
    seen = bytearray(max_streams)
    for s, t in zip(slots, tokens):
        if s < 0 or s >= max_streams or t < 0 or t >= vocab_size or seen[s]:
            return BackendResult.INVALID_ARGUMENT
        seen[s] = 1
    return BackendResult.OK


def _u32p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32))


def _f32p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


class PluginLibrary:
    """dlopen of the plugin and its symbol tables (loader.rs:157-216)."""

    def __init__(self, path: Optional[str] = None):
        path = path or os.environ.get("REDUKT_B200_LIB", DEFAULT_LIB)
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} is missing: build it with `python -m redukt_b200.build`")
        self.path = path
        self.lib = ctypes.CDLL(path)
        L = self.lib
        u32, i32, f32p, u32p = ctypes.c_uint32, ctypes.c_int32, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_uint32)
        L.redukt_backend_init.argtypes = [ctypes.c_char_p, i32, ctypes.POINTER(BackendInfo)]
        L.redukt_backend_init.restype = ctypes.c_int
        L.redukt_backend_forward.argtypes = [u32, f32p, u32]
        L.redukt_backend_forward.restype = ctypes.c_int
        L.redukt_backend_reset_state.argtypes, L.redukt_backend_reset_state.restype = [], None
        L.redukt_backend_free.argtypes, L.redukt_backend_free.restype = [], None
        self.has_v2 = all(hasattr(L, s) for s in V2_SYMBOLS)
        if self.has_v2:
            L.redukt_backend_abi_version.argtypes, L.redukt_backend_abi_version.restype = [], u32
            L.redukt_backend_batch_init.argtypes, L.redukt_backend_batch_init.restype = [u32], i32
            L.redukt_backend_batch_reset.argtypes, L.redukt_backend_batch_reset.restype = [u32p, u32], i32
            L.redukt_backend_forward_batch.argtypes = [u32, u32p, u32p, f32p, u32]
            L.redukt_backend_forward_batch.restype = i32
            self.has_v2 = L.redukt_backend_abi_version() >= BACKEND_ABI_V2
        self.has_ext = all(hasattr(L, s) for s in EXT_SYMBOLS)
        if self.has_ext:
            vp = ctypes.c_void_p
            L.redukt_backend_set_reset_every.argtypes, L.redukt_backend_set_reset_every.restype = [u32], i32
            L.redukt_backend_forward_batch_probs.argtypes = [u32, u32p, u32p, f32p, u32]
            L.redukt_backend_forward_batch_probs.restype = i32
            L.redukt_b200_forward_batch_device.argtypes = [u32, vp, vp, vp, u32, i32, vp]
            L.redukt_b200_forward_batch_device.restype = i32
            L.redukt_b200_device_error.argtypes, L.redukt_b200_device_error.restype = [u32p], i32
            L.redukt_b200_get_state.argtypes, L.redukt_b200_get_state.restype = [u32, f32p, f32p], i32
            L.redukt_b200_get_q8.argtypes, L.redukt_b200_get_q8.restype = [i32, u32, vp, f32p], i32
            L.redukt_b200_info.argtypes, L.redukt_b200_info.restype = [u32p, u32], i32
            L.redukt_b200_set_option.argtypes = [ctypes.c_char_p, ctypes.c_int64]
            L.redukt_b200_set_option.restype = i32
            L.redukt_b200_kernel_times.argtypes = [i32, ctypes.POINTER(ctypes.c_double), u32p, u32]
            L.redukt_b200_kernel_times.restype = i32
            L.redukt_b200_time_kernel.argtypes = [i32, u32, u32, ctypes.POINTER(ctypes.c_float)]
            L.redukt_b200_time_kernel.restype = i32
            L.redukt_b200_softmax_noalloc.argtypes = [vp, u32, u32, vp, vp]
            L.redukt_b200_rwkv_get_state.argtypes = [u32, f32p, f32p, f32p, f32p]
            L.redukt_b200_rwkv_get_state.restype = i32
            L.redukt_b200_softmax_noalloc.restype = i32
            L.redukt_b200_cdf_device.argtypes = [vp, u32, u32, u32, vp, u32, vp, vp, vp, vp]
            L.redukt_b200_cdf_device.restype = i32
            L.redukt_b200_cdf.argtypes = [f32p, u32, u32, u32p, u32p, u32p, u32p]
            L.redukt_b200_cdf.restype = i32
            L.redukt_b200_forward_batch_cdf.argtypes = [u32, u32p, u32p, u32p, u32p, u32p, u32p]
            L.redukt_b200_forward_batch_cdf.restype = i32
            L.redukt_b200_last_error.argtypes, L.redukt_b200_last_error.restype = [], ctypes.c_char_p

    def softmax_noalloc(self, d_logits: int, n_rows: int, vocab: int, d_probs: int, stream: int = 0) -> BackendResult:
        """Row softmax of device logits into device probabilities without any allocation
        (redukt_b200_softmax_noalloc); raw device addresses, stream 0 = legacy default stream."""
        return BackendResult.from_code(self.lib.redukt_b200_softmax_noalloc(d_logits, n_rows, vocab, d_probs,
                                                                            stream or None))

    def cdf_device(self, d_logits: int, n_rows: int, vocab: int, ld_logits: int, d_cdf: int, ld_cdf: int,
                   d_symbols: int = 0, d_cum_freqs: int = 0, d_query_out: int = 0, stream: int = 0) -> BackendResult:
        """The coder CDF of device logit rows into device rows of vocab + 1 words
        (redukt_b200_cdf_device); raw device addresses, stream 0 = legacy default stream."""
        return BackendResult.from_code(self.lib.redukt_b200_cdf_device(
            d_logits, n_rows, vocab, ld_logits, d_cdf, ld_cdf, d_symbols or None, d_cum_freqs or None,
            d_query_out or None, stream or None))

    def cdf(self, logits: np.ndarray, symbols: Optional[np.ndarray] = None, cum_freqs: Optional[np.ndarray] = None,
            want_cdf: bool = True):
        """Host rows of f32 logits -> (cdf [n, vocab + 1] uint32 or None, queries [n, 3] uint32 or None),
        the reference's cdf_from_logits_with(.., FmathV1) + Cdf::from_probs (redukt_b200_cdf).  Raises
        ValueError on INVALID_ARGUMENT and RuntimeError on any other failure."""
        x = np.ascontiguousarray(np.atleast_2d(logits), dtype=np.float32)
        n, v = x.shape
        out = np.empty((n, v + 1), dtype=np.uint32) if want_cdf else None
        q_in = symbols if symbols is not None else cum_freqs
        q_in = None if q_in is None else np.ascontiguousarray(q_in, dtype=np.uint32).reshape(n)
        q_out = np.empty((n, 3), dtype=np.uint32) if q_in is not None else None
        u32p = ctypes.POINTER(ctypes.c_uint32)
        ptr = (lambda a: a.ctypes.data_as(u32p) if a is not None else None)
        code = BackendResult.from_code(self.lib.redukt_b200_cdf(
            x.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), n, v, ptr(out),
            ptr(q_in) if symbols is not None else None, ptr(q_in) if cum_freqs is not None else None, ptr(q_out)))
        if code == BackendResult.INVALID_ARGUMENT:
            raise ValueError(f"cdf: invalid argument ({self.last_error()})")
        if code != BackendResult.OK:
            raise RuntimeError(f"cdf failed: {code.name} ({self.last_error()})")
        return out, q_out

    def last_error(self) -> str:
        if not self.has_ext:
            return ""
        return (self.lib.redukt_b200_last_error() or b"").decode("utf-8", "replace")


class PluginBackend:
    """One loaded model (the plugin is a process-global singleton: docs/api/PLUGIN-FFI-V2.md:57-58)."""

    def __init__(self, weights: str, device_id: int = 0, library: Optional[PluginLibrary] = None):
        self.libobj = library or PluginLibrary()
        self.lib = self.libobj.lib
        info = BackendInfo()
        code = BackendResult.from_code(self.lib.redukt_backend_init(weights.encode() + b"\0", device_id,
                                                                    ctypes.byref(info)))
        if code != BackendResult.OK:
            raise PluginError("redukt_backend_init", code, self.libobj.last_error())
        if info.ffi_version != BACKEND_FFI_VERSION:
            self.lib.redukt_backend_free()
            raise PluginError("ffi_version", BackendResult.VERSION_MISMATCH)
        self.info = info
        self.vocab_size = info.vocab_size
        self.hidden_dim = info.hidden_dim
        self.is_rwkv = info.name_str().startswith("b200-rwkv7")
        self.max_streams = 0
        self._closed = False

    # ---- v1 ----
    def forward(self, token: int, out: Optional[np.ndarray] = None) -> np.ndarray:
        out = np.empty(self.vocab_size, np.float32) if out is None else out
        code = BackendResult.from_code(self.lib.redukt_backend_forward(token, _f32p(out), self.vocab_size))
        if code != BackendResult.OK:
            raise PluginError("redukt_backend_forward", code, self.libobj.last_error())
        return out

    def reset_state(self) -> None:
        self.lib.redukt_backend_reset_state()

    def close(self) -> None:
        if not self._closed:
            self.lib.redukt_backend_free()
            self._closed = True

    # ---- v2 ----
    def abi_version(self) -> int:
        return int(self.lib.redukt_backend_abi_version()) if self.libobj.has_v2 else 1

    def _check_v2(self) -> None:
        if not self.libobj.has_v2:
            raise PluginError("batch API", BackendResult.VERSION_MISMATCH)

    def batch_init(self, max_streams: int) -> None:
        self._check_v2()
        code = BackendResult.from_code(self.lib.redukt_backend_batch_init(max_streams))
        if code != BackendResult.OK:
            raise PluginError("redukt_backend_batch_init", code, self.libobj.last_error())
        self.max_streams = max_streams

    def batch_reset(self, slots: Optional[Sequence[int]] = None) -> None:
        self._check_v2()
        if slots is None:
            code = self.lib.redukt_backend_batch_reset(None, 0)
        else:
            s = np.ascontiguousarray(slots, np.uint32)
            code = self.lib.redukt_backend_batch_reset(_u32p(s), len(s))
        code = BackendResult.from_code(code)
        if code != BackendResult.OK:
            raise PluginError("redukt_backend_batch_reset", code, self.libobj.last_error())

    def _batch_call(self, fn, what: str, slots, tokens, out, validate: bool) -> np.ndarray:
        s = np.ascontiguousarray(slots, np.uint32)
        t = np.ascontiguousarray(tokens, np.uint32)
        n = len(s)
        out = np.empty((n, self.vocab_size), np.float32) if out is None else out
        if validate:
            v = validate_batch_args(s.tolist(), t.tolist(), out.size, self.vocab_size, self.max_streams)
            if v != BackendResult.OK:
                raise PluginError(what, v, "rejected by host-side validation")
        code = BackendResult.from_code(fn(n, _u32p(s), _u32p(t), _f32p(out), self.vocab_size))
        if code != BackendResult.OK:
            raise PluginError(what, code, self.libobj.last_error())
        return out

    def forward_batch(self, slots: Sequence[int], tokens: Sequence[int], out: Optional[np.ndarray] = None,
                      validate: bool = True) -> np.ndarray:
        self._check_v2()
        return self._batch_call(self.lib.redukt_backend_forward_batch, "redukt_backend_forward_batch", slots,
                                tokens, out, validate)

    def forward_batch_raw(self, slots: np.ndarray, tokens: np.ndarray, out: np.ndarray) -> BackendResult:
        """forward_batch with no host validation: the plugin's own checks answer (tests)."""
        n = len(slots)
        return BackendResult.from_code(self.lib.redukt_backend_forward_batch(
            n, _u32p(slots), _u32p(tokens), _f32p(out), self.vocab_size))

    # ---- additive extensions ----
    def forward_batch_probs(self, slots: Sequence[int], tokens: Sequence[int],
                            out: Optional[np.ndarray] = None) -> np.ndarray:
        return self._batch_call(self.lib.redukt_backend_forward_batch_probs, "redukt_backend_forward_batch_probs",
                                slots, tokens, out, True)

    def forward_batch_cdf(self, slots: Sequence[int], tokens: Sequence[int], symbols: Optional[Sequence[int]] = None,
                          cum_freqs: Optional[Sequence[int]] = None, want_cdf: bool = False):
        """One step, then the coder CDF of its logits on the device (redukt_b200_forward_batch_cdf):
        returns (queries [n, 3] uint32 or None, cdf [n, vocab + 1] uint32 or None)."""
        n = len(slots)
        sl = np.ascontiguousarray(slots, dtype=np.uint32)
        tk = np.ascontiguousarray(tokens, dtype=np.uint32)
        qi = symbols if symbols is not None else cum_freqs
        qi = None if qi is None else np.ascontiguousarray(qi, dtype=np.uint32)
        q = np.empty((n, 3), dtype=np.uint32) if qi is not None else None
        c = np.empty((n, self.vocab_size + 1), dtype=np.uint32) if want_cdf else None
        ptr = (lambda a: _u32p(a) if a is not None else None)
        code = BackendResult.from_code(self.lib.redukt_b200_forward_batch_cdf(
            n, _u32p(sl), _u32p(tk), ptr(qi) if symbols is not None else None,
            ptr(qi) if cum_freqs is not None else None, ptr(q), ptr(c)))
        if code != BackendResult.OK:
            raise PluginError("redukt_b200_forward_batch_cdf", code, self.libobj.last_error())
        return q, c

    def set_reset_every(self, every: int) -> None:
        code = BackendResult.from_code(self.lib.redukt_backend_set_reset_every(every))
        if code != BackendResult.OK:
            raise PluginError("redukt_backend_set_reset_every", code, self.libobj.last_error())

    def forward_batch_device(self, n: int, d_slots: int, d_tokens: int, d_out: int, probs: bool = False,
                             stream: int = 0) -> None:
        """Device-resident step: pointers are raw device addresses (e.g. torch tensor.data_ptr()).
        `stream` is a cudaStream_t handle; 0 selects the library's own stream (not the legacy
        default stream), so callers that time with events must pass their own non-zero stream."""
        code = BackendResult.from_code(self.lib.redukt_b200_forward_batch_device(
            n, d_slots, d_tokens, d_out, self.vocab_size, 1 if probs else 0, stream or None))
        if code != BackendResult.OK:
            raise PluginError("redukt_b200_forward_batch_device", code, self.libobj.last_error())

    def device_error(self) -> int:
        w = np.zeros(1, np.uint32)
        code = BackendResult.from_code(self.lib.redukt_b200_device_error(_u32p(w)))
        if code != BackendResult.OK:
            raise PluginError("redukt_b200_device_error", code, self.libobj.last_error())
        return int(w[0])

    def kernel_times(self, enable: bool) -> dict:
        """{class: (ms, launches)} accumulated since the last call; then event timing on/off."""
        ms = np.zeros(len(KERNEL_CLASSES), np.float64)
        ln = np.zeros(len(KERNEL_CLASSES), np.uint32)
        code = BackendResult.from_code(self.lib.redukt_b200_kernel_times(
            1 if enable else 0, ms.ctypes.data_as(ctypes.POINTER(ctypes.c_double)), _u32p(ln), len(KERNEL_CLASSES)))
        if code != BackendResult.OK:
            raise PluginError("redukt_b200_kernel_times", code, self.libobj.last_error())
        return {k: (float(ms[i]), int(ln[i])) for i, k in enumerate(KERNEL_CLASSES)}

    def time_kernel(self, cls: str, n: int, reps: int = 5) -> float:
        """ms per launch of one kernel class in isolation (see redukt_b200_time_kernel)."""
        out = ctypes.c_float(0.0)
        code = BackendResult.from_code(self.lib.redukt_b200_time_kernel(KERNEL_CLASSES.index(cls), n, reps,
                                                                        ctypes.byref(out)))
        if code != BackendResult.OK:
            raise PluginError("redukt_b200_time_kernel", code, self.libobj.last_error())
        return float(out.value)

    def info_words(self) -> dict:
        w = np.zeros(13, np.uint32)
        code = BackendResult.from_code(self.lib.redukt_b200_info(_u32p(w), 13))
        if code != BackendResult.OK:
            raise PluginError("redukt_b200_info", code, self.libobj.last_error())
        keys = ("vocab", "d_model", "d_inner", "d_state", "d_conv", "dt_rank", "n_layer", "flags", "profile",
                "pool", "reset_every", "proj_path", "launches_per_step")
        return dict(zip(keys, (int(x) for x in w)))

    def rwkv_info(self) -> dict:
        """Dimensions of a loaded RWKV-7 model (redukt_b200_info words in RWKV-7 order)."""
        w = np.zeros(13, np.uint32)
        code = BackendResult.from_code(self.lib.redukt_b200_info(_u32p(w), 13))
        if code != BackendResult.OK:
            raise PluginError("redukt_b200_info", code, self.libobj.last_error())
        keys = ("vocab", "d_model", "d_ffn", "n_head", "head_size", "lora_sum", "n_layer", "flags", "profile",
                "pool", "reset_every", "proj_path", "launches_per_step")
        return dict(zip(keys, (int(x) for x in w)))

    def rwkv_state(self, slot: int):
        """(x_prev_att [L, D], wkv [L, H, N, N], x_prev_ffn [L, D], v_first [D]) of an RWKV-7 slot
        (slot=-1: the v1 stream), in the reference's layout (`Rwkv7State`)."""
        i = self.rwkv_info()
        L, D, H, N = i["n_layer"], i["d_model"], i["n_head"], i["head_size"]
        xa = np.empty((L, D), np.float32)
        wkv = np.empty((L, H, N, N), np.float32)
        xf = np.empty((L, D), np.float32)
        vf = np.empty(D, np.float32)
        code = BackendResult.from_code(self.lib.redukt_b200_rwkv_get_state(slot & 0xFFFFFFFF, _f32p(xa), _f32p(wkv),
                                                                           _f32p(xf), _f32p(vf)))
        if code != BackendResult.OK:
            raise PluginError("redukt_b200_rwkv_get_state", code, self.libobj.last_error())
        return xa, wkv, xf, vf

    def get_state(self, slot: int):
        """(conv [L, di, dc-1], ssm [L, di, ds]) of a batch slot (slot=-1: the v1 stream)."""
        i = self.info_words()
        conv = np.empty((i["n_layer"], i["d_inner"], i["d_conv"] - 1), np.float32)
        ssm = np.empty((i["n_layer"], i["d_inner"], i["d_state"]), np.float32)
        code = BackendResult.from_code(self.lib.redukt_b200_get_state(slot & 0xFFFFFFFF, _f32p(conv), _f32p(ssm)))
        if code != BackendResult.OK:
            raise PluginError("redukt_b200_get_state", code, self.libobj.last_error())
        return conv, ssm

    RWKV_Q8 = ("receptance", "key", "value", "output", "ffn_key", "ffn_value", "head")

    def get_q8(self, which: str, layer: int = 0):
        if self.is_rwkv:
            i = self.rwkv_info()
            d, f, v = i["d_model"], i["d_ffn"], i["vocab"]
            rows, cols = {"ffn_key": (f, d), "ffn_value": (d, f), "head": (v, d)}.get(which, (d, d))
            q = np.empty((rows, cols), np.int8)
            s = np.empty(rows, np.float32)
            code = BackendResult.from_code(self.lib.redukt_b200_get_q8(self.RWKV_Q8.index(which), layer, q.ctypes.data,
                                                                       _f32p(s)))
            if code != BackendResult.OK:
                raise PluginError("redukt_b200_get_q8", code, self.libobj.last_error())
            return q, s
        i = self.info_words()
        code_w = {"emb": 0, "head": 1, "in_proj": 2, "out_proj": 3}[which]
        rows, cols = {"emb": (i["vocab"], i["d_model"]), "head": (i["vocab"], i["d_model"]),
                      "in_proj": (2 * i["d_inner"], i["d_model"]), "out_proj": (i["d_model"], i["d_inner"])}[which]
        q = np.empty((rows, cols), np.int8)
        s = np.empty((rows, cols // 64), np.float32)
        code = BackendResult.from_code(self.lib.redukt_b200_get_q8(code_w, layer, q.ctypes.data, _f32p(s)))
        if code != BackendResult.OK:
            raise PluginError("redukt_b200_get_q8", code, self.libobj.last_error())
        return q, s

    def set_option(self, key: str, value: int) -> None:
        code = BackendResult.from_code(self.lib.redukt_b200_set_option(key.encode(), value))
        if code != BackendResult.OK:
            raise PluginError(f"redukt_b200_set_option({key})", code, self.libobj.last_error())


class PluginStreams:
    """Lockstep streams over the batch pool with the host-driven periodic reset of
    `PluginState::tick` (src/infrastructure/plugin_backend/model.rs:44-75): before a stream's token
    enters, its slot is reset when it has run `reset_every` forwards since the last reset.
    With `device_reset=True` the engine's device-side counters do the same without host calls."""

    def __init__(self, backend: PluginBackend, n: int, reset_every: int = 0, device_reset: bool = False):
        self.b = backend
        backend.batch_init(n)
        self.n = n
        self.reset_every = reset_every
        self.device_reset = device_reset
        self.since = np.zeros(n, np.int64)
        backend.set_reset_every(reset_every if device_reset else 0)

    def step(self, slots: Sequence[int], tokens: Sequence[int]) -> np.ndarray:
        if not self.device_reset and self.reset_every > 0:
            due = [s for s in slots if self.since[s] >= self.reset_every]
            if due:
                self.b.batch_reset(due)
                self.since[due] = 0
        self.since[np.asarray(slots, np.int64)] += 1
        return self.b.forward_batch(slots, tokens)
