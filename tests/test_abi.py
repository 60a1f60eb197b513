"""The C-ABI library: every declared symbol exported, the reference's error behaviour without a
model, host-side validation (src/domain/backend_ffi.rs:204-335).  No compute calls."""
import ctypes
import os
import re

import numpy as np
import pytest

from redukt_b200 import build as B
from redukt_b200.plugin import (V1_SYMBOLS, V2_SYMBOLS, EXT_SYMBOLS, BackendInfo, BackendResult, PluginLibrary,
                                validate_batch_args)

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "redukt_gpu.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(redukt_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    B.build()
    return PluginLibrary()


def test_header_declares_the_reference_abi():
    names = declared_functions()
    for s in V1_SYMBOLS + V2_SYMBOLS:
        assert s in names, s
    assert set(EXT_SYMBOLS) <= set(names)


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib.lib, name), name
    assert lib.has_v2 and lib.has_ext


def test_abi_version_and_info_layout(lib):
    assert lib.lib.redukt_backend_abi_version() == 2
    assert ctypes.sizeof(BackendInfo) == 12 + 64


def test_calls_before_init_report_the_reference_codes(lib):
    L = lib.lib
    out = np.zeros(256, np.float32)
    # no model loaded: v1 forward fails, v2 entry points report INIT_FAILED (mamba_cuda.cu:710-761)
    assert L.redukt_backend_forward(0, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), 256) == \
        BackendResult.FORWARD_FAILED
    assert L.redukt_backend_batch_init(4) == BackendResult.INIT_FAILED
    assert L.redukt_backend_batch_reset(None, 0) == BackendResult.INIT_FAILED
    assert L.redukt_backend_forward_batch(0, None, None, None, 256) == BackendResult.INIT_FAILED
    assert L.redukt_backend_set_reset_every(16) == BackendResult.INIT_FAILED
    assert L.redukt_b200_set_option(b"no_such_option", 1) == BackendResult.INVALID_ARGUMENT
    L.redukt_backend_reset_state()  # no-op without a model
    L.redukt_backend_free()


def test_init_without_weights_or_gpu_fails_loudly(lib, tmp_path):
    info = BackendInfo()
    rc = lib.lib.redukt_backend_init(str(tmp_path / "missing.rbin").encode(), 0, ctypes.byref(info))
    # WEIGHTS_NOT_FOUND with a GPU, INIT_FAILED without one: never OK, never a CPU fallback
    assert rc in (BackendResult.INIT_FAILED, BackendResult.WEIGHTS_NOT_FOUND)
    assert lib.last_error()


def test_from_code_roundtrip_and_unknown():
    for r in BackendResult:
        assert BackendResult.from_code(int(r)) == r
    assert BackendResult.from_code(-1) == BackendResult.FORWARD_FAILED
    assert BackendResult.from_code(99) == BackendResult.FORWARD_FAILED


def test_validate_batch_args_accepts_valid():
    assert validate_batch_args([3, 0, 7], [1, 2, 255], 3 * 256, 256, 8) == BackendResult.OK
    assert validate_batch_args([], [], 0, 256, 8) == BackendResult.OK


def test_validate_batch_args_rejects_bad_input():
    bad = BackendResult.INVALID_ARGUMENT
    assert validate_batch_args([1, 1], [0, 0], 512, 256, 4) == bad      # duplicate slot
    assert validate_batch_args([4], [0], 256, 256, 4) == bad            # slot out of range
    assert validate_batch_args([0], [256], 256, 256, 4) == bad          # token out of range
    assert validate_batch_args([0, 1], [0], 512, 256, 4) == bad         # length mismatch
    assert validate_batch_args([0], [0], 255, 256, 4) == bad            # wrong output size
    assert validate_batch_args([0, 1, 2, 3, 0], [0] * 5, 5 * 256, 256, 4) == bad  # more than the pool


def test_reference_plugin_build_exports_the_same_abi():
    from oracle import oracle as O
    if not os.path.exists(O.REF_PLUGIN_PATH):
        pytest.skip("reference plugin not built here")
    ref = ctypes.CDLL(O.REF_PLUGIN_PATH)
    for s in V1_SYMBOLS + V2_SYMBOLS:
        assert hasattr(ref, s), s
