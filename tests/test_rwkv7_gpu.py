"""RWKV-7 on the GPU through the C ABI, against the CPU oracle of the reference's RWKV-7 step.

The int8 x int8 dots of W8A8 are exact and every other operation keeps the reference's order,
so the bar is bit-identity: logits and state of every stream equal the oracle's bits, at every
batch size, on both projection paths (dp4a and tcgen05), in any slot.
"""
import os

import numpy as np
import pytest

from conftest import shared_backend
from oracle import oracle as O
from oracle import rwkv7 as W
from redukt_b200 import rwkv7_rbin as R
from redukt_b200.plugin import BackendResult

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rw_small(model_dir):
    return R.ensure_model(os.path.join(model_dir, "rwkv7_small.rbin"), R.RWKV7_TEST_DIMS)


@pytest.fixture(scope="module")
def rw_oracle(rw_small):
    return W.Model(rw_small)


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def run_oracle(m, toks):
    """toks [n, T] -> logits [n, T, V] and the final states."""
    states = [W.State(m) for _ in range(toks.shape[0])]
    out = np.stack([W.forward_multi(m, states, toks[:, t]) for t in range(toks.shape[1])], 1)
    return out, states


def run_gpu(b, slots, toks):
    return np.stack([b.forward_batch(slots, toks[:, t]) for t in range(toks.shape[1])], 1)


def test_loads_as_rwkv7(rw_small):
    b = shared_backend(rw_small)
    assert b.is_rwkv and b.info.name_str() == "b200-rwkv7-w8a8"
    i = b.rwkv_info()
    d = R.RWKV7_TEST_DIMS
    assert (i["vocab"], i["d_model"], i["d_ffn"], i["n_head"], i["head_size"], i["n_layer"]) == \
        (d.vocab, d.d_model, d.d_ffn, d.n_head, 64, d.n_layer)
    assert i["lora_sum"] == d.lora_w + d.lora_a + d.lora_v + d.lora_g and i["profile"] == 3


def test_w8_weights_bit_identical_to_oracle(rw_small, rw_oracle):
    b = shared_backend(rw_small)
    for which, name in enumerate(b.RWKV_Q8):
        for layer in ([0, 1] if which < 6 else [0]):
            q, s = b.get_q8(name, layer)
            q2, s2 = rw_oracle.q8(which, layer)
            assert np.array_equal(q, q2) and np.array_equal(bits(s), bits(s2)), (name, layer)


@pytest.mark.parametrize("path", [0, 1, 2])
def test_logits_bit_identical_to_oracle_every_batch_size(rw_small, rw_oracle, path):
    b = shared_backend(rw_small)
    b.set_option("proj_path", path)
    try:
        steps = 4
        for n in ((1, 2, 3, 5, 9, 17, 33, 70) if path == 0 else (3, 17, 40)):
            toks = R.byte_tokens(n, steps, seed=1000 + n)
            want, _ = run_oracle(rw_oracle, toks)
            b.batch_init(80)
            slots = [(11 * s + 5) % 80 for s in range(n)]
            got = run_gpu(b, slots, toks)
            for s in range(n):
                for t in range(steps):
                    assert np.array_equal(bits(got[s, t]), bits(want[s, t])), (path, n, s, t)
    finally:
        b.set_option("proj_path", 0)


def test_state_bit_identical_to_oracle(rw_small, rw_oracle):
    b = shared_backend(rw_small)
    n, steps = 6, 5
    toks = R.byte_tokens(n, steps, seed=77)
    _, states = run_oracle(rw_oracle, toks)
    b.batch_init(16)
    slots = [15 - 2 * s for s in range(n)]
    run_gpu(b, slots, toks)
    for s in range(n):
        got = b.rwkv_state(slots[s])
        want = states[s].export()
        for g, w_, name in zip(got, want, ("x_att", "wkv", "x_ffn", "v_first")):
            assert np.array_equal(bits(g), bits(w_)), (s, name)


def test_v1_equals_batch_and_oracle(rw_small, rw_oracle):
    b = shared_backend(rw_small)
    toks = R.byte_tokens(1, 6, seed=5)[0]
    st = W.State(rw_oracle)
    b.reset_state()
    for t in toks:
        assert np.array_equal(bits(b.forward(int(t))), bits(st.forward(int(t))))
    xa, wkv, xf, vf = b.rwkv_state(-1)
    assert np.array_equal(bits(wkv), bits(st.export()[1]))


def test_batch_reset_and_device_periodic_reset(rw_small, rw_oracle):
    b = shared_backend(rw_small)
    b.batch_init(8)
    toks = R.byte_tokens(3, 8, seed=9)
    slots = [1, 4, 6]
    # explicit reset of one slot mid-window
    st = [W.State(rw_oracle) for _ in range(3)]
    for t in range(8):
        if t == 4:
            b.batch_reset([4])
            st[1].reset()
        got = b.forward_batch(slots, toks[:, t])
        want = W.forward_multi(rw_oracle, st, toks[:, t])
        assert np.array_equal(bits(got), bits(want)), t
    # device-side periodic reset every 3 tokens vs the oracle's counter
    b.batch_reset()
    b.set_reset_every(3)
    try:
        st = [W.State(rw_oracle) for _ in range(3)]
        for s in st:
            s.set_reset_every(3)
        for t in range(8):
            got = b.forward_batch(slots, toks[:, t])
            want = W.forward_multi(rw_oracle, st, toks[:, t])
            assert np.array_equal(bits(got), bits(want)), t
    finally:
        b.set_reset_every(0)


def test_invalid_arguments_change_nothing(rw_small):
    b = shared_backend(rw_small)
    b.batch_init(4)
    V = b.vocab_size
    out = np.zeros((2, V), np.float32)
    slots = np.array([0, 0], np.uint32)
    assert b.forward_batch_raw(slots, np.array([1, 2], np.uint32), out) == BackendResult.INVALID_ARGUMENT
    assert b.forward_batch_raw(np.array([0, 1], np.uint32), np.array([1, V], np.uint32), out) == \
        BackendResult.INVALID_ARGUMENT
    xa, wkv, xf, vf = b.rwkv_state(0)
    assert not wkv.any() and not xa.any()


def test_probs_match_oracle_softmax(rw_small, rw_oracle):
    b = shared_backend(rw_small)
    b.batch_init(4)
    toks = R.byte_tokens(3, 3, seed=21)
    st = [W.State(rw_oracle) for _ in range(3)]
    for t in range(3):
        p = b.forward_batch_probs([0, 1, 2], toks[:, t])
        lg = W.forward_multi(rw_oracle, st, toks[:, t])
        for s in range(3):
            want = O.softmax(lg[s])
            assert np.max(np.abs(p[s] - want)) <= 1e-6 * max(1.0, float(want.max()))
            assert abs(float(p[s].sum(dtype=np.float64)) - 1.0) < 1e-4


def test_device_path_equals_host_path(rw_small):
    torch = pytest.importorskip("torch")
    b = shared_backend(rw_small)
    n, steps = 5, 3
    toks = R.byte_tokens(n, steps, seed=31)
    b.batch_init(8)
    host = run_gpu(b, list(range(n)), toks)
    b.batch_reset()
    dev = torch.device("cuda:0")
    d_slots = torch.arange(n, dtype=torch.int32, device=dev)
    d_tok = torch.empty(n, dtype=torch.int32, device=dev)
    d_out = torch.empty((n, b.vocab_size), dtype=torch.float32, device=dev)
    for t in range(steps):
        d_tok.copy_(torch.from_numpy(toks[:, t].astype(np.int32)))
        b.forward_batch_device(n, d_slots.data_ptr(), d_tok.data_ptr(), d_out.data_ptr())
        torch.cuda.synchronize()
        assert np.array_equal(bits(d_out.cpu().numpy()), bits(host[:, t])), t
    assert b.device_error() == 0


@pytest.mark.slow
def test_rwkv7_0_1b_bit_identical(model_dir):
    path = R.ensure_model(os.path.join(model_dir, "rwkv7_0_1b.rbin"), R.RWKV7_0_1B)
    m = W.Model(path)
    b = shared_backend(path)
    for n in (3, 20):
        toks = R.byte_tokens(n, 2, seed=3)
        want, _ = run_oracle(m, toks)
        b.batch_init(32)
        got = run_gpu(b, list(range(n)), toks)
        assert np.array_equal(bits(got), bits(want)), n
