"""RWKV-7 CPU oracle (oracle/rwkv7_oracle.c) against the reference's own helper tests and an
independent float64 NumPy restatement of `Rwkv7Model::forward_into` (rwkv7/model.rs:643-925).

The reference ships no RWKV-7 logits goldens (its RWKV tests need the real checkpoint), so the
whole-step values are pinned by restatement only; the element-wise helpers are pinned by the
accuracy bounds of the reference's tests (src/domain/tensor.rs:2392-2497).
"""
import hashlib
import os

import numpy as np
import pytest

from oracle import oracle as O
from oracle import rwkv7 as W
from redukt_b200 import rwkv7_rbin as R


@pytest.fixture(scope="session")
def rw_small(model_dir):
    return R.ensure_model(os.path.join(model_dir, "rwkv7_small.rbin"), R.RWKV7_TEST_DIMS)


# ---- file format ----------------------------------------------------------------------------------

def test_rbin_header_and_layout(rw_small):
    dims = R.read_header(rw_small)
    assert dims == R.RWKV7_TEST_DIMS
    assert os.path.getsize(rw_small) == R.file_bytes(dims)
    d2, arrays = R.read_arrays(rw_small)
    assert arrays["layers.1.ffn_value"].shape == (dims.d_model, dims.d_ffn)
    assert arrays["layers.0.g2"].shape == (dims.d_model, dims.lora_g)
    # decay bias: decay exp(-0.606531 sigmoid(w0)) in [0.9, 0.999] before the LoRA term
    w0 = arrays["layers.0.w0"].astype(np.float64)
    decay = np.exp(-0.606531 / (1.0 + np.exp(-w0)))
    assert decay.min() >= 0.9 - 1e-6 and decay.max() <= 0.999 + 1e-6


def test_full_size_layout_bytes():
    d = R.RWKV7_0_1B
    # 2 x (65536 x 768) embedding/head + 12 layers of 4 d^2 + 2 d d_ffn + LoRAs + vectors
    per_layer = 10 * 768 + 3 * 768 + 2 * 288 * 768 + 3 * 768 + 4 * 768 * 768 + 3 * 768 + 2 * 3072 * 768
    assert R.file_bytes(d) == 76 + 4 * (2 * 65536 * 768 + 4 * 768 + 12 * per_layer)
    assert d.n_head == 12 and d.state_floats() == 12 * (2 * 768 + 12 * 64 * 64) + 768


def test_reference_plugin_header_check_rejects_rwkv(rw_small):
    # the reference plugin accepts .rbin versions 1 and 2 only (mamba_cuda.cu:472)
    with open(rw_small, "rb") as f:
        words = np.frombuffer(f.read(8), "<u4")
    assert words[1] == 3


# ---- element-wise helpers: the reference's accuracy tests (tensor.rs:2392-2497) -------------------

def _sig64(x):
    return 1.0 / (1.0 + np.exp(-np.asarray(x, np.float64)))


def test_tanh_accuracy_and_boundaries():
    x = (np.arange(-40, 41) * 0.25).astype(np.float32)
    assert np.max(np.abs(W.tanh(x) - np.tanh(x.astype(np.float64)))) < 5e-7
    b = np.array([-100, -50, -10, -1, 0, 1, 10, 50, 100, 0.5], np.float32)  # 10 values: tail of 2
    assert np.max(np.abs(W.tanh(b) - np.tanh(b.astype(np.float64)))) < 5e-7


def test_sigmoid_family_accuracy():
    i = np.arange(768, dtype=np.float32)
    base = (np.sin(i * np.float32(0.013)) * 4.0).astype(np.float32)
    off = (np.cos(i * np.float32(0.007)) * 3.0).astype(np.float32)
    s = base.astype(np.float64) + off
    assert np.max(np.abs(W.sigmoid_add(base, off) - _sig64(s))) < 2e-7
    assert np.max(np.abs(W.decay_sigmoid(base, off) - np.exp(-0.606531 * _sig64(s)))) < 5e-7
    vf = (np.sin(i * np.float32(0.019)) * 2.0).astype(np.float32)
    v0 = (np.cos(i * np.float32(0.011)) * 1.5).astype(np.float32)
    want = v0 + (vf.astype(np.float64) - v0) * _sig64(s)
    assert np.max(np.abs(W.sigmoid_mix(v0, vf, base, off) - want)) < 5e-7
    assert np.max(np.abs(W.sigmoid(base) - _sig64(base))) < 2e-7


def test_lane_and_portable_tail_agree_closely():
    # body uses the lane functions, the len % 8 tail the portable ones (tensor.rs:1016-1020)
    x = np.linspace(-6, 6, 13).astype(np.float32)
    full = W.sigmoid(x)
    for k in range(13):
        assert abs(W.sigmoid(x[k:k + 1])[0] - full[k]) <= 2e-7


# ---- W8A8 -----------------------------------------------------------------------------------------

def _round_half_away(x32: np.ndarray) -> np.ndarray:
    x = x32.astype(np.float64)  # adding 0.5 to an f32 value is exact in f64
    return np.trunc(x + np.copysign(0.5, x))


def _np_q8_rows(w: np.ndarray):
    w = w.astype(np.float32)
    amax = np.max(np.abs(w), axis=1)
    scale = np.where(amax > 0, amax / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    inv = (np.float32(1.0) / scale).astype(np.float32)
    q = np.clip(_round_half_away((w * inv[:, None]).astype(np.float32)), -127, 127).astype(np.int8)
    return q, scale


def test_q8_quantize_rows_matches_restatement():
    rng = np.random.default_rng(7)
    w = rng.standard_normal((37, 200)).astype(np.float32) * np.float32(0.05)
    w[3] = 0.0  # zero row: scale 1
    w[5, 7] = np.float32(0.5) * (np.max(np.abs(w[5])) / np.float32(127.0))  # exact half step
    q, s = W.q8_quantize_rows(w)
    q2, s2 = _np_q8_rows(w)
    assert np.array_equal(q, q2) and np.array_equal(s, s2)
    assert s[3] == 1.0


def test_w8a8_gemv_is_the_exact_int_dot():
    rng = np.random.default_rng(8)
    w = rng.standard_normal((64, 256)).astype(np.float32)
    v = rng.standard_normal(256).astype(np.float32)
    q, s = W.q8_quantize_rows(w)
    vq, vs = W.quantize_vec(v)
    dots = q.astype(np.int64) @ vq.astype(np.int64)
    want = (dots.astype(np.float32) * (s * vs).astype(np.float32)).astype(np.float32)
    assert np.array_equal(W.gemv_w8a8(q, s, v), want)
    # W8A8 error against f32: a few quantisation steps of the largest products
    exact = w.astype(np.float64) @ v
    assert np.max(np.abs(want - exact)) < 0.03 * np.max(np.abs(exact))


# ---- whole step -----------------------------------------------------------------------------------

def _run(model, tokens_by_stream):
    states = [W.State(model) for _ in tokens_by_stream]
    outs = []
    for t in range(len(tokens_by_stream[0])):
        outs.append(W.forward_multi(model, states, [tk[t] for tk in tokens_by_stream]))
    return np.stack(outs, 1), states


def test_forward_multi_equals_single_stream_bits(rw_small):
    m = W.Model(rw_small)
    toks = R.byte_tokens(3, 6)
    multi, _ = _run(m, toks.tolist())
    for b in range(3):
        st = W.State(m)
        for t in range(6):
            assert np.array_equal(st.forward(int(toks[b, t])), multi[b, t])


def test_thread_count_does_not_change_bits(rw_small):
    m = W.Model(rw_small)
    toks = R.byte_tokens(5, 4).tolist()
    old = O.get_threads()
    try:
        O.set_threads(1)
        a, _ = _run(m, toks)
        O.set_threads(4)
        b, _ = _run(m, toks)
    finally:
        O.set_threads(old)
    assert hashlib.sha256(a.tobytes()).hexdigest() == hashlib.sha256(b.tobytes()).hexdigest()


def test_simd_tiers_agree(rw_small):
    m = W.Model(rw_small)
    toks = R.byte_tokens(2, 4).tolist()
    try:
        O.set_simd(False)
        a, _ = _run(m, toks)
        O.set_simd(True)
        b, _ = _run(m, toks)
    finally:
        O.set_simd(True)
    assert np.array_equal(a, b)


def test_reset_and_periodic_reset(rw_small):
    m = W.Model(rw_small)
    toks = [5, 9, 200, 31, 7, 7, 100]
    s = W.State(m)
    for t in toks[:4]:
        s.forward(t)
    s.reset()
    fresh = W.State(m)
    assert np.array_equal(s.forward(toks[4]), fresh.forward(toks[4]))
    xa, wkv, xf, vf = s.export()
    assert np.abs(wkv).max() > 0 and np.abs(vf).max() > 0
    # periodic: reset before the token once `since` reached the period (mamba/model.rs:315-320)
    p = W.State(m)
    p.set_reset_every(3)
    out_p = [p.forward(t) for t in toks]
    q = W.State(m)
    out_q = []
    for i, t in enumerate(toks):
        if i and i % 3 == 0:
            q.reset()
        out_q.append(q.forward(t))
    assert all(np.array_equal(a, b) for a, b in zip(out_p, out_q))


class NumpyRwkv7:
    """float64 restatement of model.rs:643-925 with the W8A8 quantisation steps in f32."""

    def __init__(self, path):
        self.d, A = R.read_arrays(path)
        d = self.d
        self.A = A
        e = A["emb"].astype(np.float64)
        self.emb = self._ln(e, A["ln0_w"], A["ln0_b"], 1e-5)
        self.q = {}
        for k, v in A.items():
            if k == "head" or k.rsplit(".", 1)[-1] in ("receptance", "key", "value", "output", "ffn_key", "ffn_value"):
                self.q[k] = _np_q8_rows(v)
        L, D, H = d.n_layer, d.d_model, d.n_head
        self.state = [np.zeros((H, 64, 64)) for _ in range(L)]
        self.xa = [np.zeros(D) for _ in range(L)]
        self.xf = [np.zeros(D) for _ in range(L)]
        self.vfirst = np.zeros(D)

    @staticmethod
    def _ln(x, w, b, eps):
        m = x.mean(-1, keepdims=True)
        v = ((x - m) ** 2).mean(-1, keepdims=True)
        return (x - m) / np.sqrt(v + eps) * w + b

    def _w8(self, name, x):
        q, s = self.q[name]
        x32 = x.astype(np.float32)
        amax = np.float32(np.max(np.abs(x32)))
        vs = amax / np.float32(127.0) if amax > 0 else np.float32(1.0)
        vq = np.clip(_round_half_away((x32 * (np.float32(1.0) / vs)).astype(np.float32)), -127, 127)
        return (q.astype(np.float64) @ vq) * (s.astype(np.float64) * np.float64(vs))

    def step(self, tok):
        A, d = self.A, self.d
        H, N = d.n_head, 64
        sig = lambda z: 1.0 / (1.0 + np.exp(-z))
        x = self.emb[tok].copy()
        for l in range(d.n_layer):
            p = f"layers.{l}."
            f = lambda k: A[p + k].astype(np.float64)
            ln = self._ln(x, f("ln1_w"), f("ln1_b"), 1e-5)
            xx = self.xa[l] - ln
            mix = {k: ln + xx * f(k) for k in ("x_r", "x_w", "x_k", "x_v", "x_a", "x_g")}
            r = self._w8(p + "receptance", mix["x_r"])
            k = self._w8(p + "key", mix["x_k"])
            v = self._w8(p + "value", mix["x_v"])
            w = np.exp(-0.606531 * sig(f("w0") + f("w2") @ np.tanh(f("w1") @ mix["x_w"])))
            a = sig(f("a0") + f("a2") @ (f("a1") @ mix["x_a"]))
            g = f("g2") @ sig(f("g1") @ mix["x_g"])
            kk = (k * f("k_k")).reshape(H, N)
            nrm = np.linalg.norm(kk, axis=1, keepdims=True)
            kk = (kk / np.where(nrm > 1e-12, nrm, np.inf)).reshape(-1)
            kmod = k * (1 + (a - 1) * f("k_a"))
            vout = v.copy()
            if l:
                vout = v + (self.vfirst - v) * sig(f("v0") + f("v2") @ (f("v1") @ mix["x_v"]))
            out = np.zeros(d.d_model)
            for h in range(H):
                sl = slice(h * N, (h + 1) * N)
                S = self.state[l][h]
                S = S * w[sl][None, :] + np.outer(S @ -kk[sl], kk[sl] * a[sl]) + np.outer(vout[sl], kmod[sl])
                self.state[l][h] = S
                out[sl] = S @ r[sl]
            on = self._ln(out.reshape(H, N), f("ln_x_w").reshape(H, N), f("ln_x_b").reshape(H, N), 64e-5).reshape(-1)
            bonus = (r * k * f("r_k")).reshape(H, N).sum(1)
            on = on + np.repeat(bonus, N) * vout
            tm = self._w8(p + "output", on * g)
            self.xa[l] = ln
            if l == 0:
                self.vfirst = v
            x = x + tm
            ln2 = self._ln(x, f("ln2_w"), f("ln2_b"), 1e-5)
            xk = ln2 + (self.xf[l] - ln2) * f("ffn_x_k")
            hdn = np.maximum(self._w8(p + "ffn_key", xk), 0.0) ** 2
            x = x + self._w8(p + "ffn_value", hdn)
            self.xf[l] = ln2
        return self._w8("head", self._ln(x, A["ln_out_w"], A["ln_out_b"], 1e-5))


def test_oracle_agrees_with_float64_restatement(rw_small):
    m = W.Model(rw_small)
    st = W.State(m)
    ref = NumpyRwkv7(rw_small)
    worst = 0.0
    for tok in [3, 250, 17, 17, 99, 0, 255, 42]:
        a = st.forward(tok).astype(np.float64)
        b = ref.step(tok)
        worst = max(worst, float(np.max(np.abs(a - b)) / np.max(np.abs(b))))
    # f32 vs f64 arithmetic plus occasional int8 rounding flips of the activations
    assert worst < 2e-3, worst
    xa, wkv, xf, vf = st.export()
    assert np.allclose(wkv, np.stack(ref.state), rtol=2e-3, atol=2e-3 * np.abs(wkv).max())
