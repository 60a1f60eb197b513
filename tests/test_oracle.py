"""The CPU oracle pinned against the reference: its known-value tests, its invariants and the
golden logits of the reference's own NumPy Mamba (tests/golden)."""
import os
import subprocess
import sys

import numpy as np
import pytest

import golden_cases
from conftest import max_dlogp
from oracle import oracle as O


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_expf_known_values():
    # src/domain/tensor.rs:2896-2911 (portable_expf_known_values)
    assert O.expf(0.0) == 1.0
    for x in (1.0, -1.0, -87.0, 88.0):
        want = np.exp(np.float64(x))
        assert abs(O.expf(x) - want) / want < 1e-6, x


def test_lnf_known_values():
    # src/domain/tensor.rs:2913-2930 (portable_lnf_known_values)
    assert O.lnf(1.0) == 0.0
    for x in (np.e, 0.5, 10.0, 1e-10):
        want = np.log(np.float64(np.float32(x)))
        tol = abs(want) * 1e-6 if abs(want) > 1.0 else 1e-6
        assert abs(O.lnf(float(np.float32(x))) - want) < tol, x
    assert O.lnf(0.0) == -np.inf
    assert np.isnan(O.lnf(-1.0))


def test_softplus_threshold_and_values():
    assert O.softplus(25.0) == 25.0
    for x in (-10.0, -1.0, 0.0, 1.0, 5.0, 19.5):
        assert abs(O.softplus(x) - np.log1p(np.exp(x))) < 2e-6 * max(1.0, abs(x)), x


def test_q8_quantizer_error_bound_and_per_row_fallback():
    # Q8 error <= scale/2 per element (src/domain/gemv.rs:678-697,741-760)
    rng = np.random.default_rng(5)
    w = rng.standard_normal((37, 256)).astype(np.float32)
    for group in (64, 0):
        q, s = O.q8_quantize(w, group)
        g = 64 if group else 256
        deq = q.astype(np.float32) * np.repeat(s, g, axis=1)
        step = np.repeat(s, g, axis=1)
        assert np.all(np.abs(w - deq) <= step / 2 + 1e-6 * np.abs(w))
        assert np.abs(q).max() <= 127
    # a group that does not divide the columns falls back to per-row (gemv.rs:259)
    q, s = O.q8_quantize(w[:, :200], 64)
    assert s.shape == (37, 1)
    z = np.zeros((2, 64), np.float32)
    q, s = O.q8_quantize(z, 64)
    assert np.all(q == 0) and np.all(s == 1.0)


def test_gemv_kernels_match_float64():
    rng = np.random.default_rng(9)
    m = rng.standard_normal((300, 771)).astype(np.float32)
    v = rng.standard_normal(771).astype(np.float32)
    got = O.gemv_f32(m, v)
    assert np.allclose(got, m.astype(np.float64) @ v, rtol=1e-4, atol=1e-4)
    q, s = O.q8_quantize(m[:, :768], 64)
    got = O.gemv_q8(q, s, v[:768], 64)
    deq = q.astype(np.float64) * np.repeat(s, 64, axis=1)
    assert np.allclose(got, deq @ v[:768].astype(np.float64), rtol=1e-4, atol=1e-4)


def test_scalar_and_avx2_tiers_bit_identical(ref_test_rbin):
    outs = []
    for simd in (False, True):
        O.set_simd(simd)
        m = O.Model(ref_test_rbin, O.PROFILE_Q8)
        st = m.new_state()
        outs.append(np.stack([m.forward((t * 977 + 7) % m.vocab, st) for t in range(4)]))
    O.set_simd(True)
    assert np.array_equal(bits(outs[0]), bits(outs[1]))


@pytest.mark.parametrize("profile", [O.PROFILE_F32, O.PROFILE_Q8])
@pytest.mark.parametrize("n", [2, 3, 5, 9])
def test_lockstep_bit_identical_to_single_stream(ref_test_rbin, profile, n):
    # forward_multi_bit_identical_to_single_stream (src/infrastructure/mamba/model.rs:1091-1134)
    m = O.Model(ref_test_rbin, profile)
    v, steps = m.vocab, 6
    toks = np.array([[(s * 131 + t * 977 + 7) % v for t in range(steps)] for s in range(n)])
    ref_logits, ref_states = [], []
    for s in range(n):
        st = m.new_state()
        for t in range(steps):
            lg = m.forward(int(toks[s, t]), st)
        ref_logits.append(lg)
        ref_states.append(st.export())
    states = [m.new_state() for _ in range(n)]
    for t in range(steps):
        out = m.forward_multi(toks[:, t].tolist(), states)
    for s in range(n):
        assert np.array_equal(bits(out[s]), bits(ref_logits[s]))
        c, ss = states[s].export()
        assert np.array_equal(bits(c), bits(ref_states[s][0]))
        assert np.array_equal(bits(ss), bits(ref_states[s][1]))


def test_periodic_reset_matches_fresh_state(ref_test_rbin):
    # maybe_periodic_reset (model.rs:315-320): with reset_every = k, forward k+1 starts from zero
    m = O.Model(ref_test_rbin, O.PROFILE_F32)
    k = 3
    st = m.new_state(k)
    toks = [5, 9, 13, 17, 21]
    out = [m.forward(t, st) for t in toks]
    fresh = m.new_state()
    assert np.array_equal(bits(out[3]), bits(m.forward(toks[3], fresh)))
    assert not np.array_equal(bits(out[1]), bits(m.forward(toks[1], m.new_state())))


def test_thread_count_does_not_change_bits(ref_test_rbin):
    code = f"""
import sys, numpy as np
sys.path.insert(0, {os.path.dirname(os.path.dirname(os.path.abspath(__file__)))!r})
from oracle import oracle as O
O.set_threads(int(sys.argv[1]))
m = O.Model({ref_test_rbin!r}, O.PROFILE_Q8)
sts = [m.new_state() for _ in range(4)]
for t in range(3):
    out = m.forward_multi([(s*131 + t*977 + 7) % m.vocab for s in range(4)], sts)
import hashlib; sys.stdout.write(hashlib.sha256(out.tobytes()).hexdigest())
"""
    outs = [subprocess.run([sys.executable, "-c", code, str(t)], capture_output=True, text=True, check=True).stdout
            for t in (1, 3)]
    assert outs[0] == outs[1]


@pytest.mark.parametrize("name", golden_cases.NAMES)
def test_oracle_matches_reference_numpy_golden(name, model_dir):
    path, toks, golden = golden_cases.load(name, model_dir)
    m = O.Model(path, O.PROFILE_F32)
    st = m.new_state()
    got = np.stack([m.forward(int(t), st) for t in toks])
    rel = np.max(np.abs(got - golden)) / np.max(np.abs(golden))
    assert rel < 1e-4, rel  # the reference's own bar for its GPU plugin is 1e-3 (notebook :254-270)
    assert max_dlogp(got, golden) < 1e-4


def test_softmax_matches_float64():
    rng = np.random.default_rng(1)
    x = (rng.standard_normal(5000) * 3).astype(np.float32)
    p = O.softmax(x)
    ref = np.exp(x.astype(np.float64) - x.max())
    ref /= ref.sum()
    assert np.allclose(p, ref, rtol=1e-5, atol=1e-9)
    assert np.allclose(O.softmax(np.full(7, -np.inf, np.float32)), 1.0 / 7)
