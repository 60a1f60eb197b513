"""GPU parity of libredukt_gpu.so against the CPU oracle, through the C ABI.

Mirrors the reference's GPU validation (notebooks/redukt-gpu-cuda-test.py:254-289): v1 vs a CPU
reference, v1 == forward_batch bits with the stream in an arbitrary slot, reset-then-step0, duplicate
slot rejection; plus the reference's lockstep test (src/infrastructure/mamba/model.rs:1091-1134):
every stream of a batch is bit-identical to the same stream run alone, for every batch size.
Tolerance against the oracle: max |delta log p| <= 1e-3 nats per token (the engine's parity bar).
"""
import numpy as np
import pytest

from conftest import logsoftmax64, max_dlogp, q8, shared_backend
from oracle import oracle as O
from redukt_b200.plugin import BackendResult, PluginBackend
from redukt_b200.workload import zipf_tokens

pytestmark = pytest.mark.gpu

TOL_NATS = 1e-3

def backend(path):
    """The plugin is a process-global singleton: re-init only when the model changes."""
    return shared_backend(path)


def oracle_model(path, profile):
    return O.Model(path, profile, 64)


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


@pytest.mark.parametrize("quant", ["f32", "q8"])
def test_v1_matches_oracle_reference_test_model(ref_test_rbin, quant):
    path = ref_test_rbin if quant == "f32" else q8(ref_test_rbin)
    b = backend(path)
    m = oracle_model(path, O.PROFILE_F32 if quant == "f32" else O.PROFILE_Q8)
    st = m.new_state()
    b.reset_state()
    worst = 0.0
    for t in range(12):
        tok = (t * 977 + 7) % m.vocab
        g = b.forward(tok)
        r = m.forward(tok, st)
        worst = max(worst, max_dlogp(g, r))
    assert worst <= TOL_NATS, worst


@pytest.mark.parametrize("quant", ["f32", "q8"])
def test_batch_bit_identical_to_v1_every_batch_size(ref_test_rbin, quant):
    path = ref_test_rbin if quant == "f32" else q8(ref_test_rbin)
    b = backend(path)
    V = b.vocab_size
    steps = 6
    nmax = 17
    toks = np.array([[(s * 131 + t * 977 + 7) % V for t in range(steps)] for s in range(nmax)], np.uint32)
    # each stream alone through v1
    single = np.empty((nmax, steps, V), np.float32)
    for s in range(nmax):
        b.reset_state()
        for t in range(steps):
            single[s, t] = b.forward(int(toks[s, t]))
    for n in (1, 2, 3, 5, 9, 17):
        b.batch_init(32)
        slots = [(7 * s + 3) % 32 for s in range(n)]  # arbitrary distinct slots
        for t in range(steps):
            out = b.forward_batch(slots, toks[:n, t])
            for s in range(n):
                assert np.array_equal(bits(out[s]), bits(single[s, t])), (quant, n, s, t)


@pytest.mark.parametrize("quant", ["f32", "q8"])
@pytest.mark.parametrize("model", ["reftest", "gauss_small"])
def test_large_batches_bit_identical_to_small(ref_test_rbin, small_gauss_rbin, model, quant):
    """Large batches take other launch shapes (several streams per scan CTA, other projection
    tiles): every stream still reproduces the bits of the same stream in a batch of four, with
    slot resets in the middle of the window.  The two models cover a channel count that is not a
    multiple of the scan's 256-channel CTA and dt ranks below and at one 8-lane body."""
    base = ref_test_rbin if model == "reftest" else small_gauss_rbin
    path = base if quant == "f32" else q8(base)
    b = backend(path)
    V = b.vocab_size
    steps = 4
    for n in (70, 300, 517):
        toks = zipf_tokens(n, steps, vocab=V, seed_base=n)
        cap = n + 3
        slots = [(7 * s + 1) % cap for s in range(n)]
        reset_at = {s for s in range(n) if s % 5 == 2}
        b.batch_init(cap)
        full = []
        for t in range(steps):
            if t == 2:
                b.batch_reset([slots[s] for s in sorted(reset_at)])
            full.append(b.forward_batch(slots, toks[:, t]).copy())
        sub = [0, 2, n // 2, n - 1]
        b.batch_init(8)
        for t in range(steps):
            if t == 2:
                b.batch_reset([i for i, s in enumerate(sub) if s in reset_at])
            out = b.forward_batch(list(range(len(sub))), toks[sub, t])
            for i, s in enumerate(sub):
                assert np.array_equal(bits(out[i]), bits(full[t][s])), (model, quant, n, s, t)


def test_reset_then_step0_and_invalid_arguments(ref_test_rbin):
    b = backend(ref_test_rbin)
    V = b.vocab_size
    b.batch_init(8)
    first = b.forward_batch([5], [11])[0].copy()
    b.forward_batch([5], [12])
    b.batch_reset([5])
    again = b.forward_batch([5], [11])[0]
    assert np.array_equal(bits(first), bits(again))
    # duplicate slot, slot out of range, token out of range, vocab mismatch: rejected, no state change
    out = np.zeros((2, V), np.float32)
    assert b.forward_batch_raw(np.array([1, 1], np.uint32), np.array([0, 0], np.uint32), out) == BackendResult.INVALID_ARGUMENT
    assert b.forward_batch_raw(np.array([8], np.uint32), np.array([0], np.uint32), out[:1]) == BackendResult.INVALID_ARGUMENT
    assert b.forward_batch_raw(np.array([0], np.uint32), np.array([V], np.uint32), out[:1]) == BackendResult.INVALID_ARGUMENT
    c_before, s_before = b.get_state(5)
    rc = b.lib.redukt_backend_forward_batch(1, None, None, None, V)
    assert rc == BackendResult.INVALID_ARGUMENT
    c_after, s_after = b.get_state(5)
    assert np.array_equal(c_before, c_after) and np.array_equal(s_before, s_after)
    assert b.lib.redukt_backend_batch_init(4097) == BackendResult.INVALID_ARGUMENT


@pytest.mark.parametrize("quant", ["f32", "q8"])
def test_state_matches_oracle(small_gauss_rbin, quant):
    path = small_gauss_rbin if quant == "f32" else q8(small_gauss_rbin)
    b = backend(path)
    m = oracle_model(path, O.PROFILE_F32 if quant == "f32" else O.PROFILE_Q8)
    b.batch_init(4)
    toks = zipf_tokens(3, 10, vocab=m.vocab)
    states = [m.new_state() for _ in range(3)]
    worst = 0.0
    for t in range(10):
        g = b.forward_batch([0, 2, 3], toks[:, t])
        r = m.forward_multi(toks[:, t].tolist(), states)
        worst = max(worst, max_dlogp(g, r))
    assert worst <= TOL_NATS
    conv_g, ssm_g = b.get_state(2)
    conv_r, ssm_r = states[1].export()
    assert np.allclose(conv_g, conv_r, rtol=1e-3, atol=1e-5)
    assert np.allclose(ssm_g, ssm_r, rtol=1e-3, atol=1e-5)


@pytest.mark.parametrize("per_row", [False, True])
def test_q8_weights_bit_exact_with_reference_quantizer(small_gauss_rbin, per_row):
    path = q8(small_gauss_rbin, per_row)
    b = backend(path)
    m = O.Model(path, O.PROFILE_Q8, 0 if per_row else 64)
    for which, layer in (("emb", 0), ("in_proj", 1), ("out_proj", 2)):
        qg, sg = b.get_q8(which, layer)
        qr, sr = m.q8(which, layer)
        assert np.array_equal(qg, qr), which
        if per_row:
            assert np.array_equal(bits(sg), bits(np.repeat(sr, sg.shape[1], axis=1))), which
        else:
            assert np.array_equal(bits(sg), bits(sr)), which


def test_device_periodic_reset_matches_oracle(ref_test_rbin):
    b = backend(ref_test_rbin)
    m = oracle_model(ref_test_rbin, O.PROFILE_F32)
    every = 3
    b.batch_init(4)
    b.set_reset_every(every)
    try:
        states = [m.new_state(every) for _ in range(2)]
        toks = zipf_tokens(2, 10, vocab=m.vocab, seed_base=99)
        for t in range(10):
            g = b.forward_batch([1, 3], toks[:, t])
            r = m.forward_multi(toks[:, t].tolist(), states)
            assert max_dlogp(g, r) <= TOL_NATS, t
        # device reset == host-driven reset (PluginState::tick) bit for bit
        b.batch_init(4)
        b.set_reset_every(0)
        host = []
        since = 0
        for t in range(10):
            if since >= every:
                b.batch_reset([1])
                since = 0
            since += 1
            host.append(b.forward_batch([1], toks[:1, t])[0].copy())
        b.batch_init(4)
        b.set_reset_every(every)
        for t in range(10):
            dev = b.forward_batch([1], toks[:1, t])[0]
            assert np.array_equal(bits(dev), bits(host[t])), t
    finally:
        b.set_reset_every(0)


def test_probs_match_softmax_of_logits(ref_test_rbin):
    b = backend(ref_test_rbin)
    b.batch_init(4)
    lg = b.forward_batch([0, 1], [3, 4])
    b.batch_reset(None)
    pr = b.forward_batch_probs([0, 1], [3, 4])
    assert np.allclose(pr.sum(axis=1), 1.0, atol=1e-5)
    ref = np.stack([O.softmax(x) for x in lg])
    assert np.max(np.abs(np.log(pr.astype(np.float64)) - np.log(ref.astype(np.float64)))) < 1e-5


@pytest.mark.slow
@pytest.mark.parametrize("quant", ["q8", "f32"])
def test_mamba130m_matches_oracle(mamba130m_rbin, quant):
    path = mamba130m_rbin if quant == "f32" else q8(mamba130m_rbin)
    b = backend(path)
    m = oracle_model(path, O.PROFILE_F32 if quant == "f32" else O.PROFILE_Q8)
    n, T = 4, 6
    b.batch_init(n)
    toks = zipf_tokens(n, T)
    states = [m.new_state() for _ in range(n)]
    worst = 0.0
    for t in range(T):
        g = b.forward_batch(list(range(n)), toks[:, t])
        r = m.forward_multi(toks[:, t].tolist(), states)
        worst = max(worst, max_dlogp(g, r))
    print(f"mamba130m {quant}: max |dlogp| = {worst:.3e}")
    assert worst <= TOL_NATS


def test_reference_plugin_agrees_with_oracle(ref_test_rbin):
    """The reference's own CUDA plugin (rebuilt for sm_100a by oracle/Makefile) vs the oracle."""
    import os
    if not os.path.exists(O.REF_PLUGIN_PATH):
        pytest.skip("reference plugin not built")
    import subprocess, sys, json
    code = f"""
import sys, json, numpy as np
sys.path.insert(0, {repr(str(__import__('os').path.dirname(__import__('os').path.dirname(__file__))))})
from redukt_b200.plugin import PluginBackend, PluginLibrary
from oracle import oracle as O
from conftest import max_dlogp
b = PluginBackend({ref_test_rbin!r}, library=PluginLibrary({O.REF_PLUGIN_PATH!r}))
m = O.Model({ref_test_rbin!r}, O.PROFILE_F32)
st = m.new_state(); worst = 0.0
for t in range(8):
    tok = (t * 977 + 7) % m.vocab
    worst = max(worst, max_dlogp(b.forward(tok), m.forward(tok, st)))
print(json.dumps(worst))
"""
    env = dict(os.environ, PYTHONPATH=os.path.dirname(__file__))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    worst = json.loads(r.stdout.strip().splitlines()[-1])
    assert worst <= TOL_NATS, worst


@pytest.mark.parametrize("name", ["reftest", "gauss_small", "gauss_ln_untied"])
def test_gpu_matches_reference_numpy_golden(name, model_dir):
    """The engine against the reference's own NumPy Mamba (committed fixtures, tests/golden)."""
    import golden_cases
    path, toks, golden = golden_cases.load(name, model_dir)
    b = backend(path)
    b.reset_state()
    got = np.stack([b.forward(int(t)).copy() for t in toks])
    assert max_dlogp(got, golden) <= TOL_NATS
    rel = np.max(np.abs(got - golden)) / np.max(np.abs(golden))
    assert rel < 1e-3, rel  # the reference notebook's bar for its own plugin (max rel err < 1e-3)


@pytest.mark.parametrize("quant", ["q8", "q8row"])
def test_tensor_core_and_cuda_core_projections_bit_identical(small_gauss_rbin, mamba130m_rbin, quant):
    """The tcgen05 kind::i8 projections and the dp4a projections compute the same exact int32 digit
    sums and run the same combine: every logit and every state element must agree bit for bit."""
    for path in (q8(small_gauss_rbin, quant == "q8row"), q8(mamba130m_rbin, quant == "q8row")):
        b = backend(path)
        V = b.vocab_size
        for n in (4, 16, 17, 33, 64, 100):
            toks = zipf_tokens(n, 3, vocab=V, seed_base=7 * n)
            outs = {}
            for mode in (1, 2):
                b.set_option("proj_path", mode)
                b.batch_init(n)
                for t in range(3):
                    outs[mode] = b.forward_batch(list(range(n)), toks[:, t]).copy()
                outs[(mode, "state")] = b.get_state(n - 1)
            b.set_option("proj_path", 0)
            assert np.array_equal(bits(outs[1]), bits(outs[2])), (path, n)
            assert np.array_equal(bits(outs[(1, "state")][1]), bits(outs[(2, "state")][1])), (path, n)


@pytest.mark.parametrize("n", [1, 5, 33, 70, 300])
def test_fused_head_softmax_matches_softmax_of_logits(small_gauss_rbin, n):
    """Q8 probabilities come from the tensor-core head's own 128-row tile partials (max and sum of
    exp) plus one normalising pass; they must agree with the softmax of the same step's logits for
    every head tile shape (16-, 32- and 64-stream tiles)."""
    b = backend(q8(small_gauss_rbin))
    V = b.vocab_size
    toks = zipf_tokens(n, 2, vocab=V, seed_base=4242)
    b.batch_init(2 * n)
    a_slots, p_slots = list(range(n)), list(range(n, 2 * n))
    for t in range(2):
        lg = b.forward_batch(a_slots, toks[:, t])
        pr = b.forward_batch_probs(p_slots, toks[:, t])
        assert np.all(np.isfinite(pr))
        assert np.allclose(pr.sum(axis=1, dtype=np.float64), 1.0, atol=1e-5)
        want = np.exp(logsoftmax64(lg))
        got = pr.astype(np.float64)
        assert np.max(np.abs(np.log(got) - np.log(want))) < 1e-5, (n, t)
    assert b.device_error() == 0


def test_softmax_edge_rows_follow_softmax_into(ref_test_rbin):
    """The normalising pass keeps softmax_into's edge semantics (src/domain/tensor.rs:1917-1933):
    a row of all -inf is uniform, and a row with one finite logit puts all mass on it (the other
    entries are the reference's clamped exp of -inf, the smallest normal float, not zero), with
    the denominator max(sum, FLT_EPSILON).  Compared with the CPU restatement of softmax_into."""
    import torch
    b = backend(ref_test_rbin)
    V = 5000
    rows = np.zeros((4, V), np.float32)
    rows[0] = -np.inf                                   # all -inf: uniform
    rows[1] = -np.inf
    rows[1, 1234] = 3.0                                 # one finite logit
    rows[2] = np.random.default_rng(1).standard_normal(V).astype(np.float32) * 4
    rows[3] = -np.inf
    rows[3, :3] = [-1e30, -1e30, -1e30]                 # finite but tiny: still normalised by its own max
    d = torch.from_numpy(rows).cuda()
    o = torch.full_like(d, float("nan"))
    assert b.libobj.softmax_noalloc(d.data_ptr(), 4, V, o.data_ptr(), 0) == BackendResult.OK
    torch.cuda.synchronize()
    p = o.cpu().numpy()
    assert np.all(p[0] == np.float32(1.0) / np.float32(V))
    assert np.array_equal(p[0], O.softmax(rows[0]))
    assert p[1, 1234] == 1.0 and np.array_equal(p[1], O.softmax(rows[1]))
    for r in (2, 3):
        want = O.softmax(rows[r])
        assert np.max(np.abs(np.log(p[r].astype(np.float64)) - np.log(want.astype(np.float64)))) < 1e-5, r
    assert np.allclose(p[3, :3], 1.0 / 3, rtol=1e-6)


@pytest.mark.parametrize("quant", ["q8", "q8row"])
def test_large_batch_tile_shapes_bit_identical(small_gauss_rbin, mamba130m_rbin, quant):
    """Above 256 streams the projections run as 64-stream tiles, one CTA per SM (large_tile 0), or
    32-stream tiles, two CTAs per SM (1).  The accumulation order is the same in both: logits,
    probabilities and states agree bit for bit."""
    for path in (q8(small_gauss_rbin, quant == "q8row"), q8(mamba130m_rbin, quant == "q8row")):
        b = backend(path)
        V = b.vocab_size
        for n in (257, 300, 640):
            toks = zipf_tokens(n, 3, vocab=V, seed_base=11 * n)
            outs = {}
            try:
                for mode in (0, 1):
                    b.set_option("large_tile", mode)
                    b.batch_init(2 * n)
                    lg_slots, pr_slots = list(range(n)), list(range(n, 2 * n))
                    for t in range(3):
                        lg = b.forward_batch(lg_slots, toks[:, t]).copy()
                        pr = b.forward_batch_probs(pr_slots, toks[:, t]).copy()
                    outs[mode] = (lg, pr, b.get_state(n - 1)[1])
            finally:
                b.set_option("large_tile", 0)
            for i in range(3):
                assert np.array_equal(bits(outs[0][i]), bits(outs[1][i])), (path, n, i)
            assert b.device_error() == 0


@pytest.mark.parametrize("quant", ["f32", "q8"])
def test_conv_in_xproj_staging_bit_identical(small_gauss_rbin, mamba130m_rbin, quant):
    """conv1d + SiLU runs either in the in_proj epilogue (conv_defer 0) or in the x_proj kernel's
    staging pass (1, in_proj then stores the x-branch before the conv).  Same arithmetic on the same
    inputs: logits, conv state and SSM state agree bit for bit, also with one stream of a
    device-path step rejected (its slot untouched)."""
    import torch

    dev = torch.device("cuda:0")
    paths = [small_gauss_rbin, mamba130m_rbin]
    for path in (paths if quant == "f32" else [q8(p) for p in paths]):
        b = backend(path)
        V = b.vocab_size
        for n in (40, 130):
            toks = zipf_tokens(n, 3, vocab=V, seed_base=13 * n)
            outs = {}
            try:
                for mode in (0, 1):
                    b.set_option("conv_defer", mode)
                    b.batch_init(n)
                    slots = list(range(n))
                    b.forward_batch(slots, toks[:, 0])
                    tk = toks[:, 1].astype(np.int32).copy()
                    tk[n // 2] = V  # rejected on the device
                    d_slots = torch.tensor(slots, dtype=torch.int32, device=dev)
                    d_tok = torch.from_numpy(tk).to(dev)
                    d_out = torch.empty((n, V), dtype=torch.float32, device=dev)
                    b.forward_batch_device(n, d_slots.data_ptr(), d_tok.data_ptr(), d_out.data_ptr())
                    torch.cuda.synchronize()
                    assert b.device_error() & 1
                    lg1 = d_out.cpu().numpy()
                    lg2 = b.forward_batch(slots, toks[:, 2]).copy()
                    outs[mode] = (lg1, lg2) + tuple(b.get_state(n - 1)) + tuple(b.get_state(n // 2))
            finally:
                b.set_option("conv_defer", 1)
            for i in range(len(outs[0])):
                assert np.array_equal(bits(outs[0][i]), bits(outs[1][i])), (path, n, i)
            assert b.device_error() == 0


def test_f32_pair_gemv_bit_identical(ref_test_rbin, small_gauss_rbin):
    """From 8 streams on, the F32 projections run k_gemv_f32_p (stream pairs on packed FMAs, a
    reduce-scatter butterfly) unless option f32_pairs is 0 (k_gemv_f32).  The per-(row, stream)
    FMA chains and the butterfly tree are the same: logits and states agree bit for bit."""
    for path in (ref_test_rbin, small_gauss_rbin):
        b = backend(path)
        V = b.vocab_size
        for n in (8, 9, 40, 130):
            toks = zipf_tokens(n, 3, vocab=V, seed_base=17 * n)
            outs = {}
            try:
                for mode in (0, 1):
                    b.set_option("f32_pairs", mode)
                    b.batch_init(n)
                    for t in range(3):
                        lg = b.forward_batch(list(range(n)), toks[:, t]).copy()
                    outs[mode] = (lg,) + tuple(b.get_state(n - 1))
            finally:
                b.set_option("f32_pairs", 1)
            for i in range(len(outs[0])):
                assert np.array_equal(bits(outs[0][i]), bits(outs[1][i])), (path, n, i)


def test_head_tile_shapes_bit_identical(small_gauss_rbin, mamba130m_rbin):
    """Above 16 streams the head runs as 32-stream tiles two CTAs per SM (head_wide 1) or with
    16-stream tiles / the layer projections' tiles (0); logits and probabilities agree bit for bit."""
    for path in (q8(small_gauss_rbin), q8(mamba130m_rbin)):
        b = backend(path)
        V = b.vocab_size
        for n in (17, 32, 65, 200, 300):
            toks = zipf_tokens(n, 2, vocab=V, seed_base=19 * n)
            outs = {}
            try:
                for mode in (0, 1):
                    b.set_option("head_wide", mode)
                    b.batch_init(2 * n)
                    for t in range(2):
                        lg = b.forward_batch(list(range(n)), toks[:, t]).copy()
                        pr = b.forward_batch_probs(list(range(n, 2 * n)), toks[:, t]).copy()
                    outs[mode] = (lg, pr)
            finally:
                b.set_option("head_wide", 1)
            assert np.array_equal(bits(outs[0][0]), bits(outs[1][0])), (path, n)
            assert np.array_equal(bits(outs[0][1]), bits(outs[1][1])), (path, n)
